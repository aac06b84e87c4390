// Expert-parallel MoE dispatch / combine over NVLink peer memory (one process per GPU).
//
// The reference's FN engine runs EP with vLLM's AgRsAll2AllManager: dispatch = host-staged all-gather of the
// tokens (optionally int8-packed, flashnext/kaggle/code_dataset/fnext/base/q8_dispatch.py:58-86), combine =
// host-staged reduce-scatter (fnext/base/host_dp.py:19, q8_rs.py:27). Here both are issued from kernels as
// peer stores into symmetric buffers:
//   ep_plan     stable per-destination slot of every routed (token, k) pair (one block, deterministic order)
//   ep_push     each pair's token row is stored straight into the owner's receive buffer (peer stores) with its
//               (local expert, source pair) metadata; the last block fences at system scope and publishes the
//               per-destination count and the layer's epoch flag on every peer
//   ep_gather   the owner waits (bounded) for every source's flag, sorts the received pairs by local expert
//               (stable), gathers their rows into the grouped GEMM's token matrix and builds, for each sorted
//               row, the peer address of the source's output row (the down-projection epilogue stores there:
//               the combine's data movement is fused into the GEMM epilogue)
//   ep_done     after the down projection: system fence + per-source completion flag
//   ep_wait     the source waits (bounded) for every owner's completion flag before its weighted combine
// Every spin gives up after a time limit, writes an error code and returns (no hang on a missing peer).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp16.h>
#include <cub/block/block_scan.cuh>
#include <cstdint>

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *flag >= want (epochs only grow). False on timeout (error code recorded).
__device__ bool wait_flag(const int64_t* flag, int64_t want, int* err, int code, uint64_t limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_sys(flag) >= want) return true;
    if ((it & 63) == 63) {
      const uint64_t now = gtimer();
      if (!t0) t0 = now;
      else if (now - t0 > limit_ns) {
        atomicCAS(err, 0, code);
        return false;
      }
      __nanosleep(100);
    }
  }
}

// epoch[0] += 1 (one thread). Runs first in every EP MoE layer so a captured graph advances it on replay.
__global__ void ep_epoch_kernel(int64_t* epoch) { epoch[0] += 1; }

// Per pair: destination rank and stable slot among the pairs with that destination. One block of 1024.
__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t* ids, int P, int e_loc, int n_ranks,
                                                       int32_t* dest_slot, int32_t* dest_count) {
  __shared__ int running[64];
  __shared__ int wcnt[32][64];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x < 64) running[threadIdx.x] = 0;
  __syncthreads();
  for (int base = 0; base < P; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int o = i < P ? min(max(ids[i], 0) / e_loc, n_ranks - 1) : -1;
    for (int q = threadIdx.x; q < 32 * 64; q += blockDim.x) (&wcnt[0][0])[q] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, o);
    const int rank_w = __popc(same & ((1u << lane) - 1));
    if (i < P && rank_w == 0) wcnt[w][o] = __popc(same);
    __syncthreads();
    if (i < P) {
      int before = 0;
      for (int ww = 0; ww < w; ++ww) before += wcnt[ww][o];
      dest_slot[i] = running[o] + before + rank_w;
    }
    __syncthreads();
    if (threadIdx.x < n_ranks) {
      int tot = 0;
      for (int ww = 0; ww < 32; ++ww) tot += wcnt[ww][threadIdx.x];
      running[threadIdx.x] += tot;
    }
    __syncthreads();
  }
  if (threadIdx.x < n_ranks) dest_count[threadIdx.x] = running[threadIdx.x];
}

struct PeerTables {
  const uint64_t* xrecv;    // [n] base of each peer's receive rows  (half,  [n_src][cap][H])
  const uint64_t* meta;     // [n] base of each peer's metadata        (int2,  [n_src][cap])
  const uint64_t* counts;   // [n] base of each peer's count array      (int64, [n_src])
  const uint64_t* flags;    // [n] base of each peer's dispatch flags   (int64, [n_src])
};

// Pushes pair rows to their owners; the last block publishes counts + epoch flags. grid = ceil(P / 4), 128 thr.
__global__ void ep_push_kernel(const __half* x, const int32_t* ids, const int32_t* dest_slot,
                               const int32_t* dest_count, int P, int k, int H, int e_loc, int cap, int me,
                               int n_ranks, PeerTables pt, const int64_t* epoch, int* done_ctr, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = blockIdx.x * 4 + warp;
  if (pair < P) {
    const int e = min(max(ids[pair], 0), n_ranks * e_loc - 1);
    const int o = e / e_loc;
    const int slot = dest_slot[pair];
    if (slot < cap) {
      const int t = pair / k;
      const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(pt.xrecv[o]) + ((int64_t)me * cap + slot) * H);
      for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
      if (lane == 0) reinterpret_cast<int2*>(pt.meta[o])[(int64_t)me * cap + slot] = make_int2(e - o * e_loc, pair);
    } else if (lane == 0) {
      atomicCAS(err, 0, 6101);  // receive buffer too small: the pair is dropped, the host sees the error
    }
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = atomicAdd(done_ctr, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (last && threadIdx.x < n_ranks) {
    __threadfence_system();
    const int o = threadIdx.x;
    const int64_t ep = epoch[0];
    reinterpret_cast<int64_t*>(pt.counts[o])[me] = dest_count[o];
    __threadfence_system();
    st_release_sys(reinterpret_cast<int64_t*>(pt.flags[o]) + me, ep);
    if (threadIdx.x == 0) *done_ctr = 0;
  }
}

// Owner side: wait for every source, then sort received pairs by local expert. One block of 1024 threads.
// Writes: sorted_src [cap_total] (index into the receive rows), items (expert tiles), n_items, row_dst (peer
// address of the source's output row for every sorted row), n_rows.
__global__ void __launch_bounds__(1024) ep_gather_plan_kernel(const int64_t* flags, const int64_t* counts,
                                                              const int2* meta, int cap, int n_ranks, int e_loc,
                                                              const int64_t* epoch, const uint64_t* peer_ybuf,
                                                              int H, int n_tile, int max_items, int32_t* sorted_src,
                                                              int4* items, int32_t* n_items, int64_t* row_dst,
                                                              int32_t* n_rows, int* err, uint64_t limit_ns) {
  extern __shared__ int smi[];
  int* cnt = smi;              // [e_loc]
  int* start = cnt + e_loc;    // [e_loc]
  int* wcnt = start + e_loc;   // [32][e_loc]
  __shared__ int s_count[64], s_base[64], s_ok;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t ep = epoch[0];
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < n_ranks) {
    if (!wait_flag(flags + threadIdx.x, ep, err, 6201 + threadIdx.x, limit_ns)) s_ok = 0;
    s_count[threadIdx.x] = min((int)counts[threadIdx.x], cap);
  }
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) {
      *n_items = 0;
      *n_rows = 0;
    }
    return;
  }
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int s = 0; s < n_ranks; ++s) {
      s_base[s] = acc;
      acc += s_count[s];
    }
    *n_rows = acc;
    s_base[n_ranks] = acc;
  }
  for (int e = threadIdx.x; e < e_loc; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int total = s_base[n_ranks];
  auto src_of = [&](int i, int& s, int& slot) {
    s = 0;
    while (s + 1 < n_ranks && i >= s_base[s + 1]) ++s;
    slot = i - s_base[s];
  };
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    int s, slot;
    src_of(i, s, slot);
    atomicAdd(&cnt[min(max(meta[(int64_t)s * cap + slot].x, 0), e_loc - 1)], 1);
  }
  __syncthreads();
  {
    using Scan = cub::BlockScan<int, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    const int e = threadIdx.x;
    const int c = e < e_loc ? cnt[e] : 0;
    const int nch = (c + n_tile - 1) / n_tile;
    int row0, item0, n_it;
    Scan(tmp).ExclusiveSum(c, row0);
    __syncthreads();
    Scan(tmp).ExclusiveSum(nch, item0, n_it);
    if (e < e_loc) {
      start[e] = row0;
      for (int q = 0; q < nch; ++q)
        if (item0 + q < max_items) items[item0 + q] = make_int4(e, row0 + q * n_tile, min(n_tile, c - q * n_tile), 0);
    }
    if (threadIdx.x == 0) *n_items = min(n_it, max_items);
  }
  __syncthreads();
  for (int base = 0; base < total; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int s = 0, slot = 0, e = -1;
    int2 m = make_int2(0, 0);
    if (i < total) {
      src_of(i, s, slot);
      m = meta[(int64_t)s * cap + slot];
      e = min(max(m.x, 0), e_loc - 1);
    }
    for (int q = threadIdx.x; q < 32 * e_loc; q += blockDim.x) wcnt[q] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(same & ((1u << lane) - 1));
    if (i < total && rank_w == 0) wcnt[w * e_loc + e] = __popc(same);
    __syncthreads();
    if (i < total) {
      int before = 0;
      for (int ww = 0; ww < w; ++ww) before += wcnt[ww * e_loc + e];
      const int pos = start[e] + before + rank_w;
      sorted_src[pos] = s * cap + slot;
      row_dst[pos] = (int64_t)(peer_ybuf[s] + (uint64_t)m.y * H * sizeof(float));
    }
    __syncthreads();
    for (int q = threadIdx.x; q < e_loc; q += blockDim.x) {
      int tot = 0;
      for (int ww = 0; ww < 32; ++ww) tot += wcnt[ww * e_loc + q];
      start[q] += tot;
    }
    __syncthreads();
  }
}

// xs[i] = xrecv[sorted_src[i]] for i < n_rows (grid-stride over rows).
__global__ void ep_gather_rows_kernel(const uint4* xrecv, const int32_t* sorted_src, const int32_t* n_rows, uint4* xs,
                                      int row_vec) {
  const int n = *n_rows;
  for (int i = blockIdx.x; i < n; i += gridDim.x) {
    const int src = sorted_src[i];
    for (int c = threadIdx.x; c < row_vec; c += blockDim.x) xs[(int64_t)i * row_vec + c] = xrecv[(int64_t)src * row_vec + c];
  }
}

// After the down projection stored every output row at its source: fence, then flag each source.
__global__ void ep_done_kernel(const uint64_t* peer_done, int me, int n_ranks, const int64_t* epoch) {
  __threadfence_system();
  if ((int)threadIdx.x < n_ranks) st_release_sys(reinterpret_cast<int64_t*>(peer_done[threadIdx.x]) + me, epoch[0]);
}

// Source side: wait until every owner has stored this layer's outputs.
__global__ void ep_wait_done_kernel(const int64_t* done, int n_ranks, const int64_t* epoch, int* err,
                                    uint64_t limit_ns) {
  if ((int)threadIdx.x < n_ranks) wait_flag(done + threadIdx.x, epoch[0], err, 6301 + threadIdx.x, limit_ns);
}

// ------------------------------------------------------------------------------------------ bindings
void ep_epoch(torch::Tensor epoch) { ep_epoch_kernel<<<1, 1, 0, STREAM>>>(epoch.data_ptr<int64_t>()); }

void ep_plan(torch::Tensor ids, int64_t e_loc, int64_t n_ranks, torch::Tensor dest_slot, torch::Tensor dest_count) {
  TORCH_CHECK(n_ranks <= 64);
  ep_plan_kernel<<<1, 1024, 0, STREAM>>>(ids.data_ptr<int32_t>(), ids.numel(), e_loc, n_ranks,
                                         dest_slot.data_ptr<int32_t>(), dest_count.data_ptr<int32_t>());
}

void ep_push(torch::Tensor x, torch::Tensor ids, torch::Tensor dest_slot, torch::Tensor dest_count, int64_t k,
             int64_t e_loc, int64_t cap, int64_t me, int64_t n_ranks, torch::Tensor xrecv_ptrs, torch::Tensor meta_ptrs,
             torch::Tensor count_ptrs, torch::Tensor flag_ptrs, torch::Tensor epoch, torch::Tensor done_ctr,
             torch::Tensor err) {
  const int P = ids.numel(), H = x.size(1);
  TORCH_CHECK(x.scalar_type() == torch::kHalf && H % 8 == 0);
  PeerTables pt{reinterpret_cast<const uint64_t*>(xrecv_ptrs.data_ptr<int64_t>()),
                reinterpret_cast<const uint64_t*>(meta_ptrs.data_ptr<int64_t>()),
                reinterpret_cast<const uint64_t*>(count_ptrs.data_ptr<int64_t>()),
                reinterpret_cast<const uint64_t*>(flag_ptrs.data_ptr<int64_t>())};
  const int grid = std::max(1, (P + 3) / 4);
  ep_push_kernel<<<grid, 128, 0, STREAM>>>((const __half*)x.data_ptr(), ids.data_ptr<int32_t>(),
                                          dest_slot.data_ptr<int32_t>(), dest_count.data_ptr<int32_t>(), P, k, H, e_loc,
                                          cap, me, n_ranks, pt, epoch.data_ptr<int64_t>(), done_ctr.data_ptr<int32_t>(),
                                          err.data_ptr<int32_t>());
}

void ep_gather(torch::Tensor flags, torch::Tensor counts, torch::Tensor meta, torch::Tensor xrecv, int64_t cap,
               int64_t n_ranks, int64_t e_loc, torch::Tensor epoch, torch::Tensor ybuf_ptrs, int64_t n_tile,
               torch::Tensor sorted_src, torch::Tensor items, torch::Tensor n_items, torch::Tensor row_dst,
               torch::Tensor n_rows, torch::Tensor xs, torch::Tensor err, int64_t timeout_ns) {
  const int H = xrecv.size(-1);
  const size_t sm = (2 * e_loc + 32 * e_loc) * sizeof(int);
  TORCH_CHECK(e_loc <= 1024 && sm <= 200 * 1024 && n_ranks < 64);
  auto kern = ep_gather_plan_kernel;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  kern<<<1, 1024, sm, STREAM>>>(flags.data_ptr<int64_t>(), counts.data_ptr<int64_t>(),
                                reinterpret_cast<const int2*>(meta.data_ptr<int32_t>()), cap, n_ranks, e_loc,
                                epoch.data_ptr<int64_t>(), reinterpret_cast<const uint64_t*>(ybuf_ptrs.data_ptr<int64_t>()),
                                H, n_tile, items.size(0), sorted_src.data_ptr<int32_t>(),
                                reinterpret_cast<int4*>(items.data_ptr<int32_t>()), n_items.data_ptr<int32_t>(),
                                row_dst.data_ptr<int64_t>(), n_rows.data_ptr<int32_t>(), err.data_ptr<int32_t>(),
                                (uint64_t)timeout_ns);
  ep_gather_rows_kernel<<<296, 128, 0, STREAM>>>((const uint4*)xrecv.data_ptr(), sorted_src.data_ptr<int32_t>(),
                                                 n_rows.data_ptr<int32_t>(), (uint4*)xs.data_ptr(), H / 8);
}

void ep_done(torch::Tensor done_ptrs, int64_t me, int64_t n_ranks, torch::Tensor epoch) {
  ep_done_kernel<<<1, 64, 0, STREAM>>>(reinterpret_cast<const uint64_t*>(done_ptrs.data_ptr<int64_t>()), me, n_ranks,
                                       epoch.data_ptr<int64_t>());
}

void ep_wait_done(torch::Tensor done, int64_t n_ranks, torch::Tensor epoch, torch::Tensor err, int64_t timeout_ns) {
  ep_wait_done_kernel<<<1, 64, 0, STREAM>>>(done.data_ptr<int64_t>(), n_ranks, epoch.data_ptr<int64_t>(),
                                            err.data_ptr<int32_t>(), (uint64_t)timeout_ns);
}

}  // namespace

void register_ep(pybind11::module& m) {
  m.def("ep_epoch", &ep_epoch);
  m.def("ep_plan", &ep_plan);
  m.def("ep_push", &ep_push);
  m.def("ep_gather", &ep_gather);
  m.def("ep_done", &ep_done);
  m.def("ep_wait_done", &ep_wait_done);
}
