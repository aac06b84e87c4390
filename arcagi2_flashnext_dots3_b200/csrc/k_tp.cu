// Tensor-parallel all-reduce over NVLink peer memory, with the producing GEMM writing straight into the peers.
//
// Every rank owns a symmetric buffer of 2 parity slots x W source slots x [T, H] fp32 plus W int64 flags per
// parity. One all-reduce (epoch e, parity e & 1):
//   1. the row-parallel GEMM's epilogue stores each output element into slot [me] of every rank's buffer (the
//      wgemm "fan-out" epilogue), or `tp_push` copies an already-computed partial there;
//   2. `tp_signal` (after the producer in stream order): system-scope fence, then flag[me] = e on every rank
//      (st.release.sys);
//   3. `tp_reduce`: wait (bounded; error code 6401 + source on timeout) until every flag has reached e
//      (ld.acquire.sys), then h += sum over sources in rank order (deterministic), or out = sum.
// Two parities suffice: a rank reuses parity p only after its previous reduce of p, which needed every peer's
// push of p, which each peer issued after its own previous reduce of p (stream order).
//
// Plays the role of the reference's host-staged two-shot all-reduce (dotsnote/engine/arcstats_pkg/arcstats/
// host_ar.py:1-12, 146; epoch flags per rank, bounded waits :47-58) with the transfer done by peer stores over
// NVLink instead of PCIe host memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

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

__global__ void tp_epoch_kernel(int64_t* epoch) { epoch[0] += 1; }

// x [n] fp32 -> slot [me] of parity (epoch & 1) on every rank; float4 copies.
__global__ void tp_push_kernel(const float4* x, int64_t n4, const uint64_t* bufs, int me, int W, int64_t slot4,
                               const int64_t* epoch) {
  const int par = (int)(epoch[0] & 1);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
#pragma unroll 1
    for (int p = 0; p < W; ++p)
      reinterpret_cast<float4*>(bufs[p])[((int64_t)par * W + me) * slot4 + i] = v;
  }
}

__global__ void tp_signal_kernel(const uint64_t* flags, int me, int W, const int64_t* epoch) {
  __threadfence_system();
  const int64_t e = epoch[0];
  const int par = (int)(e & 1);
  if ((int)threadIdx.x < W) st_release_sys(reinterpret_cast<int64_t*>(flags[threadIdx.x]) + par * W + me, e);
}

// Wait for every source of this epoch, then dst (+)= sum of the W slots. One wait per block (bounded).
__global__ void tp_reduce_kernel(const float4* buf, const int64_t* flags, int W, int64_t n4, int64_t slot4,
                                 const int64_t* epoch, float4* dst, int accumulate, int* err, uint64_t limit_ns,
                                 int* abort_word) {
  __shared__ int ok;
  const int64_t e = epoch[0];
  const int par = (int)(e & 1);
  if (threadIdx.x == 0) {
    ok = 1;
    for (int p = 0; p < W && ok; ++p) {
      uint64_t t0 = 0;
      for (uint32_t it = 0;; ++it) {
        if (ld_acquire_sys(flags + par * W + p) >= e) break;
        if (*(volatile int*)abort_word) {
          ok = 0;
          break;
        }
        if ((it & 63) == 63) {
          const uint64_t now = gtimer();
          if (!t0) t0 = now;
          else if (now - t0 > limit_ns) {
            atomicCAS(err, 0, 6401 + p);
            *(volatile int*)abort_word = 1;
            ok = 0;
            break;
          }
          __nanosleep(100);
        }
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const float4* b = buf + (int64_t)par * W * slot4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = b[i];
    for (int p = 1; p < W; ++p) {
      const float4 v = b[(int64_t)p * slot4 + i];
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    if (accumulate) {
      float4 d = dst[i];
      d.x += s.x; d.y += s.y; d.z += s.z; d.w += s.w;
      dst[i] = d;
    } else {
      dst[i] = s;
    }
  }
}

void tp_epoch(torch::Tensor epoch) { tp_epoch_kernel<<<1, 1, 0, STREAM>>>(epoch.data_ptr<int64_t>()); }

void tp_push(torch::Tensor x, torch::Tensor buf_ptrs, int64_t me, int64_t slot_elems, torch::Tensor epoch) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous() && x.numel() % 4 == 0);
  TORCH_CHECK(slot_elems % 4 == 0 && x.numel() <= slot_elems, "partial larger than a slot");
  const int W = buf_ptrs.numel();
  const int64_t n4 = x.numel() / 4;
  const int grid = (int)std::min<int64_t>(1184, (n4 + 255) / 256);
  if (n4)
    tp_push_kernel<<<grid, 256, 0, STREAM>>>(reinterpret_cast<const float4*>(x.data_ptr<float>()), n4,
                                            reinterpret_cast<const uint64_t*>(buf_ptrs.data_ptr<int64_t>()), me, W,
                                            slot_elems / 4, epoch.data_ptr<int64_t>());
}

void tp_signal(torch::Tensor flag_ptrs, int64_t me, torch::Tensor epoch) {
  const int W = flag_ptrs.numel();
  TORCH_CHECK(W <= 64);
  tp_signal_kernel<<<1, 64, 0, STREAM>>>(reinterpret_cast<const uint64_t*>(flag_ptrs.data_ptr<int64_t>()), me, W,
                                         epoch.data_ptr<int64_t>());
}

void tp_reduce(torch::Tensor buf, torch::Tensor flags, int64_t W, int64_t n, int64_t slot_elems, torch::Tensor epoch,
               torch::Tensor dst, bool accumulate, torch::Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == torch::kFloat && dst.is_contiguous() && n % 4 == 0 &&
              dst.numel() >= n);
  const int64_t n4 = n / 4;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(592, (n4 + 255) / 256));
  tp_reduce_kernel<<<grid, 256, 0, STREAM>>>(reinterpret_cast<const float4*>(buf.data_ptr<float>()),
                                             flags.data_ptr<int64_t>(), W, n4, slot_elems / 4,
                                             epoch.data_ptr<int64_t>(), reinterpret_cast<float4*>(dst.data_ptr<float>()),
                                             accumulate ? 1 : 0, err.data_ptr<int32_t>(), (uint64_t)timeout_ns,
                                             err.data_ptr<int32_t>() + 1);
}

}  // namespace

void register_tp(pybind11::module& m) {
  m.def("tp_epoch", &tp_epoch);
  m.def("tp_push", &tp_push);
  m.def("tp_signal", &tp_signal);
  m.def("tp_reduce", &tp_reduce);
}
