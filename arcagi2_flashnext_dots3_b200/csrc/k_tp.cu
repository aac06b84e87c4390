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

// ------------------------------------------------------------------------------------------------------------
// Quantized two-shot all-reduce fused with the residual add: h[:n] += sum over ranks of x_r[:n].
//
// The n elements are cut into W chunks of `chunk` elements (a multiple of 128); rank c owns chunk c. Per group
// of 128 elements a warp computes the absmax, scale = absmax / 127 and int8 codes round(x / scale). One launch,
// three phases, CTA b handling the groups g = b, b + G, ... of every chunk:
//   1. reduce-scatter: quantize the local partial; the codes and scale of chunk c's groups go into slot [me] of
//      owner c's RS area; then flag rs[me][b] = epoch on owner c (system fence, st.release.sys);
//   2. reduce: wait (bounded) for rs[s][b] >= epoch from every source s, dequantize and sum in rank order
//      (deterministic), quantize the sum and store it into slot [me] of every rank's AG area; flag ag[me][b];
//   3. gather: wait for ag[o][b] from every owner o, dequantize and add into h.
// The owner reads back its own quantized sum like every other rank, so all ranks add identical values. Per rank
// 2 (W - 1) / W bytes per element cross NVLink (plus 4 bytes of scale per 128), against 4 (W - 1) for the fp32
// fan-out. Waits only ever involve CTAs with the same index on other GPUs, and the grid never exceeds one CTA per
// SM, so every CTA a wait depends on is resident. Two parities (epoch & 1) make the areas reusable: a rank
// writes parity p again two epochs later only after the owners' AG flags of the epoch in between, which they
// set after their reads of parity p. A timed-out wait records 6410 + peer and raises the abort word; CTAs that
// see it return.
struct QArLayout {   // byte offsets inside one rank's symmetric area
  int64_t rs_q, rs_s, ag_q, ag_s, flags;
  int64_t chunk, groups;     // elements per chunk, 128-element groups per chunk
};

__device__ __forceinline__ float warp_absmax(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t pack_q8(float4 v, float inv) {
  const int a = __float2int_rn(v.x * inv), b = __float2int_rn(v.y * inv), c = __float2int_rn(v.z * inv),
            d = __float2int_rn(v.w * inv);
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) | ((uint32_t)(d & 0xff) << 24);
}

__device__ __forceinline__ float4 unpack_q8(uint32_t q, float s) {
  return make_float4((float)(int8_t)(q & 0xff) * s, (float)(int8_t)((q >> 8) & 0xff) * s,
                     (float)(int8_t)((q >> 16) & 0xff) * s, (float)(int8_t)(q >> 24) * s);
}

// 4-bit codes -7..7 of four values, two per byte, as 16 bits.
__device__ __forceinline__ uint32_t pack_q4(float4 v, float inv) {
  auto c = [&](float x) { return (uint32_t)(max(-7, min(7, __float2int_rn(x * inv))) & 0xf); };
  return c(v.x) | (c(v.y) << 4) | (c(v.z) << 8) | (c(v.w) << 12);
}

__device__ __forceinline__ float4 unpack_q4(uint32_t q, float s) {
  auto d = [&](int sh) { int c = (int)((q >> sh) & 0xf); return (float)(c >= 8 ? c - 16 : c) * s; };
  return make_float4(d(0), d(4), d(8), d(12));
}

// Orthonormal 128-point Walsh-Hadamard transform of a warp's 128 values (lane l holds elements 4l .. 4l + 3):
// butterflies of stride 1 and 2 in registers, 4 .. 64 across lanes. Symmetric and orthogonal: its own inverse.
__device__ __forceinline__ float4 wht128(float4 v) {
  float a = v.x + v.y, b = v.x - v.y, c = v.z + v.w, d = v.z - v.w;
  v = make_float4(a + c, b + d, a - c, b - d);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const float px = __shfl_xor_sync(0xffffffffu, v.x, m), py = __shfl_xor_sync(0xffffffffu, v.y, m),
                pz = __shfl_xor_sync(0xffffffffu, v.z, m), pw = __shfl_xor_sync(0xffffffffu, v.w, m);
    if (lane & m) v = make_float4(px - v.x, py - v.y, pz - v.z, pw - v.w);
    else v = make_float4(v.x + px, v.y + py, v.z + pz, v.w + pw);
  }
  const float r = 0.08838834764831845f;   // 1 / sqrt(128)
  return make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
}

struct QArOpts {
  int bits;          // 8 or 4
  int had;           // rotate each 128-group by the Walsh-Hadamard transform before quantizing
  float* carry;      // error feedback: [n_max] this rank's carried error (nullptr: off)
};

// Quantize one warp-group of four values per lane; returns the packed codes and the scale, and (when ef) the
// quantization error in the original domain.
__device__ __forceinline__ uint32_t quant_group(float4 v, const QArOpts& o, float& scale, float4* err) {
  const float qmax = o.bits == 8 ? 127.f : 7.f;
  const float amax = warp_absmax(fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  scale = amax > 0.f ? amax / qmax : 1.f;
  const uint32_t q = o.bits == 8 ? pack_q8(v, 1.f / scale) : pack_q4(v, 1.f / scale);
  if (err) {
    const float4 d = o.bits == 8 ? unpack_q8(q, scale) : unpack_q4(q, scale);
    float4 e = make_float4(v.x - d.x, v.y - d.y, v.z - d.z, v.w - d.w);
    *err = o.had ? wht128(e) : e;
  }
  return q;
}

__device__ __forceinline__ void store_codes(int8_t* base, int64_t g, int lane, uint32_t q, int bits) {
  if (bits == 8) reinterpret_cast<uint32_t*>(base + g * 128)[lane] = q;
  else reinterpret_cast<uint16_t*>(base + g * 128)[lane] = (uint16_t)q;
}

__device__ __forceinline__ float4 load_codes(const int8_t* base, int64_t g, int lane, float s, int bits) {
  if (bits == 8) return unpack_q8(reinterpret_cast<const uint32_t*>(base + g * 128)[lane], s);
  return unpack_q4(reinterpret_cast<const uint16_t*>(base + g * 128)[lane], s);
}

// Bounded wait of one thread for flag >= e; false on timeout (error 6410 + peer) or abort.
__device__ bool wait_epoch(const int64_t* flag, int64_t e, int peer, int* err, int* abort_word, uint64_t limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_sys(flag) >= e) return true;
    if (*(volatile int*)abort_word) return false;
    if ((it & 63) == 63) {
      const uint64_t now = gtimer();
      if (!t0) t0 = now;
      else if (now - t0 > limit_ns) {
        atomicCAS(err, 0, 6410 + peer);
        *(volatile int*)abort_word = 1;
        return false;
      }
      __nanosleep(64);
    }
  }
}

__global__ void __launch_bounds__(128) tp_qar_kernel(const float* __restrict__ x, float* __restrict__ h, int64_t n,
                                                     const uint64_t* bases, int me, int W, QArLayout L,
                                                     const int64_t* epoch, int* err, uint64_t limit_ns, QArOpts o) {
  __shared__ int ok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = gridDim.x, b = blockIdx.x;
  const int64_t e = epoch[0];
  const int par = (int)(e & 1);
  int* abort_word = err + 1;
  char* mine = reinterpret_cast<char*>(bases[me]);
  int64_t* my_flags = reinterpret_cast<int64_t*>(mine + L.flags);     // [2 par][2 phase][W][G]
  auto flag_at = [&](char* base, int phase, int src) {
    return reinterpret_cast<int64_t*>(base + L.flags) + (((int64_t)par * 2 + phase) * W + src) * G + b;
  };
  // ---- phase 1: quantize the partial, scatter each chunk's groups to its owner
  for (int c = 0; c < W; ++c) {
    char* peer = reinterpret_cast<char*>(bases[c]);
    int8_t* q = reinterpret_cast<int8_t*>(peer + L.rs_q) + ((int64_t)par * W + me) * L.chunk;
    float* sc = reinterpret_cast<float*>(peer + L.rs_s) + ((int64_t)par * W + me) * L.groups;
    for (int64_t g = b + (int64_t)warp * G; g < L.groups; g += 4LL * G) {
      const int64_t i0 = (int64_t)c * L.chunk + g * 128 + lane * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i0 + 3 < n) v = *reinterpret_cast<const float4*>(x + i0);
      else if (i0 < n) { v.x = x[i0]; if (i0 + 1 < n) v.y = x[i0 + 1]; if (i0 + 2 < n) v.z = x[i0 + 2]; }
      if (o.carry && i0 < n) {   // error feedback: add the error carried from the previous all-reduce
        const float4 cv = *reinterpret_cast<const float4*>(o.carry + i0);
        v.x += cv.x; v.y += cv.y; v.z += cv.z; v.w += cv.w;
      }
      if (o.had) v = wht128(v);
      float s;
      float4 e;
      const uint32_t qq = quant_group(v, o, s, o.carry ? &e : nullptr);
      store_codes(q, g, lane, qq, o.bits);
      if (lane == 0) sc[g] = s;
      if (o.carry && i0 < n) *reinterpret_cast<float4*>(o.carry + i0) = e;   // this rank's share of the error
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) st_release_sys(flag_at(reinterpret_cast<char*>(bases[threadIdx.x]), 0, me), e);
  // ---- phase 2: reduce this rank's chunk
  if (threadIdx.x == 0) {
    ok = 1;
    for (int s2 = 0; s2 < W && ok; ++s2) ok = wait_epoch(flag_at(mine, 0, s2), e, s2, err, abort_word, limit_ns);
  }
  __syncthreads();
  if (!ok) return;
  {
    const int8_t* rq = reinterpret_cast<const int8_t*>(mine + L.rs_q) + (int64_t)par * W * L.chunk;
    const float* rs = reinterpret_cast<const float*>(mine + L.rs_s) + (int64_t)par * W * L.groups;
    for (int64_t g = b + (int64_t)warp * G; g < L.groups; g += 4LL * G) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s2 = 0; s2 < W; ++s2) {
        const float4 d = load_codes(rq + (int64_t)s2 * L.chunk, g, lane, rs[(int64_t)s2 * L.groups + g], o.bits);
        acc.x += d.x; acc.y += d.y; acc.z += d.z; acc.w += d.w;
      }
      float s;
      float4 e;
      const int64_t i0 = (int64_t)me * L.chunk + g * 128 + lane * 4;
      // the error pointer must be warp-uniform (the Hadamard transform shuffles); only the store is per lane
      const uint32_t packed = quant_group(acc, o, s, o.carry ? &e : nullptr);
      if (o.carry && i0 < n) {   // the owner also carries the re-quantization error of its chunk's sum
        float4 cv = *reinterpret_cast<float4*>(o.carry + i0);
        cv.x += e.x; cv.y += e.y; cv.z += e.z; cv.w += e.w;
        *reinterpret_cast<float4*>(o.carry + i0) = cv;
      }
      for (int r = 0; r < W; ++r) {
        char* peer = reinterpret_cast<char*>(bases[r]);
        store_codes(reinterpret_cast<int8_t*>(peer + L.ag_q) + ((int64_t)par * W + me) * L.chunk, g, lane, packed,
                    o.bits);
        if (lane == 0) reinterpret_cast<float*>(peer + L.ag_s)[((int64_t)par * W + me) * L.groups + g] = s;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) st_release_sys(flag_at(reinterpret_cast<char*>(bases[threadIdx.x]), 1, me), e);
  // ---- phase 3: gather every owner's reduced chunk into h
  if (threadIdx.x == 0) {
    ok = 1;
    for (int ow = 0; ow < W && ok; ++ow) ok = wait_epoch(flag_at(mine, 1, ow), e, ow, err, abort_word, limit_ns);
  }
  __syncthreads();
  if (!ok) return;
  const int8_t* aq = reinterpret_cast<const int8_t*>(mine + L.ag_q) + (int64_t)par * W * L.chunk;
  const float* as = reinterpret_cast<const float*>(mine + L.ag_s) + (int64_t)par * W * L.groups;
  for (int ow = 0; ow < W; ++ow) {
    for (int64_t g = b + (int64_t)warp * G; g < L.groups; g += 4LL * G) {
      const int64_t i0 = (int64_t)ow * L.chunk + g * 128 + lane * 4;
      float4 d = load_codes(aq + (int64_t)ow * L.chunk, g, lane, as[(int64_t)ow * L.groups + g], o.bits);
      if (o.had) d = wht128(d);      // all lanes take part in the shuffles before any of them leaves
      if (i0 >= n) continue;
      if (i0 + 3 < n) {
        float4 t = *reinterpret_cast<float4*>(h + i0);
        t.x += d.x; t.y += d.y; t.z += d.z; t.w += d.w;
        *reinterpret_cast<float4*>(h + i0) = t;
      } else {
        h[i0] += d.x;
        if (i0 + 1 < n) h[i0 + 1] += d.y;
        if (i0 + 2 < n) h[i0 + 2] += d.z;
      }
    }
  }
}

// Layout of one rank's quantized all-reduce area for up to n_max elements over W ranks and G CTAs.
QArLayout qar_layout(int64_t n_max, int W, int G) {
  QArLayout L;
  L.chunk = ((n_max + W - 1) / W + 127) / 128 * 128;
  L.groups = L.chunk / 128;
  auto al = [](int64_t v) { return (v + 255) / 256 * 256; };
  L.rs_q = 0;
  L.rs_s = al(L.rs_q + 2LL * W * L.chunk);
  L.ag_q = al(L.rs_s + 2LL * W * L.groups * 4);
  L.ag_s = al(L.ag_q + 2LL * W * L.chunk);
  L.flags = al(L.ag_s + 2LL * W * L.groups * 4);
  return L;
}

int64_t tp_qar_bytes(int64_t n_max, int64_t W, int64_t G) {
  const QArLayout L = qar_layout(n_max, (int)W, (int)G);
  return L.flags + 2LL * 2 * W * G * 8;
}

void tp_qar(torch::Tensor x, torch::Tensor h, int64_t n, torch::Tensor bases, int64_t me, int64_t n_max, int64_t G,
            torch::Tensor epoch, torch::Tensor err, int64_t timeout_ns, int64_t bits, bool had,
            c10::optional<torch::Tensor> carry) {
  TORCH_CHECK(bits == 8 || bits == 4, "payload bits must be 8 or 4");
  QArOpts o{(int)bits, had ? 1 : 0, nullptr};
  if (carry) {
    TORCH_CHECK(carry->is_cuda() && carry->scalar_type() == torch::kFloat && carry->numel() >= n &&
                reinterpret_cast<uintptr_t>(carry->data_ptr()) % 16 == 0);
    o.carry = carry->data_ptr<float>();
  }
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat && x.is_contiguous() && x.numel() >= n);
  TORCH_CHECK(h.is_cuda() && h.scalar_type() == torch::kFloat && h.is_contiguous() && h.numel() >= n);
  TORCH_CHECK(n <= n_max, "all-reduce larger than its area");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0);
  const int W = bases.numel();
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  TORCH_CHECK(G >= 1 && G <= sms && W <= 128, "grid must be co-resident (at most one CTA per SM)");
  const QArLayout L = qar_layout(n_max, W, (int)G);
  tp_qar_kernel<<<(int)G, 128, 0, STREAM>>>(x.data_ptr<float>(), h.data_ptr<float>(), n,
                                            reinterpret_cast<const uint64_t*>(bases.data_ptr<int64_t>()), (int)me, W,
                                            L, epoch.data_ptr<int64_t>(), err.data_ptr<int32_t>(),
                                            (uint64_t)timeout_ns, o);
}

}  // namespace

void register_tp(pybind11::module& m) {
  m.def("tp_epoch", &tp_epoch);
  m.def("tp_push", &tp_push);
  m.def("tp_signal", &tp_signal);
  m.def("tp_reduce", &tp_reduce);
  m.def("tp_qar", &tp_qar);
  m.def("tp_qar_bytes", &tp_qar_bytes);
}
