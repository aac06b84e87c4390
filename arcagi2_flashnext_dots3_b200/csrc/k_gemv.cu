// Grouped low-bit GEMV for decode-sized expert groups (at most 8 tokens per item), W4/3/2 x A8.
//
// With a handful of tokens per expert the MoE projections are matrix-vector products bound by the weight stream;
// a tensor-core tile of 16+ tokens is mostly padding there. This kernel keeps the weight stream at HBM speed on
// CUDA cores by spending about one integer instruction per weight:
//
//   * activations are quantized once per row and 128-column group to int8 (scale = absmax / 127) by
//     `gemv_quant`, which also stores the group sums of the codes, with the columns of every 8-column block in the
//     order the 4-bit words unpack into (lowbit.cuh);
//   * each thread owns one weight row of a 128-row tile and streams that row's code words from HBM (word i of
//     row r at (i * 128 + r) * 4: a warp reads 128 contiguous bytes);
//   * codes are moved into byte lanes in that order with shift / mask (/ byte-permute below 4 bits) and multiplied
//     with the int8 activations by `dp4a` (4 products per instruction), exact in int32;
//   * per (row, group): y += s_w * s_x * (sum q*x - z * sum x) in fp32.
//
// The activation quantization is the one numerics change against fp16 activations (per-group int8, the same
// family as the reference's per-token-group FP8 activation quantization of its dense W8A8 GEMMs,
// dotsnote/engine/arcstats_pkg/arcstats/w8a8_ws.py:13-44).
//
// Epilogues: fp32 store (optionally to per-row destination addresses, the expert-parallel combine) and
// silu(gate) * up in the silu-pair row order (tile t = 64 gate rows then the 64 matching up rows) as fp16.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>
#include "wgemm.h"
#include "ptx.cuh"
#include "lowbit.cuh"

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()
constexpr int kMaxTok = 8;
constexpr int kMaxK = 8192;   // longest activation row staged in shared memory (int8; dynamic size 8 x K)

// ------------------------------------------------------------------------------------ activation quantization
// One warp per (row, 128-column group): lane l owns columns 4l..4l+3.
__global__ void gemv_quant_kernel(const __half* x, int rows, int K, int8_t* xq, float* xs, int* xsum) {
  fw::pdl_launch_dependents();   // the grouped GEMV that follows may launch now (it waits for these results)
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int G = K / 128;
  if (warp >= rows * G) return;
  const int r = warp / G, g = warp % G;
  const __half2* src = reinterpret_cast<const __half2*>(x + (int64_t)r * K + g * 128) + 2 * lane;
  const float2 a = __half22float2(src[0]), b = __half22float2(src[1]);
  float m = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float s = m / 127.f;
  const float inv = m > 0.f ? 127.f / m : 0.f;
  const int q0 = __float2int_rn(a.x * inv), q1 = __float2int_rn(a.y * inv);
  const int q2 = __float2int_rn(b.x * inv), q3 = __float2int_rn(b.y * inv);
  const uint32_t own =
      (uint32_t)(q0 & 255) | ((uint32_t)(q1 & 255) << 8) | ((uint32_t)(q2 & 255) << 16) | ((uint32_t)(q3 & 255) << 24);
  // columns of each 8-column block in the order [0, 4, 1, 5, 2, 6, 3, 7] (lowbit.cuh): lanes 2b and 2b+1 hold
  // columns 8b..8b+3 and 8b+4..8b+7 and write words [c0 c4 c1 c5] and [c2 c6 c3 c7]
  const uint32_t other = __shfl_xor_sync(0xffffffffu, own, 1);
  reinterpret_cast<uint32_t*>(xq + (int64_t)r * K + g * 128)[lane] =
      (lane & 1) ? __byte_perm(own, other, 0x3726) : __byte_perm(own, other, 0x5140);
  int sum = q0 + q1 + q2 + q3;
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) {
    xs[(int64_t)r * G + g] = s;
    xsum[(int64_t)r * G + g] = sum;
  }
}

using fw::lowbit::NWords;
using fw::lowbit::quad;

// dot[t] += sum over the 128 columns of group g of codes * x[t] for NT tokens (activations from shared memory,
// 16 bytes = 4 quads per load, the same address for every thread: a broadcast).
template <int FMT, int NT, int M4>
__device__ __forceinline__ void dot_quads(const uint32_t* cw, const int4* xg, int row_stride4, int* dot) {
  const uint32_t q0 = quad<FMT, 4 * M4>(cw), q1 = quad<FMT, 4 * M4 + 1>(cw);
  const uint32_t q2 = quad<FMT, 4 * M4 + 2>(cw), q3 = quad<FMT, 4 * M4 + 3>(cw);
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int4 x = xg[t * row_stride4 + M4];
    dot[t] = __dp4a((int)q0, x.x, dot[t]);
    dot[t] = __dp4a((int)q1, x.y, dot[t]);
    dot[t] = __dp4a((int)q2, x.z, dot[t]);
    dot[t] = __dp4a((int)q3, x.w, dot[t]);
  }
  if constexpr (M4 + 1 < 8) dot_quads<FMT, NT, M4 + 1>(cw, xg, row_stride4, dot);
}

// ------------------------------------------------------------------------------------ grouped GEMV
struct GemvArgs {
  const uint8_t* wbase;
  const int64_t* exp_off;
  const int8_t* exp_fmt;
  int row_tiles, kg;
  const int4* items;
  const int* n_items;
  int max_items;
  const int8_t* xq;      // [rows, K] int8 activations
  const float* xs;       // [rows, K/128] scales
  const int* xsum;       // [rows, K/128] code sums
  void* out;
  int out_ld, out_cols;
  int epi;
  const int64_t* row_dst;
};

template <int FMT, int NT>
__device__ __forceinline__ void run_item(const GemvArgs& a, int e, int t0, int n, int tile, const int* xsm,
                                         const float* xs_sm, const int* xsum_sm, float* gsh) {
  const int r = threadIdx.x;
  const uint32_t bb = fw::wgemm_block_bytes(FMT);
  constexpr int NW = NWords<FMT>::value;
  const uint8_t* base = a.wbase + a.exp_off[e] + (int64_t)tile * a.kg * bb;
  const int G = a.kg, Kw4 = a.kg * 8;  // int4 (16-byte) units of one activation row
  const int4* x4 = reinterpret_cast<const int4*>(xsm);
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  // software pipeline: the words, scale and zero of group g + 1 are in flight while group g is multiplied
  uint32_t w[NW];
  const uint32_t* wp = reinterpret_cast<const uint32_t*>(base);
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = __ldg(wp + i * 128 + r);
  unsigned short sb = __ldg(reinterpret_cast<const unsigned short*>(base + NW * 512) + r);
  int z = __ldg(base + NW * 512 + 256 + r);
  for (int g = 0; g < G; ++g) {
    uint32_t cw[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) cw[i] = w[i];
    const float s = __half2float(__ushort_as_half(sb));
    const int zc = z;
    if (g + 1 < G) {
      const uint8_t* nb = base + (int64_t)(g + 1) * bb;
      const uint32_t* nwp = reinterpret_cast<const uint32_t*>(nb);
#pragma unroll
      for (int i = 0; i < NW; ++i) w[i] = __ldg(nwp + i * 128 + r);
      sb = __ldg(reinterpret_cast<const unsigned short*>(nb + NW * 512) + r);
      z = __ldg(nb + NW * 512 + 256 + r);
    }
    int dot[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) dot[t] = 0;
    dot_quads<FMT, NT, 0>(cw, x4 + g * 8, Kw4, dot);
#pragma unroll
    for (int t = 0; t < NT; ++t)
      acc[t] = fmaf(s * xs_sm[t * G + g], (float)(dot[t] - zc * xsum_sm[t * G + g]), acc[t]);
  }
  const int row = tile * 128 + r;
  if (a.epi == 0) {
    if (row < a.out_cols) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < n) {
          float* dst = a.row_dst ? reinterpret_cast<float*>(a.row_dst[t0 + t])
                                 : reinterpret_cast<float*>(a.out) + (int64_t)(t0 + t) * a.out_ld;
          dst[row] = acc[t];
        }
      }
    }
  } else {
    __syncthreads();
    if (r >= 64) {
#pragma unroll
      for (int t = 0; t < NT; ++t) gsh[t * 64 + (r - 64)] = acc[t];
    }
    __syncthreads();
    if (r < 64) {
      const int f = tile * 64 + r;
      if (f < a.out_cols) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < n) {
            const float gt = acc[t], up = gsh[t * 64 + r];
            reinterpret_cast<__half*>(a.out)[(int64_t)(t0 + t) * a.out_ld + f] =
                __float2half_rn(gt / (1.f + __expf(-gt)) * up);
          }
        }
      }
    }
  }
}

// MINB: CTAs per SM the register budget is sized for (FW_GEMV_OCC=5/6/8 overrides the choice by row length)
template <int MINB>
__global__ void __launch_bounds__(128, MINB) gemv_grouped_kernel(GemvArgs a) {
  extern __shared__ int xsm[];   // [kMaxTok][K/4] int8x4 activations of the current item
  __shared__ float gsh[kMaxTok * 64];
  __shared__ float xs_sm[kMaxTok * (kMaxK / 128)];
  __shared__ int xsum_sm[kMaxTok * (kMaxK / 128)];
  fw::pdl_wait();                // launched early behind gemv_quant: its activations must be complete
  const int n_items = min(*a.n_items, a.max_items);
  const int total = n_items * a.row_tiles;
  const int Kw = a.kg * 32;
  int staged = -1;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    const int item = w / a.row_tiles, tile = w % a.row_tiles;
    const int4 it = a.items[item];
    const int e = it.x, t0 = it.y, n = min(it.z, kMaxTok);
    if (n <= 0) continue;
    if (staged != item) {
      // the unit's first weight group heads for L2 while its activations are staged (a block's row words are
      // 512 bytes apart: one prefetch per word of this thread's row)
      const int fmt0 = a.exp_fmt[e];
      const int nw0 = fmt0 == 4 ? 16 : fmt0 == 3 ? 13 : 8;
      const uint8_t* b0 = a.wbase + a.exp_off[e] + (int64_t)tile * a.kg * fw::wgemm_block_bytes(fmt0);
      for (int i = 0; i < nw0; ++i)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(b0 + (i * 128 + threadIdx.x) * 4));
      __syncthreads();
      const int4* src = reinterpret_cast<const int4*>(a.xq + (int64_t)t0 * Kw * 4);
      int4* dst = reinterpret_cast<int4*>(xsm);
      for (int i = threadIdx.x; i < n * Kw / 4; i += blockDim.x) dst[i] = src[i];
      for (int i = threadIdx.x; i < n * a.kg; i += blockDim.x) {
        xs_sm[i] = a.xs[(int64_t)t0 * a.kg + i];
        xsum_sm[i] = a.xsum[(int64_t)t0 * a.kg + i];
      }
      __syncthreads();
      staged = item;
    }
    const int fmt = a.exp_fmt[e];
#define FW_GEMV_NT(F)                                                                           \
  if (n <= 1) run_item<F, 1>(a, e, t0, n, tile, xsm, xs_sm, xsum_sm, gsh);                      \
  else if (n <= 2) run_item<F, 2>(a, e, t0, n, tile, xsm, xs_sm, xsum_sm, gsh);                 \
  else if (n <= 4) run_item<F, 4>(a, e, t0, n, tile, xsm, xs_sm, xsum_sm, gsh);                 \
  else run_item<F, 8>(a, e, t0, n, tile, xsm, xs_sm, xsum_sm, gsh);
    if (fmt == 4) {
      FW_GEMV_NT(4)
    } else if (fmt == 3) {
      FW_GEMV_NT(3)
    } else if (fmt == 2) {
      FW_GEMV_NT(2)
    }
#undef FW_GEMV_NT
  }
}

// ------------------------------------------------------------------------------------ TMA-fed variant
// The same per-row arithmetic, with the weight stream moved off the row threads: a producer warp copies each
// (tile, group) block (4.5 to 8.6 KB, contiguous in the packed layout) into a 4-stage shared-memory ring with
// 1-D bulk copies, so every SM keeps ~100 KB of weights in flight (3 CTAs x 4 stages) where the row threads'
// own loads kept one group per thread. Row threads read their code words from shared memory (word i of row r
// at (i * 128 + r) * 4: conflict-free) and release the stage after the loads. Opt-in (FW_GEMV_TMA=1): on the
// decode shapes measured it ran on par with the direct-load kernel, so the weight stream is not latency-bound.
constexpr int kStages = 4;
constexpr int kStageBytes = 8576;   // the largest block (4-bit)
constexpr int kTmaThreads = 160;    // warps 0-3 rows, warp 4 producer

struct Ring {
  uint32_t buf, full0, empty0;
  int* err;
  volatile int* abort_w;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int FMT, int NT>
__device__ __forceinline__ bool run_item_ring(const GemvArgs& a, int t0, int n, int tile, const int* xsm,
                                              const float* xs_sm, const int* xsum_sm, float* gsh, const Ring& R,
                                              int& cnt) {
  const int r = threadIdx.x, lane = r & 31;
  constexpr int NW = NWords<FMT>::value;
  const int G = a.kg, Kw4 = a.kg * 8;
  const int4* x4 = reinterpret_cast<const int4*>(xsm);
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.f;
  for (int g = 0; g < G; ++g) {
    const int s = cnt % kStages;
    if (!fw::mbar_wait_warp(R.full0 + 8 * s, (cnt / kStages) & 1, R.err, 7301, R.abort_w, R.timeout_ns)) return false;
    const uint32_t sb = R.buf + s * kStageBytes;
    uint32_t cw[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) cw[i] = lds32(sb + (i * 128 + r) * 4);
    unsigned short sbits;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sbits) : "r"(sb + NW * 512 + 2 * r));
    uint32_t zb;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(zb) : "r"(sb + NW * 512 + 256 + r));
    __syncwarp();
    if (lane == 0) fw::mbar_arrive(R.empty0 + 8 * s);
    ++cnt;
    const float sc = __half2float(__ushort_as_half(sbits));
    const int zc = (int)zb;
    int dot[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) dot[t] = 0;
    dot_quads<FMT, NT, 0>(cw, x4 + g * 8, Kw4, dot);
#pragma unroll
    for (int t = 0; t < NT; ++t)
      acc[t] = fmaf(sc * xs_sm[t * G + g], (float)(dot[t] - zc * xsum_sm[t * G + g]), acc[t]);
  }
  const int row = tile * 128 + r;
  if (a.epi == 0) {
    if (row < a.out_cols) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        if (t < n) {
          float* dst = a.row_dst ? reinterpret_cast<float*>(a.row_dst[t0 + t])
                                 : reinterpret_cast<float*>(a.out) + (int64_t)(t0 + t) * a.out_ld;
          dst[row] = acc[t];
        }
      }
    }
  } else {
    fw::named_barrier(1, 128);
    if (r >= 64) {
#pragma unroll
      for (int t = 0; t < NT; ++t) gsh[t * 64 + (r - 64)] = acc[t];
    }
    fw::named_barrier(1, 128);
    if (r < 64) {
      const int f = tile * 64 + r;
      if (f < a.out_cols) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (t < n) {
            const float gt = acc[t], up = gsh[t * 64 + r];
            reinterpret_cast<__half*>(a.out)[(int64_t)(t0 + t) * a.out_ld + f] =
                __float2half_rn(gt / (1.f + __expf(-gt)) * up);
          }
        }
      }
    }
  }
  return true;
}

__global__ void __launch_bounds__(kTmaThreads, 3) gemv_grouped_tma_kernel(GemvArgs a, int* err, uint64_t timeout_ns) {
  extern __shared__ __align__(1024) int xsm[];   // [kMaxTok][K/4] int8x4 activations, then the weight ring
  __shared__ float gsh[kMaxTok * 64];
  __shared__ float xs_sm[kMaxTok * (kMaxK / 128)];
  __shared__ int xsum_sm[kMaxTok * (kMaxK / 128)];
  __shared__ __align__(8) uint64_t bars[2 * kStages];
  __shared__ int abort_sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = min(*a.n_items, a.max_items);
  const int total = n_items * a.row_tiles;
  const int Kw = a.kg * 32;
  Ring R;
  R.buf = fw::smem_u32(xsm) + (uint32_t)(kMaxTok * a.kg * 128);
  R.full0 = fw::smem_u32(&bars[0]);
  R.empty0 = fw::smem_u32(&bars[kStages]);
  R.err = err;
  R.abort_w = &abort_sm;
  R.timeout_ns = timeout_ns;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      fw::mbar_init(R.full0 + 8 * s, 1);
      fw::mbar_init(R.empty0 + 8 * s, 4);
    }
    abort_sm = 0;
    fw::fence_mbar_init();
  }
  __syncthreads();
  if (warp == 4) {
    if (lane == 0) {
      const uint64_t pol = fw::l2_policy_evict_first();
      int cnt = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        const int item = w / a.row_tiles, tile = w % a.row_tiles;
        const int4 it = a.items[item];
        if (min(it.z, kMaxTok) <= 0) continue;
        const uint32_t bb = fw::wgemm_block_bytes(a.exp_fmt[it.x]);
        const uint8_t* base = a.wbase + a.exp_off[it.x] + (int64_t)tile * a.kg * bb;
        for (int g = 0; g < a.kg; ++g) {
          const int s = cnt % kStages;
          if (cnt >= kStages &&
              !fw::mbar_wait(R.empty0 + 8 * s, ((cnt / kStages) - 1) & 1, err, 7302, &abort_sm, timeout_ns)) {
            ok = false;
            break;
          }
          fw::mbar_arrive_expect_tx(R.full0 + 8 * s, bb);
          fw::tma_bulk_g2s(R.buf + s * kStageBytes, base + (int64_t)g * bb, bb, R.full0 + 8 * s, pol);
          ++cnt;
        }
      }
      // no copy may still be in flight when the CTA exits
      volatile int no_abort = 0;
      for (int c = max(0, cnt - kStages); c < cnt; ++c)
        fw::mbar_wait(R.full0 + 8 * (c % kStages), (c / kStages) & 1, err, 7303, &no_abort, timeout_ns);
    }
    __syncwarp();
  } else {
    int staged = -1, cnt = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      const int item = w / a.row_tiles, tile = w % a.row_tiles;
      const int4 it = a.items[item];
      const int e = it.x, t0 = it.y, n = min(it.z, kMaxTok);
      if (n <= 0) continue;
      if (staged != item) {
        fw::named_barrier(1, 128);
        const int4* src = reinterpret_cast<const int4*>(a.xq + (int64_t)t0 * Kw * 4);
        int4* dst = reinterpret_cast<int4*>(xsm);
        for (int i = tid; i < n * Kw / 4; i += 128) dst[i] = src[i];
        for (int i = tid; i < n * a.kg; i += 128) {
          xs_sm[i] = a.xs[(int64_t)t0 * a.kg + i];
          xsum_sm[i] = a.xsum[(int64_t)t0 * a.kg + i];
        }
        fw::named_barrier(1, 128);
        staged = item;
      }
      const int fmt = a.exp_fmt[e];
      bool ok = true;
#define FW_GEMV_NT(F)                                                                                        \
  if (n <= 1) ok = run_item_ring<F, 1>(a, t0, n, tile, xsm, xs_sm, xsum_sm, gsh, R, cnt);                    \
  else if (n <= 2) ok = run_item_ring<F, 2>(a, t0, n, tile, xsm, xs_sm, xsum_sm, gsh, R, cnt);               \
  else if (n <= 4) ok = run_item_ring<F, 4>(a, t0, n, tile, xsm, xs_sm, xsum_sm, gsh, R, cnt);               \
  else ok = run_item_ring<F, 8>(a, t0, n, tile, xsm, xs_sm, xsum_sm, gsh, R, cnt);
      if (fmt == 4) {
        FW_GEMV_NT(4)
      } else if (fmt == 3) {
        FW_GEMV_NT(3)
      } else if (fmt == 2) {
        FW_GEMV_NT(2)
      }
#undef FW_GEMV_NT
      if (!ok) break;
    }
  }
  __syncthreads();
}

void gemv_quant(torch::Tensor x, torch::Tensor xq, torch::Tensor xs, torch::Tensor xsum) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kHalf && x.is_contiguous() && x.size(1) % 128 == 0, "x fp16");
  const int rows = x.size(0), K = x.size(1);
  TORCH_CHECK(xq.scalar_type() == torch::kInt8 && xq.numel() >= (int64_t)rows * K, "xq int8");
  TORCH_CHECK(xs.numel() >= (int64_t)rows * (K / 128) && xsum.numel() >= (int64_t)rows * (K / 128), "xs/xsum");
  const int64_t warps = (int64_t)rows * (K / 128);
  if (warps)
    gemv_quant_kernel<<<(warps * 32 + 255) / 256, 256, 0, STREAM>>>(
        reinterpret_cast<const __half*>(x.data_ptr()), rows, K, xq.data_ptr<int8_t>(), xs.data_ptr<float>(),
        xsum.data_ptr<int>());
}

void gemv_grouped(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, int64_t row_tiles, int64_t kg,
                  torch::Tensor items, torch::Tensor n_items, int64_t max_items, torch::Tensor xq, torch::Tensor xs,
                  torch::Tensor xsum, torch::Tensor out, int64_t out_cols, int64_t epi,
                  c10::optional<torch::Tensor> row_dst, c10::optional<torch::Tensor> err, int64_t timeout_ns) {
  TORCH_CHECK(xq.is_cuda() && xq.scalar_type() == torch::kInt8 && xq.size(1) == kg * 128, "xq int8 [rows, K]");
  TORCH_CHECK(kg * 128 <= kMaxK, "K too large for the staged activations");
  TORCH_CHECK(items.scalar_type() == torch::kInt32 && items.size(1) == 4, "items int32 [n, 4]");
  TORCH_CHECK(epi == 0 ? out.scalar_type() == torch::kFloat : out.scalar_type() == torch::kHalf, "out dtype");
  TORCH_CHECK(out.is_contiguous(), "out contiguous");
  const c10::cuda::CUDAGuard guard(xq.device());
  GemvArgs a{};
  a.wbase = wbase.data_ptr<uint8_t>();
  a.exp_off = exp_off.data_ptr<int64_t>();
  a.exp_fmt = exp_fmt.data_ptr<int8_t>();
  a.row_tiles = row_tiles;
  a.kg = kg;
  a.items = reinterpret_cast<const int4*>(items.data_ptr<int32_t>());
  a.n_items = n_items.data_ptr<int32_t>();
  a.max_items = max_items;
  a.xq = xq.data_ptr<int8_t>();
  a.xs = xs.data_ptr<float>();
  a.xsum = xsum.data_ptr<int>();
  a.out = out.data_ptr();
  a.out_ld = out.size(1);
  a.out_cols = out_cols;
  a.epi = epi;
  a.row_dst = row_dst ? row_dst->data_ptr<int64_t>() : nullptr;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = (size_t)kMaxTok * kg * 128;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemv_grouped_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxTok * kMaxK);
    cudaFuncSetAttribute(gemv_grouped_kernel<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxTok * kMaxK);
    cudaFuncSetAttribute(gemv_grouped_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxTok * kMaxK);
    attr = true;
  }
  // short rows (K <= 8 groups, e.g. the FN down projection) gain from more resident CTAs (0.098 -> 0.091 ms),
  // long rows do not (gate_up 0.147 -> 0.152 ms)
  static const int occ_env = getenv("FW_GEMV_OCC") ? atoi(getenv("FW_GEMV_OCC")) : 0;
  const int occ = occ_env > 0 ? occ_env : (kg <= 8 ? 8 : 5);
  const int64_t work = max_items * row_tiles;
  // FW_GEMV_TMA=1: weight blocks through a bulk-copy ring (measured on par with the direct loads: 0.154 vs 0.146 ms
  // gate_up, 0.094 vs 0.098 ms down on the FN layer), kept for shapes where the load latency is exposed
  static const bool tma = getenv("FW_GEMV_TMA") && atoi(getenv("FW_GEMV_TMA"));
  if (tma && err) {
    // TMA-fed ring: activations + 4 weight stages per CTA, up to 3 CTAs per SM
    const size_t smem_tma = (size_t)kMaxTok * kg * 128 + (size_t)kStages * kStageBytes;
    static bool attr_tma = false;
    if (!attr_tma) {
      cudaFuncSetAttribute(gemv_grouped_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
      attr_tma = true;
    }
    TORCH_CHECK(smem_tma <= 200 * 1024, "grouped GEMV: activations + ring exceed shared memory");
    const int per_sm = (int)std::max<size_t>(1, std::min<size_t>(3, (227 * 1024) / (smem_tma + 8 * 1024)));
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(work, (int64_t)sms * per_sm));
    gemv_grouped_tma_kernel<<<grid, kTmaThreads, smem_tma, STREAM>>>(a, err->data_ptr<int32_t>(),
                                                                     (uint64_t)timeout_ns);
    return;
  }
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(work, (int64_t)sms * 12));
  // programmatic launch behind gemv_quant (FW_PDL=0: plain launch)
  static const bool pdl = !(getenv("FW_PDL") && atoi(getenv("FW_PDL")) == 0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = STREAM;
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = la;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  if (occ >= 8) e = cudaLaunchKernelEx(&cfg, gemv_grouped_kernel<8>, a);
  else if (occ == 6) e = cudaLaunchKernelEx(&cfg, gemv_grouped_kernel<6>, a);
  else e = cudaLaunchKernelEx(&cfg, gemv_grouped_kernel<5>, a);
  TORCH_CHECK(e == cudaSuccess, "gemv_grouped launch failed: ", cudaGetErrorString(e));
}

}  // namespace

void register_gemv(pybind11::module& m) {
  m.def("gemv_quant", &gemv_quant);
  m.def("gemv_grouped", &gemv_grouped);
}
