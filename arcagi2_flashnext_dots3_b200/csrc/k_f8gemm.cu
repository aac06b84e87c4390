// Dense FP8 GEMM for decode batches on tcgen05 `kind::f8f6f4` (e4m3 x e4m3 -> fp32 in TMEM), sm_100a.
//
// y[t, r] = sum_kb  sw[r/128, kb] * sx[t, kb] * sum_{k in kb} W8[r, k] * X8[t, k]
//
// Weights W8 [R, K] are the checkpoint's e4m3 codes in plain row-major order with one fp32 scale per 128x128 block
// (the `weight_scale_inv` convention); activations are quantized per (token, 128-column group) to e4m3 by
// `f8_quant_kernel` (scale = absmax / 448), the per-token-group FP8 activations of the reference's W8A8 GEMMs
// (dotsnote/engine/arcstats_pkg/arcstats/w8a8_ws.py:13-44 FUSE_Q, :76 ws_mm). Both operands reach shared memory
// by 2-D TMA in the 128-byte swizzle, which for 8-bit data is exactly one 128-column group per row: the MMA reads
// the weight tile as TMA wrote it, with no conversion step in between.
//
// Because both scales change with the 128-column group, each group's four K=32 MMAs accumulate into their own
// TMEM buffer (a ring of 4), and the epilogue warps fold buffer kb into registers with sw * sx[t] while the MMA
// fills the next one (the scale promotion of block-scaled FP8 GEMMs, here per group of 128).
//
// CTA (320 threads, one per SM):
//   warp 0      TMA producer: weight tile [128 rows x 128 B] + activation tile [NT tokens x 128 B] per stage
//   warp 1      TMEM allocation; one elected thread issues tcgen05.mma (M=128, N=NT, 4 x K32 per group)
//   warps 2-9   epilogue: tcgen05.ld of the group's buffer (lane quarter = warp % 4, column half = (warp-2)/4),
//               scale and accumulate in registers
// Grid (S, row tiles, token tiles) with clusters of S CTAs along K: the S CTAs of a cluster each reduce a
// contiguous range of groups; their partial tiles meet in distributed shared memory and CTA c sums token rows
// [c*NT/S, (c+1)*NT/S) over the S partials in cluster-rank order (a fixed order: the bits do not depend on
// timing) and runs the store or silu(gate)*up epilogue. No workspace, no second launch, no atomics.
// The GEMM is launched with programmatic stream serialization behind its activation quantizer: the CTA's prologue
// and its first weight stages overlap the quantizer, and only the activation tiles and scales wait for it
// (griddepcontrol.wait). Every mbarrier wait is bounded (%globaltimer); a timeout records an error code, the CTA
// waits (bounded) for its copies and MMAs in flight, frees its TMEM and leaves without storing.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cudaTypedefs.h>
#include <cstdint>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "ptx.cuh"
#include "wgemm.h"

namespace fw {
namespace f8 {

constexpr int kAcc = 4;                  // TMEM accumulator ring (one 128 x NT fp32 buffer per group in flight)
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;
constexpr int kWBytes = 128 * 128;       // weight tile: 128 rows x 128 e4m3

struct Args {
  int R, K, KB, T;
  int splits;                            // CTAs per cluster along K
  const float* wscale;                   // [ceil(R/128), KB]
  const float* xscale;                   // [KB, xs_ld]
  int xs_ld;                             // >= token tiles * NT, multiple of 4
  void* out;
  int out_ld, out_cols, out_dtype, epi, accumulate;
  float alpha;
  int* err;
  unsigned long long timeout_ns;
};

template <int NT>
struct Cfg {
  static constexpr int kXBytes = NT * 128;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  static constexpr int kStages = NT == 128 ? 6 : 8;
  static constexpr int kTmemCols = kAcc * NT < 32 ? 32 : kAcc * NT;
  static constexpr int kBarBytes = 8 * (2 * kStages + 2 * kAcc) + 16;
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + kBarBytes;
  static_assert(NT * 128 * 4 <= kStages * kStageBytes, "partial tile must fit over the stage ring");
};

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_cluster_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Wait for a phase without looking at the abort flag (used to drain copies and MMAs after an abort).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return;
  }
}

__device__ __forceinline__ void store_out(const Args& a, int tok, int col, float v) {
  if (a.out_dtype == WGEMM_OUT_F32) {
    float* p = reinterpret_cast<float*>(a.out) + (size_t)tok * a.out_ld + col;
    *p = a.accumulate ? *p + v : v;
  } else if (a.out_dtype == WGEMM_OUT_BF16) {
    reinterpret_cast<__nv_bfloat16*>(a.out)[(size_t)tok * a.out_ld + col] = __float2bfloat16(v);
  } else {
    reinterpret_cast<__half*>(a.out)[(size_t)tok * a.out_ld + col] = __float2half(v);
  }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
    f8gemm_kernel(const Args a, const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap) {
  using C = Cfg<NT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + C::kStages * C::kStageBytes;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (C::kStages + s); };
  auto accf = [&](int b) { return bars + 8u * (2 * C::kStages + b); };
  auto acce = [&](int b) { return bars + 8u * (2 * C::kStages + kAcc + b); };
  const uint32_t tmem_slot = bars + 8u * (2 * C::kStages + 2 * kAcc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (tmem_slot + 4 - base));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.splits;
  const int split = blockIdx.x, rb = blockIdx.y, tt = blockIdx.z;
  const int kb0 = (int)((int64_t)split * a.KB / S), kb1 = (int)((int64_t)(split + 1) * a.KB / S);
  const int n_kb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(accf(b), 1);
      mbar_init(acce(b), kEpiThreads / 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
  }
  if (warp == 1) tmem_alloc_dyn(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));
  const uint64_t lim = a.timeout_ns;

  int issued = 0;                        // producer: stages issued; MMA: groups issued
  float acc[NT / 2];
#pragma unroll
  for (int j = 0; j < NT / 2; ++j) acc[j] = 0.f;
  const int q = warp & 3;                // TMEM lane quarter this warp may access
  const int h = (warp - 2) >> 2;         // column half of the epilogue warps

  if (warp == 0) {
    if (lane == 0) {
      // The weights do not depend on the previous kernel (the activation quantizer): their first stages are in
      // flight before the wait for its results, the activation tiles of those stages follow it.
      const int pre = n_kb < C::kStages ? n_kb : C::kStages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(full(i), C::kStageBytes);
        tma_load_2d(base + i * C::kStageBytes, &wmap, (kb0 + i) * 128, rb * 128, full(i));
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(base + i * C::kStageBytes + kWBytes, &xmap, (kb0 + i) * 128, tt * NT, full(i));
      issued = pre;
      for (int i = pre; i < n_kb; ++i) {
        const int s = i % C::kStages;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
        if (!mbar_wait_sleepy(empty(s), ph ^ 1u, a.err, 7101, abort_flag, lim, 2000u)) break;
        const uint32_t st = base + s * C::kStageBytes;
        mbar_arrive_expect_tx(full(s), C::kStageBytes);
        tma_load_2d(st, &wmap, (kb0 + i) * 128, rb * 128, full(s));
        tma_load_2d(st + kWBytes, &xmap, (kb0 + i) * 128, tt * NT, full(s));
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(128, NT, 0);   // A, B e4m3 (format 0), D fp32, K-major
      for (int i = 0; i < n_kb; ++i) {
        const int s = i % C::kStages, b = i % kAcc;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u, bph = (uint32_t)(i / kAcc) & 1u;
        if (!mbar_wait(full(s), ph, a.err, 7102, abort_flag, lim)) break;
        if (!mbar_wait(acce(b), bph ^ 1u, a.err, 7103, abort_flag, lim)) break;
        tc_fence_after();
        const uint32_t st = base + s * C::kStageBytes;
        const uint64_t ad = umma_desc_sw128(st), bd = umma_desc_sw128(st + kWBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f8(tmem + b * NT, ad + 2 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
        umma_commit(empty(s));
        umma_commit(accf(b));
        issued = i + 1;
      }
    }
  } else {
    pdl_wait();                          // activation scales (and an accumulated output) come from earlier kernels
    const float* xs_base = a.xscale + tt * NT + h * (NT / 2);
    const float* ws_row = a.wscale + (size_t)rb * a.KB;
    // The group's scales (its weight block's, and the NT/2 activation scales of this thread's token half) are in
    // registers before the group's accumulator is: loaded one group ahead (two when NT <= 64, where the registers
    // allow), so their latency overlaps the wait instead of following it.
    constexpr int NC = NT / 8;
    constexpr bool kAhead = NT <= 64;
    float4 cn[NC];
    float swn = 0.f;
    if (kAhead && n_kb > 0) {
      const float4* x0 = reinterpret_cast<const float4*>(xs_base + (size_t)kb0 * a.xs_ld);
#pragma unroll
      for (int m = 0; m < NC; ++m) cn[m] = __ldg(x0 + m);
      swn = __ldg(ws_row + kb0);
    }
    for (int i = 0; i < n_kb; ++i) {
      const int b = i % kAcc, kb = kb0 + i;
      const uint32_t bph = (uint32_t)(i / kAcc) & 1u;
      float4 cc[NC];
      float sw;
      if constexpr (kAhead) {
#pragma unroll
        for (int m = 0; m < NC; ++m) cc[m] = cn[m];
        sw = swn;
        if (i + 1 < n_kb) {
          const float4* xn = reinterpret_cast<const float4*>(xs_base + (size_t)(kb + 1) * a.xs_ld);
#pragma unroll
          for (int m = 0; m < NC; ++m) cn[m] = __ldg(xn + m);
          swn = __ldg(ws_row + kb + 1);
        }
      } else {
        const float4* xs4 = reinterpret_cast<const float4*>(xs_base + (size_t)kb * a.xs_ld);
#pragma unroll
        for (int m = 0; m < NC; ++m) cc[m] = __ldg(xs4 + m);
        sw = __ldg(ws_row + kb);
      }
      if (!mbar_wait_warp(accf(b), bph, a.err, 7104, abort_flag, lim)) break;
      tc_fence_after();
      uint32_t v[NT / 32][16];
#pragma unroll
      for (int c = 0; c < NT / 32; ++c)
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * NT + h * (NT / 2) + 16 * c), v[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce(b));
#pragma unroll
      for (int m = 0; m < NC; ++m) {
        const float4 c4 = cc[m];
        const int j = 4 * m;
        acc[j + 0] = fmaf(__uint_as_float(v[j >> 4][(j + 0) & 15]), sw * c4.x, acc[j + 0]);
        acc[j + 1] = fmaf(__uint_as_float(v[j >> 4][(j + 1) & 15]), sw * c4.y, acc[j + 1]);
        acc[j + 2] = fmaf(__uint_as_float(v[j >> 4][(j + 2) & 15]), sw * c4.z, acc[j + 2]);
        acc[j + 3] = fmaf(__uint_as_float(v[j >> 4][(j + 3) & 15]), sw * c4.w, acc[j + 3]);
      }
    }
  }
  __syncwarp();
  // After an abort, copies and MMAs still in flight must land before the stage ring is reused or TMEM freed.
  if (*abort_flag && lane == 0) {
    if (warp == 0)
      for (int i = issued > C::kStages ? issued - C::kStages : 0; i < issued; ++i)
        drain_wait(full(i % C::kStages), (uint32_t)(i / C::kStages) & 1u, lim);
    if (warp == 1 && issued > 0)
      drain_wait(accf((issued - 1) % kAcc), (uint32_t)((issued - 1) / kAcc) & 1u, lim);
  }
  __syncthreads();                       // the ring is drained: its memory now holds the partial tile
  const uint32_t P = base;               // fp32 [NT tokens][128 rows]
  if (warp >= 2 && !*abort_flag) {
    const int row = q * 32 + lane;
#pragma unroll
    for (int j = 0; j < NT / 2; ++j) st_shared_f32(P + (uint32_t)(((h * (NT / 2) + j) * 128 + row) * 4), acc[j]);
  }
  if (S > 1) cluster_sync_all(); else __syncthreads();

  const int rank = S > 1 ? (int)cluster_rank() : 0;
  const int t_lo = rank * NT / S, t_hi = (rank + 1) * NT / S;
  const bool ok = !*abort_flag;
  if (a.epi == WGEMM_EPI_STORE) {
    const int n = (t_hi - t_lo) * 32;
    for (int e = threadIdx.x; e < n && ok; e += kThreads) {
      const int t = t_lo + e / 32, r4 = (e % 32) * 4;
      const uint32_t off = (uint32_t)((t * 128 + r4) * 4);
      float4 s4 = S > 1 ? ld_cluster_v4(map_rank(P + off, 0)) : ld_shared_v4(P + off);
      for (int p = 1; p < S; ++p) {
        const float4 o = ld_cluster_v4(map_rank(P + off, p));
        s4.x += o.x; s4.y += o.y; s4.z += o.z; s4.w += o.w;
      }
      const int tok = tt * NT + t, row = rb * 128 + r4;
      if (tok >= a.T) continue;
      const float vv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (row + u < a.out_cols) store_out(a, tok, row + u, vv[u] * a.alpha);
    }
  } else {                               // silu(gate) * up: rows 0..63 of the tile are gates, 64..127 the ups
    const int n = (t_hi - t_lo) * 16;
    for (int e = threadIdx.x; e < n && ok; e += kThreads) {
      const int t = t_lo + e / 16, f4 = (e % 16) * 4;
      const uint32_t og = (uint32_t)((t * 128 + f4) * 4), ou = og + 64 * 4;
      float4 g = S > 1 ? ld_cluster_v4(map_rank(P + og, 0)) : ld_shared_v4(P + og);
      float4 u = S > 1 ? ld_cluster_v4(map_rank(P + ou, 0)) : ld_shared_v4(P + ou);
      for (int p = 1; p < S; ++p) {
        const float4 g2 = ld_cluster_v4(map_rank(P + og, p)), u2 = ld_cluster_v4(map_rank(P + ou, p));
        g.x += g2.x; g.y += g2.y; g.z += g2.z; g.w += g2.w;
        u.x += u2.x; u.y += u2.y; u.z += u2.z; u.w += u2.w;
      }
      const int tok = tt * NT + t, col = rb * 64 + f4;
      if (tok >= a.T) continue;
      const float gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int w = 0; w < 4; ++w)
        if (col + w < a.out_cols) store_out(a, tok, col + w, silu_f(gg[w]) * uu[w]);
    }
  }
  if (S > 1) cluster_sync_all();         // peers may still read this CTA's partial tile
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------ activation quantization
// One warp per (token, 128-column group); lane l owns columns 4l..4l+3. scale = absmax / 448 (0 for an all-zero
// group); codes = e4m3(x * 448 / absmax), round to nearest even, saturating. Tokens T..T_pad-1 get zero codes
// and scale 0 (the token tiles' padding rows, so no TMA box is taller than its tensor).
template <typename TIn>
__device__ __forceinline__ float4 load4(const TIn* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(u32_as_h2(u.x)), b = __half22float2(u32_as_h2(u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

template <typename TIn>
__global__ void __launch_bounds__(256) f8_quant_kernel(const TIn* __restrict__ x, int T, int KB, int x_ld,
                                                       uint8_t* __restrict__ x8, float* __restrict__ xs, int xs_ld,
                                                       int T_pad) {
  pdl_launch_dependents();              // the GEMM may start its prologue and weight loads now
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int t = gw / KB, kb = gw % KB;
  if (t >= T_pad) return;
  if (t >= T) {
    reinterpret_cast<uint32_t*>(x8 + (size_t)t * KB * 128 + kb * 128)[lane] = 0u;
    if (lane == 0) xs[(size_t)kb * xs_ld + t] = 0.f;
    return;
  }
  const float4 v = load4<TIn>(x + (size_t)t * x_ld + kb * 128 + 4 * lane);
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const float inv = m > 0.f ? 448.f / m : 0.f;
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v.x * inv, v.y * inv), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v.z * inv, v.w * inv), __NV_SATFINITE, __NV_E4M3);
  reinterpret_cast<uint32_t*>(x8 + (size_t)t * KB * 128 + kb * 128)[lane] = (uint32_t)lo | ((uint32_t)hi << 16);
  if (lane == 0) xs[(size_t)kb * xs_ld + t] = m / 448.f;
}

// ------------------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// uint8 [rows, cols] row-major, box [box_rows, 128 B], 128-byte swizzle (rows past `rows` read as zero).
static int tmap_u8(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  auto enc = encoder();
  if (!enc) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return (int)enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int NT>
static int launch(const Args& a, const CUtensorMap& wm, const CUtensorMap& xm, int row_tiles, int tok_tiles,
                  cudaStream_t st, bool pdl) {
  using C = Cfg<NT>;
  auto k = f8gemm_kernel<NT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  if (e != cudaSuccess) return (int)e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, row_tiles, tok_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl) {                             // overlap the prologue and the first weight stages with the quantizer
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (a.splits > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = a.splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  e = cudaLaunchKernelEx(&cfg, k, a, wm, xm);
  return (int)(e != cudaSuccess ? e : cudaGetLastError());
}

}  // namespace f8
}  // namespace fw

namespace {

// y = x @ W^T (epi 0) or silu(gate) * up over the silu-pair row order (epi 1) with W given as e4m3 codes
// w8 [Rp, K] (Rp a multiple of 128, rows >= `rows` zero) and fp32 block scales [Rp/128, K/128]; x [T, K]
// fp16 / bf16 / fp32. Quantizes x per 128-column group, then runs the FP8 GEMM. Returns the launch count.
int64_t f8_linear(torch::Tensor x, torch::Tensor w8, torch::Tensor wscale, int64_t rows, torch::Tensor out,
                  int64_t epi, bool accumulate, double alpha, int64_t nt, int64_t splits, torch::Tensor err,
                  int64_t timeout_ns) {
  TORCH_CHECK(x.is_cuda() && w8.is_cuda() && wscale.is_cuda() && out.is_cuda() && err.is_cuda(), "CUDA tensors");
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be a contiguous [T, K] matrix");
  TORCH_CHECK(w8.scalar_type() == torch::kUInt8 && w8.dim() == 2 && w8.is_contiguous(), "w8 must be uint8 [Rp, K]");
  TORCH_CHECK(wscale.scalar_type() == torch::kFloat && wscale.is_contiguous(), "wscale must be fp32");
  TORCH_CHECK(err.scalar_type() == torch::kInt32, "err must be int32");
  const int64_t T = x.size(0), K = x.size(1), Rp = w8.size(0);
  TORCH_CHECK(K % 128 == 0 && w8.size(1) == K, "K must be a multiple of 128 and match the weight");
  TORCH_CHECK(Rp % 128 == 0 && rows <= Rp && rows > 0, "weight rows must be padded to a multiple of 128");
  TORCH_CHECK(wscale.numel() == (Rp / 128) * (K / 128), "wscale must be [Rp/128, K/128]");
  TORCH_CHECK(((uintptr_t)w8.data_ptr()) % 16 == 0 && ((uintptr_t)x.data_ptr()) % 16 == 0, "16-byte alignment");
  TORCH_CHECK(nt == 32 || nt == 64 || nt == 128, "nt must be 32, 64 or 128");
  const int64_t KB = K / 128;
  TORCH_CHECK(splits >= 1 && splits <= 8 && splits <= KB, "splits must be in [1, min(8, K/128)]");
  TORCH_CHECK(epi == fw::WGEMM_EPI_STORE || (epi == fw::WGEMM_EPI_SILU_MUL && rows % 128 == 0), "bad epilogue");
  const int64_t cols = epi == fw::WGEMM_EPI_SILU_MUL ? rows / 2 : rows;
  TORCH_CHECK(out.dim() == 2 && out.size(0) == T && out.size(1) >= cols && out.stride(1) == 1, "out must be [T, cols]");
  int out_dtype;
  if (out.scalar_type() == torch::kFloat) out_dtype = fw::WGEMM_OUT_F32;
  else if (out.scalar_type() == torch::kBFloat16) out_dtype = fw::WGEMM_OUT_BF16;
  else if (out.scalar_type() == torch::kHalf) out_dtype = fw::WGEMM_OUT_F16;
  else TORCH_CHECK(false, "out must be fp32/bf16/fp16");
  TORCH_CHECK(!accumulate || out_dtype == fw::WGEMM_OUT_F32, "accumulate needs an fp32 output");
  if (T == 0) return 0;
  const c10::cuda::CUDAGuard guard(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const int64_t tok_tiles = (T + nt - 1) / nt, T_pad = tok_tiles * nt;
  auto x8 = torch::empty({T_pad, K}, x.options().dtype(torch::kUInt8));
  auto xs = torch::empty({KB, T_pad}, x.options().dtype(torch::kFloat));
  const int64_t warps = T_pad * KB;
  const int qb = (int)((warps + 7) / 8);
  if (x.scalar_type() == torch::kHalf)
    fw::f8::f8_quant_kernel<__half><<<qb, 256, 0, st>>>(reinterpret_cast<const __half*>(x.data_ptr()), (int)T,
        (int)KB, (int)K, x8.data_ptr<uint8_t>(), xs.data_ptr<float>(), (int)T_pad, (int)T_pad);
  else if (x.scalar_type() == torch::kBFloat16)
    fw::f8::f8_quant_kernel<__nv_bfloat16><<<qb, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), (int)T, (int)KB, (int)K, x8.data_ptr<uint8_t>(),
        xs.data_ptr<float>(), (int)T_pad, (int)T_pad);
  else if (x.scalar_type() == torch::kFloat)
    fw::f8::f8_quant_kernel<float><<<qb, 256, 0, st>>>(x.data_ptr<float>(), (int)T, (int)KB, (int)K,
        x8.data_ptr<uint8_t>(), xs.data_ptr<float>(), (int)T_pad, (int)T_pad);
  else TORCH_CHECK(false, "x must be fp16/bf16/fp32");
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "f8 activation quantization launch failed");
  CUtensorMap wm, xm;
  TORCH_CHECK(fw::f8::tmap_u8(&wm, w8.data_ptr(), Rp, K, 128) == 0, "weight tensor map");
  TORCH_CHECK(fw::f8::tmap_u8(&xm, x8.data_ptr(), T_pad, K, (uint32_t)nt) == 0, "activation tensor map");
  fw::f8::Args a{};
  a.R = (int)rows; a.K = (int)K; a.KB = (int)KB; a.T = (int)T; a.splits = (int)splits;
  a.wscale = wscale.data_ptr<float>(); a.xscale = xs.data_ptr<float>(); a.xs_ld = (int)T_pad;
  a.out = out.data_ptr(); a.out_ld = (int)out.stride(0); a.out_cols = (int)cols; a.out_dtype = out_dtype;
  a.epi = (int)epi; a.accumulate = accumulate ? 1 : 0; a.alpha = (float)alpha;
  a.err = err.data_ptr<int32_t>(); a.timeout_ns = (unsigned long long)timeout_ns;
  const int rt = (int)(Rp / 128);
  static const bool pdl = !(getenv("FW_PDL") && atoi(getenv("FW_PDL")) == 0);   // FW_PDL=0: plain launches
  int rc;
  if (nt == 32) rc = fw::f8::launch<32>(a, wm, xm, rt, (int)tok_tiles, st, pdl);
  else if (nt == 64) rc = fw::f8::launch<64>(a, wm, xm, rt, (int)tok_tiles, st, pdl);
  else rc = fw::f8::launch<128>(a, wm, xm, rt, (int)tok_tiles, st, pdl);
  TORCH_CHECK(rc == 0, "f8gemm launch failed: ", cudaGetErrorString((cudaError_t)rc));
  return 2;
}

}  // namespace

// How many clusters of `splits` CTAs of the nt-token GEMM can be resident at once on the current device
// (cudaOccupancyMaxActiveClusters): a launch plan whose clusters exceed it runs in more than one wave.
int64_t f8_max_clusters(int64_t nt, int64_t splits) {
  TORCH_CHECK(nt == 32 || nt == 64 || nt == 128, "nt must be 32, 64 or 128");
  TORCH_CHECK(splits >= 1 && splits <= 8, "splits must be in [1, 8]");
  auto query = [&](auto kernel, size_t smem) -> int64_t {
    TORCH_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess,
                "f8gemm shared memory attribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)splits, 1, 1);
    cfg.blockDim = dim3(fw::f8::kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    TORCH_CHECK(e == cudaSuccess, "cudaOccupancyMaxActiveClusters: ", cudaGetErrorString(e));
    return n;
  };
  if (nt == 32) return query(fw::f8::f8gemm_kernel<32>, fw::f8::Cfg<32>::kSmem);
  if (nt == 64) return query(fw::f8::f8gemm_kernel<64>, fw::f8::Cfg<64>::kSmem);
  return query(fw::f8::f8gemm_kernel<128>, fw::f8::Cfg<128>::kSmem);
}

void register_f8gemm(pybind11::module& m) {
  m.def("f8_linear", &f8_linear, "dense FP8 GEMM (tcgen05 kind::f8f6f4) with per-group FP8 activations");
  m.def("f8_max_clusters", &f8_max_clusters, "co-resident clusters of the FP8 GEMM for a token tile and K split");
}
