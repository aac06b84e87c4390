// Latent (MLA) attention over FP8 cache rows on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Per query row t (a decode token or one row of a prefill chunk) and head h:
//     s_j = (q_lat[h] . c_j[:kvr] + q_pe[h] . c_j[kvr:]) * scale,   o[h] = sum_j softmax(s)_j c_j[:kvr]
// over the rows j of the DSA top-k list, the sliding window, or all causal rows. Every head reads the same
// rows (multi-query form of MLA), so per 32-key chunk the work is two small GEMMs:
//     S   [heads x keys]  = Q [heads x D] . K^T           (M = 64 head rows, N = 32 keys, K = D = kvr + dr)
//     O^T [kvr x heads]  += V^T [kvr x keys] . P^T         (M = 128 latent dims per tile, N = heads, K = 32 keys)
// Heads are the M rows of the score MMA (M = 64: head 16w + l sits in TMEM lane 32w + l), so each softmax thread
// owns one head's scores and runs the online softmax without cross-thread reductions. The P.V product is written
// transposed so that O for up to 64 heads x 512 latent dims fits in TMEM next to two score buffers, and so that
// V^T is the same shared-memory tile as the key chunk, read as an MN-major operand: one fp8 -> fp16 conversion
// per chunk feeds both MMAs.
//
// CTA = (row t, head group, key split); warp-specialized pipeline over chunks i:
//   warp 8      loader: resolves the chunk's 32 key positions to cache rows (DSA list / window / causal, paged
//               block table) and fetches each FP8 row with a 1-D bulk copy into a ring stage
//   warps 4-7   convert stage -> fp16 key tile K[i & 1] (128-byte-swizzled K-major), record the key mask
//   warp 9      MMA issuer (one thread): S(i) as soon as K[i & 1] is ready, then P.V(i - 1) once P(i - 1) is,
//               so the score MMA of the next chunk runs under the softmax of the current one
//   warps 0-3   softmax (lanes 0-15 = heads) into P[i & 1], lazy O rescale (only when a head's max grows by more
//               than 2^8; waits for the previous P.V), epilogue (lanes = latent dims)
// Q is staged once per CTA with only the group's heads; the score MMA's rows past them read the following shared
// memory and produce rows that are never used. Key splits write unnormalized partials (O, running max, sum)
// merged by mla_tc_combine_kernel. Every wait is bounded (%globaltimer); a timeout records an error code, each
// role drains out, the loader waits for its copies in flight and the MMA thread for its last MMAs, and TMEM is
// released before the CTA exits.
//
// Replaces the reference's CUDA-core sparse MLA decode (dotsnote/engine/arcstats_pkg/arcstats/csrc/
// offload_attn.cu, K2 "v5": 576-byte FP8 rows, online softmax over the selected rows) and the window-513 SWA
// kernel (arcstats/csrc/swa_attn.cu, 1088-byte rows); math of dotsnote/training/finetune/student.py:209-259.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cfloat>
#include "ptx.cuh"

namespace {

using namespace fw;

#define STREAM at::cuda::getCurrentCUDAStream()

constexpr int NK = 32;           // keys per chunk
constexpr int kThreads = 320;    // warps 0-3 softmax/epilogue, 4-7 convert, 8 load, 9 MMA
constexpr int kMaxStages = 3;
constexpr int kMaxKB = 17;       // D / 64 <= 17 (kvr <= 1024, dr = 64)
constexpr float kRescaleLog2 = 8.f;
constexpr int NACC = 4;          // interleaved score accumulators: consecutive MMAs do not wait on each other
static_assert(NK * 4 == 128, "the conversion maps 4 threads to each key of a chunk");

struct MlaTcArgs {
  const __nv_bfloat16* q_lat;   // [H, T, kvr]
  const float* q_pe;            // [T, H, dr]
  const uint8_t* cache;         // [n_blocks * bs, D] FP8 e4m3 rows
  const int* block_table;
  int max_blocks, bs;
  const int *slots, *positions;
  int n_tok;
  const int* sel;               // [T, topk] positions (first entry -1 = no list) or null
  int topk, window;
  int T, H, kvr, dr, D;
  int HGp;                      // heads per CTA (multiple of 16, <= 64)
  int splits, stages;
  float scale_log2;
  __nv_bfloat16* o_lat;         // [H, T, kvr] when splits == 1
  float* part_o;                // [splits, T, H, kvr]
  float* part_ml;               // [splits, T, H, 2]
  int* err;
  uint64_t timeout_ns;
  unsigned long long* trace;    // optional: phase timestamps of CTA (0, 0, 0), [chunk][8]
};

// barrier indices (8 bytes each)
enum : int {
  kRawFull = 0,                  // [kMaxStages] loader -> converters (tx bytes)
  kRawEmpty = kMaxStages,        // [kMaxStages] converters -> loader (4 warps)
  kKcFull = 2 * kMaxStages,      // [2] converters -> MMA, softmax (4 warps)
  kKcEmpty = kKcFull + 2,        // [2] MMA commit after P.V(i) -> converters
  kSFull = kKcEmpty + 2,         // [2] MMA commit after S(i) -> softmax
  kPFull = kSFull + 2,           // [2] softmax -> MMA (4 warps)
  kPvDone = kPFull + 2,          // MMA commit after every P.V
  kNumBars = kPvDone + 1
};

struct Smem {                   // byte offsets from the 1024-aligned base
  uint32_t q, kc, p, raw, rows, vm, corr, lsum, bars, misc, total;
};

__host__ __device__ inline Smem smem_plan(int D, int HGp, int stages) {
  Smem s{};
  uint32_t o = 0;
  const uint32_t kc_bytes = (D / 64) * NK * 128, p_bytes = ((HGp * 128 + 1023) / 1024) * 1024;
  s.q = o;  o += (D / 64) * HGp * 128;
  s.kc = o; o += 2 * kc_bytes;
  s.p = o;  o += 2 * p_bytes;
  s.raw = o; o += ((stages * NK * D + 1023) / 1024) * 1024;
  // the score MMA reads 64 rows of Q from the last k-block: keep that window inside the allocation
  const uint32_t q_reach = s.q + (D / 64 - 1) * HGp * 128 + 64 * 128;
  if (o < q_reach) o = q_reach;
  s.rows = o; o += kMaxStages * NK * 4;
  s.vm = o; o += 2 * 4;
  s.corr = o; o += 64 * 4;
  s.lsum = o; o += 64 * 4;
  s.bars = o; o += kNumBars * 8;
  s.misc = o; o += 16;          // tmem base, abort word
  s.total = o + 1024;           // slack for aligning the dynamic base
  return s;
}

__device__ __forceinline__ bool bar_any(uint32_t id, uint32_t n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MN-major operand, 128-byte swizzle: atoms of 64 MN-elements (128 B) x 8 K-rows (1024 B); `lbo` = byte stride
// between atoms along MN, `sbo` = byte stride between 8-row groups along K.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// no "memory" clobber: the caller orders these loads against the loader's writes with the stage barrier
__device__ __forceinline__ uint4 lds128_nc(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t two) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xFFFF), __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

// 2^x with the MUFU approximation (inputs here are <= 8; -inf gives 0)
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

#define MLA_TRACE(chunk, slot)                                                                        \
  if (a.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (chunk) < 62)              \
    a.trace[(chunk) * 8 + (slot)] = globaltimer_ns();

__global__ void __launch_bounds__(kThreads, 1) mla_tc_kernel(const MlaTcArgs a) {
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t base = (smem_u32(smem_dyn) + 1023) & ~1023u;
  uint8_t* gbase = smem_dyn + (base - smem_u32(smem_dyn));
  const Smem L = smem_plan(a.D, a.HGp, a.stages);
  const uint32_t sQ = base + L.q, sK = base + L.kc, sP = base + L.p, sRaw = base + L.raw;
  const uint32_t kc_bytes = (a.D / 64) * NK * 128, p_bytes = ((a.HGp * 128 + 1023) / 1024) * 1024;
  int* rows = reinterpret_cast<int*>(gbase + L.rows);
  volatile unsigned* vm_sm = reinterpret_cast<volatile unsigned*>(gbase + L.vm);
  float* corr_sm = reinterpret_cast<float*>(gbase + L.corr);
  float* l_sm = reinterpret_cast<float*>(gbase + L.lsum);
  const uint32_t bars = base + L.bars;
  auto bar = [&](int i) -> uint32_t { return bars + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L.misc);
  volatile int* abort_w = reinterpret_cast<volatile int*>(gbase + L.misc + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x, g = blockIdx.y, sp = blockIdx.z;
  const int HGp = a.HGp, h0 = g * HGp, hn = min(HGp, a.H - h0);
  const int D = a.D, kvr = a.kvr, RS = a.stages, nkb = D / 64;
  const int b = t / a.n_tok;
  const int pos = a.positions[b] + t % a.n_tok, slot = a.slots[b];
  const int* sel = a.sel ? a.sel + (int64_t)t * a.topk : nullptr;
  const bool sparse = sel != nullptr && sel[0] >= 0;
  int lo = 0, n;
  if (sparse) {
    n = a.topk;
  } else {
    lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
    n = pos - lo + 1;
  }
  const int n_chunks = (n + NK - 1) / NK;
  const int per = (n_chunks + a.splits - 1) / a.splits;
  const int c0 = min(n_chunks, sp * per), nc = max(0, min(n_chunks, c0 + per) - c0);
  const int n_mt = kvr / 128;
  // TMEM: score buffer b, partial accumulator k at columns (b * NACC + k) * NK; O^T tiles from O0
  const uint32_t O0 = 2 * NACC * NK;

  if (tid == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(bar(kRawFull + s), 1);
      mbar_init(bar(kRawEmpty + s), 4);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(bar(kKcFull + k), 4);
      mbar_init(bar(kKcEmpty + k), 1);
      mbar_init(bar(kSFull + k), 1);
      mbar_init(bar(kPFull + k), 4);
    }
    mbar_init(bar(kPvDone), 1);
    *abort_w = 0;
    fence_mbar_init();
  }
  uint32_t tcols = 32;
  while (tcols < (uint32_t)(O0 + n_mt * HGp)) tcols <<= 1;
  if (warp == 0) tmem_alloc_dyn(smem_u32(tmem_slot), tcols);
  // Q (fp16, K-major, 128-byte swizzle, HGp rows per 64-column block); padding heads are zero. Loads are issued
  // eight units at a time so their latencies overlap.
  if (warp < 8) {
    const int cpr = D / 8, total = HGp * cpr;
    for (int i0 = tid; i0 < total; i0 += 256 * 8) {
      uint4 v0[8], v1[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        v0[k] = make_uint4(0u, 0u, 0u, 0u);
        v1[k] = make_uint4(0u, 0u, 0u, 0u);
        const int i = i0 + k * 256;
        if (i < total) {
          const int h = i / cpr, d0 = (i % cpr) * 8;
          if (h < hn) {
            if (d0 < kvr) {
              v0[k] = __ldg(reinterpret_cast<const uint4*>(a.q_lat + ((int64_t)(h0 + h) * a.T + t) * kvr + d0));
            } else {
              const uint4* src =
                  reinterpret_cast<const uint4*>(a.q_pe + ((int64_t)t * a.H + h0 + h) * a.dr + (d0 - kvr));
              v0[k] = __ldg(src);
              v1[k] = __ldg(src + 1);
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int i = i0 + k * 256;
        if (i < total) {
          const int h = i / cpr, d0 = (i % cpr) * 8;
          uint32_t w[4];
          if (d0 < kvr) {
            const uint32_t u[4] = {v0[k].x, v0[k].y, v0[k].z, v0[k].w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[q]));
              w[q] = pack_h2(f.x, f.y);
            }
          } else {
            w[0] = pack_h2(__uint_as_float(v0[k].x), __uint_as_float(v0[k].y));
            w[1] = pack_h2(__uint_as_float(v0[k].z), __uint_as_float(v0[k].w));
            w[2] = pack_h2(__uint_as_float(v1[k].x), __uint_as_float(v1[k].y));
            w[3] = pack_h2(__uint_as_float(v1[k].z), __uint_as_float(v1[k].w));
          }
          sts128(sQ + (d0 / 64) * HGp * 128 + h * 128 + ((((d0 & 63) >> 3) ^ (h & 7)) << 4), w[0], w[1], w[2],
                 w[3]);
        }
      }
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------------------------------ loader
    const uint64_t pol = a.H > HGp ? l2_policy_evict_last() : l2_policy_evict_first();
    auto resolve = [&](int c) -> int {
      const int kk = c * NK + lane;
      int p = -1;
      if (kk < n) p = sparse ? __ldg(sel + kk) : lo + kk;
      return p;
    };
    auto to_row = [&](int p) -> int {
      if (p < 0 || p > pos) return -1;
      return __ldg(a.block_table + (int64_t)slot * a.max_blocks + p / a.bs) * a.bs + p % a.bs;
    };
    int cr0 = -1, cr1 = -1, cr2 = -1, cr3 = -1;
    int issued = 0;
    for (int i = 0; i < nc; ++i) {
      const int s = i % RS;
      if ((i & 3) == 0) {  // four chunks resolved together: their dependent loads overlap
        const int p0 = resolve(c0 + i), p1 = i + 1 < nc ? resolve(c0 + i + 1) : -1,
                  p2 = i + 2 < nc ? resolve(c0 + i + 2) : -1, p3 = i + 3 < nc ? resolve(c0 + i + 3) : -1;
        cr0 = to_row(p0);
        cr1 = to_row(p1);
        cr2 = to_row(p2);
        cr3 = to_row(p3);
      }
      if (i >= RS && !mbar_wait_warp(bar(kRawEmpty + s), ((i / RS) - 1) & 1, a.err, 7101, abort_w, a.timeout_ns))
        break;
      if (*abort_w) break;
      const int q = i & 3;
      const int crow = q == 0 ? cr0 : q == 1 ? cr1 : q == 2 ? cr2 : cr3;
      rows[s * NK + lane] = crow;
      const unsigned m = __ballot_sync(0xffffffffu, crow >= 0);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(bar(kRawFull + s), (uint32_t)__popc(m) * (uint32_t)D);
      __syncwarp();
      if (crow >= 0)
        tma_bulk_g2s(sRaw + (s * NK + lane) * D, a.cache + (int64_t)crow * D, D, bar(kRawFull + s), pol);
      if (lane == 0) { MLA_TRACE(i, 0) }
      issued = i + 1;
    }
    // no copy may still be in flight when the CTA exits
    if (lane == 0)
      for (int i = max(0, issued - RS); i < issued; ++i) {
        volatile int no_abort = 0;
        mbar_wait(bar(kRawFull + i % RS), (i / RS) & 1, a.err, 7102, &no_abort, a.timeout_ns);
      }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------------------------------ converters
    const int tc = tid - 128, j = tc >> 2, q = tc & 3;
    const uint32_t c_lo = ((2 * q) ^ (j & 7)) << 4, c_hi = ((2 * q + 1) ^ (j & 7)) << 4;
    for (int i = 0; i < nc; ++i) {
      const int s = i % RS, kb2 = i & 1;
      if (!mbar_wait_warp(bar(kRawFull + s), (i / RS) & 1, a.err, 7103, abort_w, a.timeout_ns)) break;
      // the whole row slice of this thread into registers, then the stage is free for the loader
      const int row = rows[s * NK + j];
      const unsigned vmask = __ballot_sync(0xffffffffu, rows[s * NK + lane] >= 0);
      uint4 v[kMaxKB];
      const uint32_t src = sRaw + (s * NK + j) * D + q * 16;
#pragma unroll
      for (int kb = 0; kb < kMaxKB; ++kb)
        v[kb] = (kb < nkb && row >= 0) ? lds128_nc(src + kb * 64) : make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kRawEmpty + s));
      if (i >= 2 && !mbar_wait_warp(bar(kKcEmpty + kb2), ((i >> 1) - 1) & 1, a.err, 7104, abort_w, a.timeout_ns))
        break;
      if (i < 62 && tc == 0) { MLA_TRACE(i, 1) }
      const uint32_t dst = sK + kb2 * kc_bytes + j * 128;
#pragma unroll
      for (int kb = 0; kb < kMaxKB; ++kb) {
        if (kb < nkb) {
          const uint32_t r = dst + kb * (NK * 128);
          sts128(r + c_lo, fp8x2_to_h2(v[kb].x), fp8x2_to_h2(v[kb].x >> 16), fp8x2_to_h2(v[kb].y),
                 fp8x2_to_h2(v[kb].y >> 16));
          sts128(r + c_hi, fp8x2_to_h2(v[kb].z), fp8x2_to_h2(v[kb].z >> 16), fp8x2_to_h2(v[kb].w),
                 fp8x2_to_h2(v[kb].w >> 16));
        }
      }
      if (tc == 0) vm_sm[kb2] = vmask;
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kKcFull + kb2));
      if (tc == 0) { MLA_TRACE(i, 2) }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(64, NK, 0);
      const uint32_t idesc_pv = umma_idesc_f16(128, HGp, 0) | (1u << 15);  // A (V^T) MN-major
      const uint64_t qd0 = umma_desc_sw128(sQ);
      int s_issued = 0, pv_issued = 0;
      for (int i = 0; i <= nc; ++i) {
        if (i < nc) {
          const int kb2 = i & 1;
          if (!mbar_wait(bar(kKcFull + kb2), (i >> 1) & 1, a.err, 7105, abort_w, a.timeout_ns)) break;
          MLA_TRACE(i, 7)
          tc_fence_after();
          const uint64_t kd0 = umma_desc_sw128(sK + kb2 * kc_bytes);
          // the 16-wide K steps of each 64-column block go to NACC separate accumulators (summed by the softmax)
          const uint32_t d_s = tmem + kb2 * NACC * NK;
          for (int kb = 0; kb < nkb; ++kb) {
            const uint64_t qd = qd0 + (uint64_t)((kb * HGp * 128) >> 4), kd = kd0 + (uint64_t)((kb * NK * 128) >> 4);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4)
              umma_f16(d_s + (k4 % NACC) * NK, qd + 2 * k4, kd + 2 * k4, idesc_s, (kb > 0 || k4 >= NACC) ? 1u : 0u);
          }
          umma_commit(bar(kSFull + kb2));
          s_issued = i + 1;
          MLA_TRACE(i, 3)
        }
        if (i > 0) {
          const int pi = i - 1, pb = pi & 1;
          if (!mbar_wait(bar(kPFull + pb), (pi >> 1) & 1, a.err, 7106, abort_w, a.timeout_ns)) break;
          tc_fence_after();
          const uint64_t ad0 = umma_desc_sw128_mn(sK + pb * kc_bytes, NK * 128, 1024);
          const uint64_t bd0 = umma_desc_sw128(sP + pb * p_bytes);
#pragma unroll
          for (int ks = 0; ks < NK / 16; ++ks)  // tiles inner: consecutive MMAs write different accumulators
            for (int mt = 0; mt < n_mt; ++mt)
              umma_f16(tmem + O0 + mt * HGp, ad0 + (uint64_t)(((2 * mt) * NK * 128 + (2 * ks) * 1024) >> 4),
                       bd0 + 2 * ks, idesc_pv, (pi > 0 || ks > 0) ? 1u : 0u);
          umma_commit(bar(kKcEmpty + pb));
          umma_commit(bar(kPvDone));
          pv_issued = pi + 1;
          MLA_TRACE(pi, 6)
        }
      }
      // every issued MMA has finished before TMEM is released
      volatile int no_abort = 0;
      if (pv_issued > 0) mbar_wait(bar(kPvDone), (pv_issued - 1) & 1, a.err, 7107, &no_abort, a.timeout_ns);
      if (s_issued > pv_issued)
        mbar_wait(bar(kSFull + ((s_issued - 1) & 1)), ((s_issued - 1) >> 1) & 1, a.err, 7108, &no_abort,
                  a.timeout_ns);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------------------------ softmax + epilogue
    float m_run = -INFINITY, l_run = 0.f;
    const int h = warp * 16 + lane;              // M = 64 score rows: head 16w + l in TMEM lane 32w + l
    const bool head_lane = lane < 16 && h < HGp;
    bool failed = false;
    int done = 0;
    for (int i = 0; i < nc; ++i) {
      const int kb2 = i & 1;
      bool ok = mbar_wait_warp(bar(kSFull + kb2), (i >> 1) & 1, a.err, 7109, abort_w, a.timeout_ns);
      if (ok) ok = mbar_wait_warp(bar(kKcFull + kb2), (i >> 1) & 1, a.err, 7110, abort_w, a.timeout_ns);
      if (bar_any(1, 128, !ok || *abort_w)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (tid == 0) { MLA_TRACE(i, 4) }
      const unsigned vmask = vm_sm[kb2];
      float sv[NK];
      {
        const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + kb2 * NACC * NK;
        uint32_t r[NACC][NK];
#pragma unroll
        for (int k = 0; k < NACC; ++k) {
          tmem_ld16(ta + k * NK, *reinterpret_cast<uint32_t(*)[16]>(&r[k][0]));
          tmem_ld16(ta + k * NK + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[k][16]));
        }
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < NK; ++jj) {
          float x = 0.f;
#pragma unroll
          for (int k = 0; k < NACC; ++k) x += __uint_as_float(r[k][jj]);
          sv[jj] = ((vmask >> jj) & 1u) ? x * a.scale_log2 : -INFINITY;
        }
      }
      bool need = false;
      if (head_lane) {
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int jj = 0; jj < NK; ++jj) mx4[jj & 3] = fmaxf(mx4[jj & 3], sv[jj]);
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        float corr = 1.f;
        if (mx > m_run + kRescaleLog2) {   // also true when m_run is -inf and the chunk has a valid key
          corr = m_run == -INFINITY ? 0.f : ex2_fast(m_run - mx);
          m_run = mx;
          need = i > 0;
        }
        uint32_t pw[NK / 2];
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        // padding heads, and heads with no valid key yet: every p is exp2(-inf) = 0
        const float mref = (h < hn && m_run != -INFINITY) ? m_run : INFINITY;
#pragma unroll
        for (int jj = 0; jj < NK; jj += 2) {
          const float p0 = ex2_fast(sv[jj] - mref), p1 = ex2_fast(sv[jj + 1] - mref);
          const __half2 hp = __floats2half2_rn(p0, p1);
          const float2 back = __half22float2(hp);
          sum4[(jj >> 1) & 3] += back.x + back.y;
          pw[jj / 2] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        l_run = l_run * corr + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
        corr_sm[h] = corr;
        const uint32_t prow = sP + kb2 * p_bytes + h * 128;
#pragma unroll
        for (int c = 0; c < NK / 8; ++c)
          sts128(prow + ((c ^ (h & 7)) << 4), pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      }
      if (bar_any(1, 128, need)) {
        // O^T[:, h] *= corr[h] once the previous P.V has landed (each lane is one latent dim of each tile)
        ok = mbar_wait_warp(bar(kPvDone), (i - 1) & 1, a.err, 7111, abort_w, a.timeout_ns);
        if (bar_any(1, 128, !ok)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t to = tmem + ((uint32_t)(warp * 32) << 16) + O0;
        for (int mt = 0; mt < n_mt; ++mt)
          for (int c16 = 0; c16 < HGp / 16; ++c16) {
            uint32_t r[16];
            tmem_ld16(to + mt * HGp + c16 * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 16; ++k) r[k] = __float_as_uint(__uint_as_float(r[k]) * corr_sm[c16 * 16 + k]);
            tmem_st16(to + mt * HGp + c16 * 16, r);
          }
        tmem_st_wait();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kPFull + kb2));
      if (tid == 0) { MLA_TRACE(i, 5) }
      done = i + 1;
    }
    // last P.V done
    bool have_o = false;
    if (!failed && done == nc && nc > 0)
      have_o = mbar_wait_warp(bar(kPvDone), (nc - 1) & 1, a.err, 7112, abort_w, a.timeout_ns);
    have_o = !bar_any(1, 128, !have_o);
    tc_fence_after();
    if (head_lane) l_sm[h] = l_run;
    named_barrier(1, 128);
    // epilogue: lane = latent dim within the tile, 16 heads per TMEM load
    for (int mt = 0; mt < n_mt; ++mt) {
      const int lat = mt * 128 + warp * 32 + lane;
      for (int c16 = 0; c16 < HGp / 16; ++c16) {
        uint32_t r[16];
        if (have_o) {
          tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + O0 + mt * HGp + c16 * 16, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) r[k] = 0u;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int hh = c16 * 16 + k;
          if (hh < hn) {
            const float v = __uint_as_float(r[k]);
            if (a.splits == 1) {
              const float l = l_sm[hh];
              a.o_lat[((int64_t)(h0 + hh) * a.T + t) * kvr + lat] = __float2bfloat16_rn(l > 0.f ? v / l : 0.f);
            } else {
              a.part_o[(((int64_t)sp * a.T + t) * a.H + h0 + hh) * kvr + lat] = v;
            }
          }
        }
      }
    }
    if (a.splits > 1 && head_lane && h < hn) {
      float* ml = a.part_ml + (((int64_t)sp * a.T + t) * a.H + h0 + h) * 2;
      ml[0] = have_o ? m_run : -INFINITY;
      ml[1] = have_o ? l_run : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, tcols);
}

// o[h, t] = sum_s 2^(m_s - m*) O_s / sum_s 2^(m_s - m*) l_s
__global__ void mla_tc_combine_kernel(const float* part_o, const float* part_ml, int splits, int T, int H, int kvr,
                                      __nv_bfloat16* o_lat) {
  const int t = blockIdx.x, h = blockIdx.y;
  __shared__ float w[16];
  __shared__ float inv_l;
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_ml[(((int64_t)s * T + t) * H + h) * 2]);
    float l = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float* ml = part_ml + (((int64_t)s * T + t) * H + h) * 2;
      w[s] = (ml[0] == -INFINITY) ? 0.f : exp2f(ml[0] - mx);
      l += w[s] * ml[1];
    }
    inv_l = l > 0.f ? 1.f / l : 0.f;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kvr; d += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < splits; ++s)
      if (w[s] != 0.f) acc += w[s] * part_o[(((int64_t)s * T + t) * H + h) * kvr + d];
    o_lat[((int64_t)h * T + t) * kvr + d] = __float2bfloat16_rn(acc * inv_l);
  }
}

int sm_count_cached() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

bool tc_supported(int64_t kvr, int64_t dr) {
  return kvr % 128 == 0 && kvr <= 1024 && (kvr + dr) % 64 == 0 && (kvr + dr) / 64 <= kMaxKB && dr % 8 == 0;
}

void d3_mla_attn_tc(torch::Tensor q_lat, torch::Tensor q_pe, torch::Tensor cache, torch::Tensor block_table,
                    torch::Tensor slots, torch::Tensor positions, int64_t n_tok, c10::optional<torch::Tensor> sel,
                    int64_t window, double scale, torch::Tensor o_lat, torch::Tensor err, int64_t timeout_ns,
                    int64_t force_splits, c10::optional<torch::Tensor> trace) {
  MlaTcArgs a{};
  a.H = q_lat.size(0);
  a.T = q_lat.size(1);
  a.kvr = q_lat.size(2);
  a.dr = q_pe.size(2);
  a.D = a.kvr + a.dr;
  TORCH_CHECK(tc_supported(a.kvr, a.dr), "tensor-core MLA needs kvr % 128 == 0 (<= 1024) and D % 64 == 0");
  TORCH_CHECK(q_lat.scalar_type() == torch::kBFloat16 && q_lat.is_contiguous() && o_lat.sizes() == q_lat.sizes() &&
              o_lat.scalar_type() == torch::kBFloat16 && o_lat.is_contiguous(), "q_lat / o_lat bf16 [H, T, kvr]");
  TORCH_CHECK(q_pe.scalar_type() == torch::kFloat && q_pe.is_contiguous() && q_pe.size(0) == a.T &&
              q_pe.size(1) == a.H, "q_pe fp32 [T, H, dr]");
  TORCH_CHECK(cache.scalar_type() == at::kFloat8_e4m3fn && cache.is_contiguous() && cache.size(2) == a.D,
              "cache fp8 [blocks, bs, kvr + dr]");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && slots.scalar_type() == torch::kInt32 &&
              positions.scalar_type() == torch::kInt32, "int32 tables");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.numel() >= 2, "err word");
  if (!a.T) return;
  const c10::cuda::CUDAGuard guard(q_lat.device());
  a.q_lat = reinterpret_cast<const __nv_bfloat16*>(q_lat.data_ptr());
  a.q_pe = q_pe.data_ptr<float>();
  a.cache = reinterpret_cast<const uint8_t*>(cache.data_ptr());
  a.block_table = block_table.data_ptr<int32_t>();
  a.max_blocks = block_table.size(1);
  a.bs = cache.size(1);
  a.slots = slots.data_ptr<int32_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.n_tok = n_tok;
  if (sel) {
    TORCH_CHECK(sel->scalar_type() == torch::kInt32 && sel->is_contiguous() && sel->size(0) == a.T, "sel int32 [T, k]");
    a.sel = sel->data_ptr<int32_t>();
    a.topk = sel->size(1);
  }
  a.window = window;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  // heads per CTA: O^T needs (kvr / 128) x HGp TMEM columns next to the double-buffered score accumulators,
  // and Q, the two key tiles and a loader stage must fit in shared memory
  int hgp = std::min(std::min(64, (512 - 2 * NACC * NK) / (a.kvr / 128) / 16 * 16), (int)((a.H + 15) / 16 * 16));
  while (hgp > 16 && smem_plan(a.D, hgp, 1).total > 227 * 1024) hgp -= 16;
  a.HGp = hgp;
  const int G = (a.H + a.HGp - 1) / a.HGp;
  int stages = kMaxStages;
  while (stages > 1 && smem_plan(a.D, a.HGp, stages).total > 227 * 1024) --stages;
  const Smem L = smem_plan(a.D, a.HGp, stages);
  TORCH_CHECK(L.total <= 227 * 1024, "MLA tile does not fit in shared memory");
  a.stages = stages;
  // key splits: fill the SMs (one CTA per SM); split lengths are whole chunks
  const int64_t n_max = a.sel ? a.topk : (window > 0 ? window : (int64_t)a.max_blocks * a.bs);
  const int64_t chunks = (n_max + NK - 1) / NK;
  int splits = (int)std::max<int64_t>(1, std::min<int64_t>({16, (sm_count_cached() + a.T * G - 1) / (a.T * G),
                                                            std::max<int64_t>(1, chunks / 4)}));
  if (force_splits > 0) splits = (int)std::min<int64_t>(16, force_splits);
  a.splits = splits;
  a.o_lat = reinterpret_cast<__nv_bfloat16*>(o_lat.data_ptr());
  torch::Tensor po, pml;
  if (splits > 1) {
    po = torch::empty({splits, a.T, a.H, a.kvr}, q_pe.options());
    pml = torch::empty({splits, a.T, a.H, 2}, q_pe.options());
    a.part_o = po.data_ptr<float>();
    a.part_ml = pml.data_ptr<float>();
  }
  a.err = err.data_ptr<int32_t>();
  a.timeout_ns = (uint64_t)timeout_ns;
  if (trace) {
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->numel() >= 64 * 8, "trace int64 [64 * 8]");
    a.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(mla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr = true;
  }
  mla_tc_kernel<<<dim3(a.T, G, splits), kThreads, L.total, STREAM>>>(a);
  if (splits > 1)
    mla_tc_combine_kernel<<<dim3(a.T, a.H), 128, 0, STREAM>>>(a.part_o, a.part_ml, splits, a.T, a.H, a.kvr,
                                                               a.o_lat);
}

}  // namespace

void register_mla(pybind11::module& m) {
  m.def("d3_mla_attn_tc", &d3_mla_attn_tc);
  m.def("d3_mla_tc_supported", &tc_supported);
}
