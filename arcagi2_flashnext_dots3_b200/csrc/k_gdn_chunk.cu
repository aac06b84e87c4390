// Gated DeltaNet prefill in chunks of 64 tokens on tcgen05 (bf16 operands, fp32 accumulation in TMEM), sm_100a.
//
// Recurrence (per value head, state S [dk x dv]): S_t = e^{g_t} S_{t-1} + k_t u_t^T with
// u_t = beta_t (v_t - S_{t-1}'^T k_t) (S' = the decayed state), o_t = S_t^T q_t; q, k l2-normalized (q also scaled
// by dk^-1/2). Within a chunk of C tokens with inclusive log-decay sums gc and Gamma[i][j] = e^{gc_i - gc_j}
// (j <= i), the sequential updates become matrix products (the WY form the reference trains with through fla's
// chunked kernel, flashnext/training/student/student_fn.py:251; statement in training/gdn_chunk.py):
//
//   L      = strictly_lower(diag(beta) K K^T o Gamma)        T = (I + L)^-1 (unit lower triangular)
//   U      = T (beta o V)                                   W = T (beta o e^{gc} o K)
//   V_new  = U - W S                                        (the u_t of every token of the chunk)
//   O      = diag(e^{gc}) Q S + (Q K^T o Gamma_incl) V_new
//   S     <- e^{gc_last} S + (e^{gc_last - gc} o K)^T V_new
//
// One CTA of 128 threads per (sequence, value head) walks its chunks in order. The eight products per chunk run
// on the tensor cores (M 64 token rows or 128 key rows, K-major bf16 operands in the 128-byte swizzle, one
// issuing thread, tcgen05.commit to an mbarrier); the triangular solve runs on 64 threads (one column each,
// forward substitution in fp32), the masks, decays, transposes and the gated RMSNorm output in the other phases.
// TMEM (512 columns): K K^T 64 | Q K^T 64 | U -> V_new 128 | W -> O 128 | S 128 (fp32 master state). Every wait is
// bounded (%globaltimer); a timeout records an error code (77xx) and the CTA finishes its chunks without
// results (every thread takes the same barriers) and frees its TMEM.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "ptx.cuh"

namespace fw {
namespace gdnc {

constexpr int C = 64;              // tokens per chunk
constexpr int D = 128;             // dk = dv
constexpr int kThreads = 128;
// shared-memory tiles (bytes), K-major bf16 in the 128-byte swizzle: [rows][K] stored as K/64 blocks of rows x 128 B
constexpr int kTileQ = C * D * 2;        // Q, K, W: [64 tokens][128]
constexpr int kTileT = C * C * 2;        // T, P: [64][64]
constexpr int kTileX = D * C * 2;        // (beta V)^T, (beta e^gc K)^T, V_new^T, (e^{gl-gc} K)^T: [128][64 tokens]
constexpr int kTileS = D * D * 2;        // S^T: [128 dv][128 dk]
constexpr int oQ = 0, oK = oQ + kTileQ, oW = oK + kTileQ, oT = oW + kTileQ, oP = oT + kTileT, oVb = oP + kTileT,
              oKb = oVb + kTileX, oVn = oKb + kTileX, oKd = oVn + kTileX, oS = oKd + kTileX,
              oL = oS + kTileS,                      // fp32 L [64][64]
              oTf = oL + C * C * 4,                  // fp32 T [64 rows][64 cols]
              oX = oTf + C * C * 4,                  // fp32 [3][16][16] partial products of the blocked solve
              oVec = oX + 3 * 256 * 4,               // gc [64], beta [64]
              oBar = oVec + 2 * C * 4, kSmemUsed = oBar + 64;
constexpr size_t kSmem = 1024 + (size_t)kSmemUsed;
// fp32 staging of 64 rows x 128 (V rows in the load phase, output rows at the end) over the L / T / X area
constexpr int kStage = 132;              // row stride in floats (16-byte rows, conflict-free column reads)
static_assert(C * kStage * 4 <= oVec - oL, "staging area");
// TMEM columns
constexpr uint32_t tA = 0, tQK = 64, tU = 128, tW = 256, tS = 384;

__device__ __forceinline__ float sigm_f(float x) { return 1.f / (1.f + __expf(-x)); }

// byte offset of element (r, k) in a K-major swizzled bf16 tile of `rows` rows
__device__ __forceinline__ uint32_t sw_off(int r, int k, int rows) {
  const int blk = k >> 6, kk = k & 63;
  return (uint32_t)(blk * rows * 128 + r * 128 + ((((kk >> 3) ^ (r & 7)) << 4) | ((kk & 7) << 1)));
}

__device__ __forceinline__ void st_bf16(uint32_t addr, float v) {
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<const unsigned short*>(&b)) : "memory");
}

// 8 consecutive k (a 16-byte chunk, k % 8 == 0) of row r
__device__ __forceinline__ void st_chunk8(uint32_t tile, int r, int k, int rows, const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tile + sw_off(r, k, rows)), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3])
               : "memory");
}

__device__ __forceinline__ void ld_chunk8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// D[tmem] (+)= A * B^T over K = 16 * nk16, A [M rows][K] and B [N rows][K] K-major swizzled tiles
__device__ __forceinline__ void mma_tiles(uint32_t d, uint32_t a, int a_rows, uint32_t b, int b_rows, int nk16,
                                          uint32_t idesc, bool accumulate) {
  for (int s = 0; s < nk16; ++s) {
    const int blk = s >> 2, in = (s & 3) * 32;
    umma_f16(d, umma_desc_sw128(a + blk * a_rows * 128 + in), umma_desc_sw128(b + blk * b_rows * 128 + in), idesc,
             (accumulate || s > 0) ? 1u : 0u);
  }
}

struct Args {
  const __nv_bfloat16* q;       // [rows, nk, 128] l2-normalized, scaled
  const __nv_bfloat16* k;       // [rows, nk, 128] l2-normalized
  const float* qkv;             // [rows, Cq] conv outputs (v at 2*nk*128 + hv*128)
  const float* gb;              // [rows, nv, 2]: log decay g, beta
  const float* proj;            // [rows, ldp] (z gate at Cq + hv*128)
  int ldp, Cq;
  const float* norm_w;          // [128]
  __nv_bfloat16* ssm;           // [S, nv, 128, 128] state (bf16)
  const int* slots;
  __half* out;                  // [rows, nv*128]
  int nk, nv, n_tok;
  float eps;
  int gate_sigmoid;
  int* err;
  unsigned long long timeout_ns;
  long long* trace;             // optional: %globaltimer at phase starts of CTA (0, 0), [chunks][16]
};

// Wait for an MMA commit; every thread polls (bounded). False (and the shared abort flag set) on timeout.
__device__ __forceinline__ bool wait_commit(uint32_t bar, uint32_t parity, const Args& a, int code,
                                            volatile int* abort_flag) {
  return mbar_wait(bar, parity, a.err, code, abort_flag, a.timeout_ns);
}

__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_kernel(const Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  float* sL = reinterpret_cast<float*>(g + oL);
  float* sTf = reinterpret_cast<float*>(g + oTf);
  float* sgc = reinterpret_cast<float*>(g + oVec);
  float* sbeta = sgc + C;
  const uint32_t bar = base + oBar;      // one mbarrier, phases counted below
  volatile int* abort_flag = reinterpret_cast<volatile int*>(g + oBar + 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(g + oBar + 16);

  const int b = blockIdx.x, hv = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = hv / (a.nv / a.nk);
  const int slot = a.slots[b];
  __nv_bfloat16* Sg = a.ssm + ((int64_t)slot * a.nv + hv) * D * D;
  // M = 64 results: token row 16w + l sits in TMEM lane 32w + l (l < 16)
  const bool row_lane = lane < 16;
  const int ti = 16 * warp + lane;       // token row of this thread in M = 64 results (when row_lane)
  const uint32_t lane_base = (uint32_t)(32 * warp) << 16;

  if (tid == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc_dyn(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  constexpr uint32_t id64x64 = umma_idesc_f16(64, 64, 1);
  constexpr uint32_t id64x128 = umma_idesc_f16(64, 128, 1);
  constexpr uint32_t id64x128_neg = umma_idesc_f16(64, 128, 1) | (1u << 13);   // negate A
  constexpr uint32_t id128x128 = umma_idesc_f16(128, 128, 1);
  uint32_t phase = 0;
  bool pending = false;                  // thread 0: MMAs committed and not yet seen complete
  uint32_t pending_phase = 0;

  // initial state: fp32 into TMEM (thread = key row d), bf16 transpose into S^T
  {
    const int d = tid;
    float row[D];
#pragma unroll
    for (int n = 0; n < D; n += 8) ld_chunk8(Sg + (int64_t)d * D + n, row + n);
#pragma unroll
    for (int n = 0; n < D; ++n) st_bf16(base + oS + sw_off(n, d, D), row[n]);
    uint32_t v[32];
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(row[32 * c4 + i]);
      tmem_st32(tmem + lane_base + tS + 32 * c4, v);
    }
    tmem_st_wait();
  }
  const int n_chunks = (a.n_tok + C - 1) / C;
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int t0 = ch * C;
    const int nreal = min(C, a.n_tok - t0);
    const int64_t row0 = (int64_t)b * a.n_tok + t0;
    // ---------------------------------------------------------------- P0: load the chunk
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 0] = (long long)globaltimer_ns();
    if (warp == 0) {                     // inclusive cumulative log decay and beta (padded tokens: g 0, beta 0)
      float gg[2], bb[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = lane + 32 * h;
        const bool real = i < nreal;
        gg[h] = real ? a.gb[((row0 + i) * a.nv + hv) * 2] : 0.f;
        bb[h] = real ? a.gb[((row0 + i) * a.nv + hv) * 2 + 1] : 0.f;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, gg[h], o);
          if (lane >= o) gg[h] += y;
        }
      }
      const float carry = __shfl_sync(0xffffffffu, gg[0], 31);
      gg[1] += carry;
      sgc[lane] = gg[0];
      sgc[lane + 32] = gg[1];
      sbeta[lane] = bb[0];
      sbeta[lane + 32] = bb[1];
    }
    __syncthreads();
    {
      // Q and K rows (two threads per token row, 64 columns each) into their tiles, V rows (fp32) into the
      // staging area for the transposed operands
      const int i = tid >> 1, half = tid & 1;
      const bool real = i < nreal;
      const __nv_bfloat16* qp = a.q + ((row0 + i) * a.nk + hk) * D + 64 * half;
      const __nv_bfloat16* kp = a.k + ((row0 + i) * a.nk + hk) * D + 64 * half;
      const float* vp = a.qkv + (row0 + i) * a.Cq + 2 * a.nk * D + hv * D + 64 * half;
      float* stg = reinterpret_cast<float*>(g + oL) + i * kStage + 64 * half;
#pragma unroll
      for (int c8 = 0; c8 < 64; c8 += 8) {
        float vq[8], vk[8];
        float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
        if (real) {
          ld_chunk8(qp + c8, vq);
          ld_chunk8(kp + c8, vk);
          v0 = *reinterpret_cast<const float4*>(vp + c8);
          v1 = *reinterpret_cast<const float4*>(vp + c8 + 4);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) vq[e] = vk[e] = 0.f;
        }
        st_chunk8(base + oQ, i, 64 * half + c8, C, vq);
        st_chunk8(base + oK, i, 64 * half + c8, C, vk);
        *reinterpret_cast<float4*>(stg + c8) = v0;
        *reinterpret_cast<float4*>(stg + c8 + 4) = v1;
      }
    }
    __syncthreads();
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 10] = (long long)globaltimer_ns();
    {
      // transposed operands: thread = feature n, reading column n of the staged V rows and of the K tile
      const int n = tid;
      const float gl = sgc[C - 1];
      const float* stg = reinterpret_cast<const float*>(g + oL);
      const uint8_t* ktile = g + oK;
#pragma unroll 2
      for (int j8 = 0; j8 < C; j8 += 8) {
        float vb[8], kb[8], kd[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = j8 + e;
          const float vv = stg[j * kStage + n];
          const float kk = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(ktile + sw_off(j, n, C)));
          const float gj = sgc[j];
          vb[e] = sbeta[j] * vv;
          kb[e] = sbeta[j] * __expf(gj) * kk;
          kd[e] = __expf(gl - gj) * kk;
        }
        st_chunk8(base + oVb, n, j8, D, vb);
        st_chunk8(base + oKb, n, j8, D, kb);
        st_chunk8(base + oKd, n, j8, D, kd);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    // ---------------------------------------------------------------- P1: K K^T and Q K^T
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 1] = (long long)globaltimer_ns();
    if (tid == 0 && !*abort_flag) {
      tc_fence_after();
      mma_tiles(tmem + tA, base + oK, C, base + oK, C, D / 16, id64x64, false);
      mma_tiles(tmem + tQK, base + oQ, C, base + oK, C, D / 16, id64x64, false);
      umma_commit(bar);
      pending = true;
      pending_phase = phase;
    }
    if (!*abort_flag && wait_commit(bar, phase, a, 7701, abort_flag) && tid == 0) pending = false;
    phase ^= 1u;
    tc_fence_after();
    // ---------------------------------------------------------------- P2: L (fp32) and P (bf16) rows
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 2] = (long long)globaltimer_ns();
    {
      uint32_t ra[32], rq[32];
      float l[C], p[C];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld16(tmem + lane_base + tA + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(ra));
        tmem_ld16(tmem + lane_base + tA + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(ra + 16));
        tmem_ld16(tmem + lane_base + tQK + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(rq));
        tmem_ld16(tmem + lane_base + tQK + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(rq + 16));
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          l[32 * c + e] = __uint_as_float(ra[e]);
          p[32 * c + e] = __uint_as_float(rq[e]);
        }
      }
      if (row_lane) {
        const float gi = sgc[ti], bi = sbeta[ti];
#pragma unroll
        for (int j = 0; j < C; ++j) {
          const float dec = j <= ti ? __expf(gi - sgc[j]) : 0.f;
          sL[ti * C + j] = j < ti ? bi * l[j] * dec : 0.f;
          p[j] *= dec;
        }
#pragma unroll
        for (int j8 = 0; j8 < C; j8 += 8) st_chunk8(base + oP, ti, j8, C, p + j8);
      }
    }
    __syncthreads();
    // ---------------------------------------------------------------- P3: T = (I + L)^-1, one column per thread
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 3] = (long long)globaltimer_ns();
    {
      // blocked: the four 16 x 16 diagonal blocks by forward substitution (one column per thread), then the
      // off-diagonal blocks by block diagonals, T_ij = -T_ii sum_{k=j}^{i-1} L_ik T_kj (16 x 16 products)
      float* sX = reinterpret_cast<float*>(g + oX);
      if (tid < C) {
        const int kb = tid >> 4, c = tid & 15, col = 16 * kb + c;
        for (int r = 0; r < 16 * kb; ++r) sTf[r * C + col] = 0.f;
        for (int ri = 0; ri < 16; ++ri) {
          const int r = 16 * kb + ri;
          float v;
          if (ri < c) {
            v = 0.f;
          } else if (ri == c) {
            v = 1.f;
          } else {
            float acc = 0.f;
            for (int jj = c; jj < ri; ++jj) acc += sL[r * C + 16 * kb + jj] * sTf[(16 * kb + jj) * C + col];
            v = -acc;
          }
          sTf[r * C + col] = v;
        }
        for (int r = 16 * kb + 16; r < C; ++r) sTf[r * C + col] = 0.f;   // below: filled by the block levels
      }
      __syncthreads();
      for (int d = 1; d < 4; ++d) {
        const int nb = 4 - d;
        for (int e = tid; e < nb * 256; e += kThreads) {
          const int bj = e >> 8, bi = bj + d, r = (e >> 4) & 15, c = e & 15;
          float acc = 0.f;
          for (int kk = bj; kk < bi; ++kk) {
#pragma unroll
            for (int m = 0; m < 16; ++m) acc += sL[(16 * bi + r) * C + 16 * kk + m] * sTf[(16 * kk + m) * C + 16 * bj + c];
          }
          sX[e] = acc;
        }
        __syncthreads();
        for (int e = tid; e < nb * 256; e += kThreads) {
          const int bj = e >> 8, bi = bj + d, r = (e >> 4) & 15, c = e & 15;
          float acc = 0.f;
          for (int m = 0; m <= r; ++m) acc += sTf[(16 * bi + r) * C + 16 * bi + m] * sX[(bj << 8) + (m << 4) + c];
          sTf[(16 * bi + r) * C + 16 * bj + c] = -acc;
        }
        __syncthreads();
      }
      for (int e = tid; e < C * 8; e += kThreads) {     // bf16 operand rows
        const int r = e >> 3, c8 = (e & 7) * 8;
        st_chunk8(base + oT, r, c8, C, sTf + r * C + c8);
      }
    }
    fence_proxy_async_smem();
    __syncthreads();
    // ---------------------------------------------------------------- P4: U = T (beta V), W = T (beta e^gc K)
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 4] = (long long)globaltimer_ns();
    if (tid == 0 && !*abort_flag) {
      tc_fence_after();
      mma_tiles(tmem + tU, base + oT, C, base + oVb, D, C / 16, id64x128, false);
      mma_tiles(tmem + tW, base + oT, C, base + oKb, D, C / 16, id64x128, false);
      umma_commit(bar);
      pending = true;
      pending_phase = phase;
    }
    if (!*abort_flag && wait_commit(bar, phase, a, 7702, abort_flag) && tid == 0) pending = false;
    phase ^= 1u;
    tc_fence_after();
    // ---------------------------------------------------------------- P5: W rows -> bf16 operand
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 5] = (long long)globaltimer_ns();
    {
      uint32_t r[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld16(tmem + lane_base + tW + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tW + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
        if (row_lane) {
          float w[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __uint_as_float(r[e]);
#pragma unroll
          for (int e8 = 0; e8 < 32; e8 += 8) st_chunk8(base + oW, ti, 32 * c + e8, C, w + e8);
        }
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- P6: V_new = U - W S, O1 = Q S
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 6] = (long long)globaltimer_ns();
    if (tid == 0 && !*abort_flag) {
      tc_fence_after();
      mma_tiles(tmem + tU, base + oW, C, base + oS, D, D / 16, id64x128_neg, true);
      mma_tiles(tmem + tW, base + oQ, C, base + oS, D, D / 16, id64x128, false);
      umma_commit(bar);
      pending = true;
      pending_phase = phase;
    }
    if (!*abort_flag && wait_commit(bar, phase, a, 7703, abort_flag) && tid == 0) pending = false;
    phase ^= 1u;
    tc_fence_after();
    // ---------------------------------------------------------------- P7: V_new^T, e^gc O1, e^gl S
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 7] = (long long)globaltimer_ns();
    {
      const float gl = sgc[C - 1];
      uint32_t r[32];
      const float egi = row_lane ? __expf(sgc[ti]) : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld16(tmem + lane_base + tU + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tU + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
        if (row_lane) {
#pragma unroll
          for (int e = 0; e < 32; ++e) st_bf16(base + oVn + sw_off(32 * c + e, ti, D), __uint_as_float(r[e]));
        }
        tmem_ld16(tmem + lane_base + tW + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tW + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * egi);
        tmem_st32(tmem + lane_base + tW + 32 * c, r);
        // the state: all 128 lanes are key rows (M = 128)
        tmem_ld16(tmem + lane_base + tS + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tS + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
        const float egl = __expf(gl);
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * egl);
        tmem_st32(tmem + lane_base + tS + 32 * c, r);
      }
      tmem_st_wait();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---------------------------------------------------------------- P8: O += P V_new, S += Kd^T V_new
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 8] = (long long)globaltimer_ns();
    if (tid == 0 && !*abort_flag) {
      tc_fence_after();
      mma_tiles(tmem + tW, base + oP, C, base + oVn, D, C / 16, id64x128, true);
      mma_tiles(tmem + tS, base + oKd, D, base + oVn, D, C / 16, id128x128, true);
      umma_commit(bar);
      pending = true;
      pending_phase = phase;
    }
    if (!*abort_flag && wait_commit(bar, phase, a, 7704, abort_flag) && tid == 0) pending = false;
    phase ^= 1u;
    tc_fence_after();
    // ---------------------------------------------------------------- P9: output rows, S^T for the next chunk
    if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 9] = (long long)globaltimer_ns();
    {
      float o[D];
      uint32_t r[32];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld16(tmem + lane_base + tW + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tW + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[32 * c + e] = __uint_as_float(r[e]);
      }
      // rows normalized by their own threads into the staging area, then written out column-parallel (the z
      // gates read and the outputs written in full rows of 128 per warp instruction)
      float* stg = reinterpret_cast<float*>(g + oL);
      if (row_lane) {
        float ss = 0.f;
#pragma unroll
        for (int n = 0; n < D; ++n) ss += o[n] * o[n];
        const float rn = rsqrtf(ss / D + a.eps);
#pragma unroll
        for (int n = 0; n < D; n += 4)
          *reinterpret_cast<float4*>(stg + ti * kStage + n) =
              make_float4(o[n] * rn, o[n + 1] * rn, o[n + 2] * rn, o[n + 3] * rn);
      }
      __syncthreads();
      if (!*abort_flag) {
        const int n = tid;
        const float nw = a.norm_w[n];
        const float* zp = a.proj + row0 * a.ldp + a.Cq + hv * D + n;
        __half* op = a.out + row0 * (a.nv * D) + hv * D + n;
        for (int i0 = 0; i0 < nreal; i0 += 16) {
          float zz[16];                  // a batch of gate loads in flight before the stores
#pragma unroll
          for (int e = 0; e < 16; ++e) zz[e] = i0 + e < nreal ? __ldg(zp + (int64_t)(i0 + e) * a.ldp) : 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int i = i0 + e;
            if (i < nreal) {
              const float gz = a.gate_sigmoid ? sigm_f(zz[e]) : zz[e] * sigm_f(zz[e]);
              op[(int64_t)i * (a.nv * D)] = __float2half_rn(stg[i * kStage + n] * nw * gz);
            }
          }
        }
      }
      if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 11] = (long long)globaltimer_ns();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld16(tmem + lane_base + tS + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
        tmem_ld16(tmem + lane_base + tS + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) st_bf16(base + oS + sw_off(32 * c + e, tid, D), __uint_as_float(r[e]));
      }
      if (a.trace && tid == 0 && blockIdx.x == 0 && blockIdx.y == 0) a.trace[ch * 16 + 12] = (long long)globaltimer_ns();
    }
    fence_proxy_async_smem();
    __syncthreads();
  }
  // final state back to the cache (bf16), thread = key row
  if (!*abort_flag) {
    uint32_t r[32];
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      tmem_ld16(tmem + lane_base + tS + 32 * c, *reinterpret_cast<uint32_t(*)[16]>(r));
      tmem_ld16(tmem + lane_base + tS + 32 * c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const __nv_bfloat162 p2 = __floats2bfloat162_rn(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        *reinterpret_cast<__nv_bfloat162*>(Sg + (int64_t)tid * D + 32 * c + e) = p2;
      }
    }
  }
  if (tid == 0 && pending) {             // after an abort: MMAs still in flight must land before TMEM is freed
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, pending_phase) && globaltimer_ns() - t0 < a.timeout_ns) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Per (token, key head): q, k l2-normalized (eps 1e-6 inside the root, q scaled by dk^-1/2) to bf16; per (token,
// value head): g = -e^{A_log} softplus(a + dt_bias) and beta = sigmoid(b). One warp per (token, key head).
__global__ void gdn_chunk_prep_kernel(const float* qkv, int Cq, const float* proj, int ldp, const float* A_log,
                                      const float* dt_bias, int rows, int nk, int nv, __nv_bfloat16* q,
                                      __nv_bfloat16* k, float* gb) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= rows * nk) return;
  const int row = w / nk, hk = w % nk;
  const float* x = qkv + (int64_t)row * Cq;
  const float4 qv = *reinterpret_cast<const float4*>(x + hk * D + 4 * lane);
  const float4 kv = *reinterpret_cast<const float4*>(x + nk * D + hk * D + 4 * lane);
  float qs = qv.x * qv.x + qv.y * qv.y + qv.z * qv.z + qv.w * qv.w;
  float ks = kv.x * kv.x + kv.y * kv.y + kv.z * kv.z + kv.w * kv.w;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    qs += __shfl_xor_sync(0xffffffffu, qs, o);
    ks += __shfl_xor_sync(0xffffffffu, ks, o);
  }
  const float qf = rsqrtf(qs + 1e-6f) * rsqrtf((float)D), kf = rsqrtf(ks + 1e-6f);
  __nv_bfloat162* qo = reinterpret_cast<__nv_bfloat162*>(q + ((int64_t)row * nk + hk) * D + 4 * lane);
  __nv_bfloat162* ko = reinterpret_cast<__nv_bfloat162*>(k + ((int64_t)row * nk + hk) * D + 4 * lane);
  qo[0] = __floats2bfloat162_rn(qv.x * qf, qv.y * qf);
  qo[1] = __floats2bfloat162_rn(qv.z * qf, qv.w * qf);
  ko[0] = __floats2bfloat162_rn(kv.x * kf, kv.y * kf);
  ko[1] = __floats2bfloat162_rn(kv.z * kf, kv.w * kf);
  const int r = nv / nk;
  if (lane < r) {
    const int hv = hk * r + lane;
    const float* pr = proj + (int64_t)row * ldp;
    const float bb = pr[Cq + nv * D + hv], aa = pr[Cq + nv * D + nv + hv];
    const float sp = aa + dt_bias[hv] > 20.f ? aa + dt_bias[hv] : log1pf(__expf(aa + dt_bias[hv]));
    gb[((int64_t)row * nv + hv) * 2] = -__expf(A_log[hv]) * sp;
    gb[((int64_t)row * nv + hv) * 2 + 1] = 1.f / (1.f + __expf(-bb));
  }
}

}  // namespace gdnc
}  // namespace fw

namespace {

// Prefill of n_tok tokens per sequence through the chunked gated delta rule. qkv: conv outputs [rows, Cq] (fp32,
// from gdn_conv), proj: [rows, ldp] (z | b | a after Cq), ssm: bf16 state [S, nv, 128, 128] (updated), out: fp16
// [rows, nv*128] gated-RMSNorm outputs.
void gdn_chunk(torch::Tensor qkv, torch::Tensor proj, torch::Tensor ssm, torch::Tensor A_log, torch::Tensor dt_bias,
               torch::Tensor norm_w, torch::Tensor slots, torch::Tensor out, int64_t nk, int64_t nv, int64_t n_tok,
               double eps, int64_t gate_sigmoid, torch::Tensor err, int64_t timeout_ns,
               c10::optional<torch::Tensor> trace) {
  using namespace fw::gdnc;
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == torch::kFloat && qkv.is_contiguous(), "qkv fp32");
  TORCH_CHECK(proj.scalar_type() == torch::kFloat && proj.is_contiguous(), "proj fp32");
  TORCH_CHECK(ssm.scalar_type() == torch::kBFloat16 && ssm.is_contiguous(), "bf16 state");
  TORCH_CHECK(ssm.size(-1) == D && ssm.size(-2) == D && nv % nk == 0 && nv / nk <= 32, "128 x 128 heads");
  TORCH_CHECK(out.scalar_type() == torch::kHalf && out.is_contiguous(), "fp16 out");
  const int rows = qkv.size(0);
  if (!rows) return;
  TORCH_CHECK(rows % n_tok == 0, "rows = sequences x n_tok");
  const int B = rows / n_tok;
  const int Cq = qkv.size(1);
  TORCH_CHECK(Cq == 2 * nk * D + nv * D, "qkv width");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto q = torch::empty({rows, nk, D}, qkv.options().dtype(torch::kBFloat16));
  auto k = torch::empty({rows, nk, D}, qkv.options().dtype(torch::kBFloat16));
  auto gb = torch::empty({rows, nv, 2}, qkv.options());
  const int64_t warps = (int64_t)rows * nk;
  gdn_chunk_prep_kernel<<<(warps * 32 + 255) / 256, 256, 0, st>>>(
      qkv.data_ptr<float>(), Cq, proj.data_ptr<float>(), proj.size(1), A_log.data_ptr<float>(),
      dt_bias.data_ptr<float>(), rows, nk, nv, (__nv_bfloat16*)q.data_ptr(), (__nv_bfloat16*)k.data_ptr(),
      gb.data_ptr<float>());
  Args a{};
  a.q = (const __nv_bfloat16*)q.data_ptr();
  a.k = (const __nv_bfloat16*)k.data_ptr();
  a.qkv = qkv.data_ptr<float>();
  a.gb = gb.data_ptr<float>();
  a.proj = proj.data_ptr<float>();
  a.ldp = proj.size(1);
  a.Cq = Cq;
  a.norm_w = norm_w.data_ptr<float>();
  a.ssm = (__nv_bfloat16*)ssm.data_ptr();
  a.slots = slots.data_ptr<int32_t>();
  a.out = (__half*)out.data_ptr();
  a.nk = nk;
  a.nv = nv;
  a.n_tok = n_tok;
  a.eps = (float)eps;
  a.gate_sigmoid = (int)gate_sigmoid;
  a.err = err.data_ptr<int32_t>();
  a.timeout_ns = (unsigned long long)timeout_ns;
  if (trace) {
    TORCH_CHECK(trace->scalar_type() == torch::kInt64 && trace->numel() >= (n_tok + C - 1) / C * 16, "trace int64");
    a.trace = reinterpret_cast<long long*>(trace->data_ptr<int64_t>());
  }
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) ==
                    cudaSuccess, "gdn_chunk shared memory attribute");
    attr = true;
  }
  gdn_chunk_kernel<<<dim3(B, nv), kThreads, kSmem, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  TORCH_CHECK(e == cudaSuccess, "gdn_chunk launch failed: ", cudaGetErrorString(e));
}

}  // namespace

void gdn_conv_prefill(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor slots,
                      torch::Tensor qkv, int64_t n_tok);   // k_fn.cu

namespace {

// Prefill step of a GDN layer (no commit count): the convolution over every token, then the chunked delta rule.
// Same contract as gdn_step for bf16 states.
void gdn_prefill(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor ssm,
                 torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor slots,
                 torch::Tensor out, int64_t nk, int64_t nv, int64_t n_tok, double eps, int64_t gate_sigmoid,
                 torch::Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(proj.is_cuda() && proj.scalar_type() == torch::kFloat && proj.is_contiguous(), "proj fp32");
  const int rows = proj.size(0);
  if (!rows) return;
  const int64_t Cq = 2 * nk * fw::gdnc::D + nv * fw::gdnc::D;
  auto qkv = torch::empty({rows, Cq}, proj.options());
  gdn_conv_prefill(proj, conv_w, conv_state, slots, qkv, n_tok);
  gdn_chunk(qkv, proj, ssm, A_log, dt_bias, norm_w, slots, out, nk, nv, n_tok, eps, gate_sigmoid, err, timeout_ns,
            c10::nullopt);
}

}  // namespace

void register_gdn_chunk(pybind11::module& m) {
  m.def("gdn_chunk", &gdn_chunk, "Gated DeltaNet delta rule in chunks of 64 tokens on tcgen05 (conv outputs in)");
  m.def("gdn_prefill", &gdn_prefill, "GDN prefill: parallel convolution + chunked delta rule on tcgen05");
}
