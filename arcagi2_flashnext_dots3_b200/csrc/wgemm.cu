// Weight-dequant grouped GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// One kernel serves every weight-streaming GEMM of the engine:
//   * the low-bit MoE expert projections (2/3/4-bit GPTQ codes, group-128 fp16 scales, uint8 zeros), with
//     experts of different bit widths mixed in one launch (the reference's K17/K18/K21 Triton and Marlin GEMMs,
//     dotsnote/engine/arcstats_pkg/arcstats/lowbit_moe.py:31, flashnext/kaggle/code_dataset/fnext/moe/lowbit2.py:97);
//   * FP8 block-scaled (128x128) dense weights (the reference's K22/K37/K39 W8A8 and online-FP8 GEMMs,
//     dotsnote/engine/arcstats_pkg/arcstats/w8a8_v2.py:32, flashnext/kaggle/code_dataset/fnext/moe/dense.py:29);
//   * plain fp16 weights.
//
// Formulation ("weights as M"): y[tok, row] = sum_k W[row, k] * x[tok, k]. A 128-row tile of W is the MMA's
// M operand, up to N tokens are the N operand, so decode batches of a few tokens per expert still run on the
// tensor core (M=128, N>=16). Per CTA (persistent, one per SM):
//   warp 0      TMA: 1-D bulk copies of the packed weight block of each 128-column group into a smem ring
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (8 x K16 per group) into TMEM
//   warp 2      TMA: 2-D tiled loads of the token tile (fp16, SWIZZLE_128B) + TMEM allocation
//   warps 4-15  dequant: packed codes -> fp16 s*(q-z) in registers -> SWIZZLE_128B smem A tile (3 teams of
//               4 warps on alternating stages; a thread converts one row of its team's 128-column group)
//   warps 16-19 epilogue: tcgen05.ld of the double-buffered accumulator, store or silu(gate)*up
// Every mbarrier wait is bounded (%globaltimer); a timeout records an error code and all roles drain out.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include "ptx.cuh"
#include "wgemm.h"
#include <cudaTypedefs.h>

namespace fw {

constexpr int kTeams = 3;                         // dequant teams of 4 warps (maximum), alternating stages
constexpr int kDqThreads = 128 * kTeams;          // warps 4 .. 4 + 4 * kTeams - 1
constexpr int kEpiThreads = 128;                  // the last 4 warps
constexpr int kEpiWarp0 = 4 + 4 * kTeams;
constexpr int kEpiFirst = 32 * kEpiWarp0;
constexpr int kThreads = kEpiFirst + kEpiThreads;

struct WGemmSmem {
  // offsets relative to the 1024-aligned dynamic smem base
  uint32_t ab, w, bars, epi;
  uint32_t ab_stage_bytes;
};

__device__ __forceinline__ uint32_t hadd2_u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hadd2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  return h2_as_u32(__hfma2(u32_as_h2(a), u32_as_h2(b), u32_as_h2(c)));
}
__device__ __forceinline__ uint32_t h2c(float v) { return h2_as_u32(__float2half2_rn(v)); }
// fp16x2 bit patterns of the exact power-of-two field multipliers (no runtime conversion in the dequant loop)
constexpr uint32_t kH2_1_4 = 0x34003400u, kH2_1_8 = 0x30003000u, kH2_1_16 = 0x2C002C00u, kH2_1_64 = 0x24002400u,
                   kH2_1_256 = 0x1C001C00u;

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Dequant of one code pair (two adjacent columns) at "magic" field position. v = (w & mask) | 0x6400.. is the
// fp16 pair 1024 + q * 2^sh; v * 2^-sh + c with c = -(1024 * 2^-sh + z) is q - z exactly; times s rounds once.
struct DqConst {
  uint32_t s2;       // (s, s)
  uint32_t c[8];     // per field shift class: -(1024 * 2^-sh + z)
};

#define FW_MAGIC 0x64006400u

// 4-bit: word = 4 pairs, pair k at bits 4k / 16+4k.
__device__ __forceinline__ void dq4_word(uint32_t w, const DqConst& K, uint32_t (&o)[4]) {
  const uint32_t m16 = kH2_1_16;
  uint32_t v0 = (w & 0x000F000Fu) | FW_MAGIC;
  uint32_t v1 = (w & 0x00F000F0u) | FW_MAGIC;
  uint32_t w8 = w >> 8;
  uint32_t v2 = (w8 & 0x000F000Fu) | FW_MAGIC;
  uint32_t v3 = (w8 & 0x00F000F0u) | FW_MAGIC;
  o[0] = hmul2_u(hadd2_u(v0, K.c[0]), K.s2);
  o[1] = hmul2_u(hfma2_u(v1, m16, K.c[1]), K.s2);
  o[2] = hmul2_u(hadd2_u(v2, K.c[0]), K.s2);
  o[3] = hmul2_u(hfma2_u(v3, m16, K.c[1]), K.s2);
}

// 3-bit: word = 5 pairs, pair k at bits 3k / 16+3k.
__device__ __forceinline__ uint32_t dq3_pair(uint32_t w, int k, const DqConst& K) {
  uint32_t ww = k >= 3 ? (w >> 9) : w;
  int kk = k >= 3 ? k - 3 : k;
  uint32_t v;
  if (kk == 0) {
    v = (ww & 0x00070007u) | FW_MAGIC;
    return hmul2_u(hadd2_u(v, K.c[0]), K.s2);
  } else if (kk == 1) {
    v = (ww & 0x00380038u) | FW_MAGIC;
    return hmul2_u(hfma2_u(v, kH2_1_8, K.c[1]), K.s2);
  } else {
    v = (ww & 0x01C001C0u) | FW_MAGIC;
    return hmul2_u(hfma2_u(v, kH2_1_64, K.c[2]), K.s2);
  }
}

// 2-bit: word = 8 pairs, pair k at bits 2k / 16+2k.
__device__ __forceinline__ uint32_t dq2_pair(uint32_t w, int k, const DqConst& K) {
  uint32_t ww = k >= 5 ? (w >> 10) : w;
  int kk = k >= 5 ? k - 5 : k;
  const uint32_t masks[5] = {0x00030003u, 0x000C000Cu, 0x00300030u, 0x00C000C0u, 0x03000300u};
  const uint32_t mul[5] = {0x3C003C00u, kH2_1_4, kH2_1_16, kH2_1_64, kH2_1_256};
  uint32_t v = (ww & masks[kk]) | FW_MAGIC;
  if (kk == 0) return hmul2_u(hadd2_u(v, K.c[0]), K.s2);
  return hmul2_u(hfma2_u(v, mul[kk], K.c[kk]), K.s2);
}

__device__ __forceinline__ uint32_t cvt_e4m3x2_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// Dequantize this thread's 64 columns (half h of the 128-column group) of row r from the packed block at `wb`
// into the A stage at `a_kb` (the k-block of this half, 128 rows x 128 B, 128-byte swizzle).
template <int FMT, int H>
__device__ __forceinline__ void dequant_half(uint32_t wb, int r, uint32_t a_kb) {
  const uint32_t row_base = a_kb + r * 128;
  const int sw = r & 7;
  if constexpr (FMT == 4 || FMT == 3 || FMT == 2) {
    constexpr int NW = FMT == 4 ? 16 : (FMT == 3 ? 13 : 8);
    const uint32_t sz = wb + NW * 512;
    uint16_t sbits;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sbits) : "r"(sz + 2 * r));
    uint32_t zb;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(zb) : "r"(sz + 256 + r));
    DqConst K;
    __half sh = __ushort_as_half(sbits);
    K.s2 = h2_as_u32(__half2(sh, sh));
    const float z = (float)zb;
    if constexpr (FMT == 4) {
      K.c[0] = h2c(-(1024.f + z));
      K.c[1] = h2c(-(64.f + z));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        uint32_t w = lds32(wb + ((8 * H + i) * 128 + r) * 4);
        uint32_t o[4];
        dq4_word(w, K, o);
        sts128(row_base + ((i ^ sw) << 4), o[0], o[1], o[2], o[3]);
      }
    } else if constexpr (FMT == 3) {
      K.c[0] = h2c(-(1024.f + z));
      K.c[1] = h2c(-(128.f + z));
      K.c[2] = h2c(-(16.f + z));
      constexpr int W0 = (32 * H) / 5;
      constexpr int W1 = (32 * H + 31) / 5;
      uint32_t wr[W1 - W0 + 1];
#pragma unroll
      for (int i = 0; i <= W1 - W0; ++i) wr[i] = lds32(wb + ((W0 + i) * 128 + r) * 4);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int p = 32 * H + 4 * c + j;
          o[j] = dq3_pair(wr[p / 5 - W0], p % 5, K);
        }
        sts128(row_base + ((c ^ sw) << 4), o[0], o[1], o[2], o[3]);
      }
    } else {
      K.c[0] = h2c(-(1024.f + z));
      K.c[1] = h2c(-(256.f + z));
      K.c[2] = h2c(-(64.f + z));
      K.c[3] = h2c(-(16.f + z));
      K.c[4] = h2c(-(4.f + z));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t w = lds32(wb + ((4 * H + i) * 128 + r) * 4);
        uint32_t o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = dq2_pair(w, k, K);
        sts128(row_base + (((2 * i) ^ sw) << 4), o[0], o[1], o[2], o[3]);
        sts128(row_base + (((2 * i + 1) ^ sw) << 4), o[4], o[5], o[6], o[7]);
      }
    }
  } else if constexpr (FMT == 8) {
    float scale;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(scale) : "r"(wb + 32 * 512));
    const uint32_t s2 = h2c(scale);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t w0 = lds32(wb + ((16 * H + 2 * c) * 128 + r) * 4);
      uint32_t w1 = lds32(wb + ((16 * H + 2 * c + 1) * 128 + r) * 4);
      uint32_t o0 = hmul2_u(cvt_e4m3x2_f16x2((uint16_t)(w0 & 0xFFFF)), s2);
      uint32_t o1 = hmul2_u(cvt_e4m3x2_f16x2((uint16_t)(w0 >> 16)), s2);
      uint32_t o2 = hmul2_u(cvt_e4m3x2_f16x2((uint16_t)(w1 & 0xFFFF)), s2);
      uint32_t o3 = hmul2_u(cvt_e4m3x2_f16x2((uint16_t)(w1 >> 16)), s2);
      sts128(row_base + ((c ^ sw) << 4), o0, o1, o2, o3);
    }
  } else {  // fp16 passthrough
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = lds32(wb + ((32 * H + 4 * c + j) * 128 + r) * 4);
      sts128(row_base + ((c ^ sw) << 4), o[0], o[1], o[2], o[3]);
    }
  }
}

template <int FMT>
__device__ __forceinline__ void dequant_block(uint32_t wb, int r, int h, uint32_t a_stage) {
  if (h == 0)
    dequant_half<FMT, 0>(wb, r, a_stage);
  else
    dequant_half<FMT, 1>(wb, r, a_stage + 16384);
}

struct Work {
  int e, t0, nt, item, tile, split, g0, g1;
};

__device__ __forceinline__ void item_of(const WGemmArgs& a, int idx, int& e, int& t0, int& nt);

// Work index -> (token item, 128-row tile, K split); splits of one tile are consecutive.
__device__ __forceinline__ Work decode_work(const WGemmArgs& a, int w, int KS) {
  Work wk;
  wk.split = w % KS;
  const int rest = w / KS;
  wk.tile = rest % a.row_tiles;
  wk.item = rest / a.row_tiles;
  item_of(a, wk.item, wk.e, wk.t0, wk.nt);
  wk.g0 = wk.split * a.kg / KS;
  wk.g1 = (wk.split + 1) * a.kg / KS;
  return wk;
}

__device__ __forceinline__ void item_of(const WGemmArgs& a, int idx, int& e, int& t0, int& nt) {
  if (a.dense_T >= 0) {
    e = 0;
    t0 = idx * a.n_tile;
    nt = min(a.n_tile, a.dense_T - t0);
  } else {
    int4 it = a.items[idx];
    e = it.x;
    t0 = it.y;
    nt = it.z;
  }
}

template <int N>
__global__ void __launch_bounds__(kThreads, 1)
    wgemm_kernel(const WGemmArgs a, const __grid_constant__ CUtensorMap bmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - smem_u32(smem_raw));

  const int P = a.ab_stages, S = a.w_stages;
  const uint32_t a_bytes = 32768, b_bytes = 2 * N * 128;
  const uint32_t ab_stage = a_bytes + b_bytes;
  const uint32_t w_off = P * ab_stage;
  const uint32_t bar_off = w_off + S * a.w_stage_bytes;
  // barriers: w_full[S], w_empty[S], b_full[P], a_ready[P], ab_empty[P], acc_full[2], acc_empty[2], done
  const uint32_t bar_w_full = base + bar_off;
  const uint32_t bar_w_empty = bar_w_full + 8 * S;
  const uint32_t bar_b_full = bar_w_empty + 8 * S;
  const uint32_t bar_a_ready = bar_b_full + 8 * P;
  const uint32_t bar_ab_empty = bar_a_ready + 8 * P;
  const uint32_t bar_acc_full = bar_ab_empty + 8 * P;
  const uint32_t bar_acc_empty = bar_acc_full + 16;
  const uint32_t bar_done = bar_acc_empty + 16;
  const uint32_t misc_off = bar_off + 8 * (2 * S + 3 * P + 5);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base_ptr + misc_off + 4);
  const uint32_t epi_off = (misc_off + 16 + 127) & ~127u;  // 64 x 16 fp32 exchange for silu*up

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ncols = N * 2 < 32 ? 32 : N * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(bar_w_full + 8 * s, 1);
      mbar_init(bar_w_empty + 8 * s, 4);  // one dequant team (4 warps) per stage
    }
    for (int p = 0; p < P; ++p) {
      mbar_init(bar_b_full + 8 * p, 1);
      mbar_init(bar_a_ready + 8 * p, 4);
      mbar_init(bar_ab_empty + 8 * p, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, kEpiThreads / 32);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc_dyn(base + misc_off, ncols);
  }
  if (warp == 0 && lane == 0) prefetch_tmap(&bmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_items = a.dense_T >= 0 ? (a.dense_T + a.n_tile - 1) / a.n_tile : min(*a.n_items, a.max_items);
  const int KS = a.k_splits > 1 ? a.k_splits : 1;
  const int total = n_items * a.row_tiles * KS;
  const uint64_t lim = a.timeout_ns;
  int* err = a.err;

  if (warp == 0) {
    // ---------------------------------------------------------------- weight producer (bulk TMA)
    if (elect_one()) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t k = 0;
      for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
        const Work wk = decode_work(a, w, KS);
        const int fmt = a.exp_fmt[wk.e];
        const uint32_t bb = wgemm_block_bytes(fmt);
        const uint8_t* src = a.wbase + a.exp_off[wk.e] + (size_t)wk.tile * a.kg * bb;
        for (int g = wk.g0; g < wk.g1; ++g, ++k) {
          const int s = k % S;
          if (!mbar_wait_sleepy(bar_w_empty + 8 * s, ((k / S) & 1) ^ 1, err, 1001, abort_flag, lim, a.sleep_ns)) break;
          if (a.dbg & 8) {
            mbar_arrive(bar_w_full + 8 * s);
          } else {
            mbar_arrive_expect_tx(bar_w_full + 8 * s, bb);
            tma_bulk_g2s(base + w_off + s * a.w_stage_bytes, src + (size_t)g * bb, bb, bar_w_full + 8 * s, pol);
          }
        }
      }
      // drain: the last S copies must have landed before the CTA may exit
      volatile int no_abort = 0;
      for (uint32_t j = (k > (uint32_t)S ? k - S : 0); j < k; ++j)
        mbar_wait(bar_w_full + 8 * (j % S), (j / S) & 1, err, 1002, &no_abort, lim);
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- token-tile producer (2-D TMA)
    if (elect_one()) {
      uint32_t j = 0;
      for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x) {
        const Work wk = decode_work(a, w, KS);
        for (int g = wk.g0; g < wk.g1; ++g, ++j) {
          const int p = j % P;
          if (!mbar_wait_sleepy(bar_ab_empty + 8 * p, ((j / P) & 1) ^ 1, err, 2001, abort_flag, lim, a.sleep_ns)) break;
          if (a.dbg & 16) {
            mbar_arrive(bar_b_full + 8 * p);
            continue;
          }
          const uint32_t bdst = base + p * ab_stage + a_bytes;
          mbar_arrive_expect_tx(bar_b_full + 8 * p, b_bytes);
          tma_load_2d(bdst, &bmap, g * 128, a.b_row0 + wk.t0, bar_b_full + 8 * p);
          tma_load_2d(bdst + N * 128, &bmap, g * 128 + 64, a.b_row0 + wk.t0, bar_b_full + 8 * p);
        }
      }
      volatile int no_abort = 0;
      for (uint32_t q = (j > (uint32_t)P ? j - P : 0); q < j; ++q)
        mbar_wait(bar_b_full + 8 * (q % P), (q / P) & 1, err, 2002, &no_abort, lim);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = umma_idesc_f16(128, N, 0);
      uint32_t j = 0;
      int it = 0;
      for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x, ++it) {
        const Work wk = decode_work(a, w, KS);
        const int buf = it & 1;
        if (!mbar_wait(bar_acc_empty + 8 * buf, ((it >> 1) & 1) ^ 1, err, 3001, abort_flag, lim)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + buf * N;
        bool ok = true;
        for (int g = wk.g0; g < wk.g1; ++g, ++j) {
          const int p = j % P;
          const uint32_t par = (j / P) & 1;
          if (!mbar_wait(bar_b_full + 8 * p, par, err, 3002, abort_flag, lim) ||
              !mbar_wait(bar_a_ready + 8 * p, par, err, 3003, abort_flag, lim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t as = base + p * ab_stage;
          const uint32_t bs = as + a_bytes;
          if (!(a.dbg & 2)) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t ad = umma_desc_sw128(as + (kk >> 2) * 16384 + (kk & 3) * 32);
              const uint64_t bd = umma_desc_sw128(bs + (kk >> 2) * (N * 128) + (kk & 3) * 32);
              umma_f16(d, ad, bd, idesc, (g != wk.g0 || kk != 0) ? 1u : 0u);
            }
          }
          umma_commit(bar_ab_empty + 8 * p);
        }
        if (!ok) break;
        umma_commit(bar_acc_full + 8 * buf);
      }
      umma_commit(bar_done);
      volatile int no_abort = 0;
      mbar_wait(bar_done, 0, err, 3004, &no_abort, lim);
    }
  } else if (warp >= 4 && warp < kEpiWarp0) {
    // ---------------------------------------------------------------- dequant (kTeams x 128 threads)
    // kTeams teams of 4 warps take stages round-robin, each thread converting one full row of its team's
    // group, so kTeams groups are converted concurrently: a group's latency chain (wait, convert,
    // signal) is per warp, and with every warp on every group that chain bounded the group rate.
    // Safety of the parity waits: a team may start waiting for use u of a stage only if use u-1 of that stage
    // was its own (parity waits cannot tell use u-1 from u+1); the host makes both ring depths multiples of
    // a.teams, so stage j % P and j % S always recur on the same team (j % a.teams).
    const int d = threadIdx.x - 128;
    const int r = d & 127, team = d >> 7;
    const int teams = a.teams;
    uint32_t k = 0, j = 0;
    for (int w = blockIdx.x; w < total && !*abort_flag && team < teams; w += gridDim.x) {
      const Work wk = decode_work(a, w, KS);
      const int fmt = a.exp_fmt[wk.e];
      bool ok = true;
      for (int g = wk.g0; g < wk.g1; ++g, ++k, ++j) {
        if ((int)(j % teams) != team) continue;
        const int s = k % S, p = j % P;
        // one poller per warp (a.dbg & 64: every thread polls, for comparison)
        const bool waited = (a.dbg & 64)
            ? (mbar_wait(bar_w_full + 8 * s, (k / S) & 1, err, 4001, abort_flag, lim) &&
               mbar_wait(bar_ab_empty + 8 * p, ((j / P) & 1) ^ 1, err, 4002, abort_flag, lim))
            : (mbar_wait_warp(bar_w_full + 8 * s, (k / S) & 1, err, 4001, abort_flag, lim) &&
               mbar_wait_warp(bar_ab_empty + 8 * p, ((j / P) & 1) ^ 1, err, 4002, abort_flag, lim));
        if (!waited) {
          ok = false;
          break;
        }
        const uint32_t wb = base + w_off + s * a.w_stage_bytes;
        const uint32_t as = base + p * ab_stage;
        if (!(a.dbg & 1)) {
          switch (fmt) {
            case 4: dequant_block<4>(wb, r, 0, as); dequant_block<4>(wb, r, 1, as); break;
            case 3: dequant_block<3>(wb, r, 0, as); dequant_block<3>(wb, r, 1, as); break;
            case 2: dequant_block<2>(wb, r, 0, as); dequant_block<2>(wb, r, 1, as); break;
            case 8: dequant_block<8>(wb, r, 0, as); dequant_block<8>(wb, r, 1, as); break;
            default: dequant_block<16>(wb, r, 0, as); dequant_block<16>(wb, r, 1, as); break;
          }
        }
        if (!(a.dbg & 4)) fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_w_empty + 8 * s);
          mbar_arrive(bar_a_ready + 8 * p);
        }
      }
      if (!ok) break;
    }
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue (128 threads)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    float* xch = reinterpret_cast<float*>(base_ptr + epi_off);  // [64 rows][17] fp32
    volatile int* last_flag = reinterpret_cast<volatile int*>(base_ptr + misc_off + 8);
    int it = 0;
    for (int w = blockIdx.x; w < total && !*abort_flag; w += gridDim.x, ++it) {
      const Work wk = decode_work(a, w, KS);
      const int buf = it & 1;
      if (!mbar_wait_sleepy(bar_acc_full + 8 * buf, (it >> 1) & 1, err, 5001, abort_flag, lim, a.sleep_ns)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * N;
      bool emit = !(a.dbg & 32);
      float* part = nullptr;
      if (KS > 1 && emit) {
        // park this split's partial; the last split to arrive for the tile does the epilogue
        const size_t tile_id = (size_t)wk.item * a.row_tiles + wk.tile;
        part = a.workspace + tile_id * (size_t)KS * N * 128;
#pragma unroll 1
        for (int c = 0; c < N / 16; ++c) {
          uint32_t v[16];
          tmem_ld16(taddr + c * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) part[((size_t)wk.split * N + c * 16 + i) * 128 + row] = __uint_as_float(v[i]);
        }
      }
      if (KS > 1 && emit && a.ext_reduce) {
        emit = false;   // the follow-up reduce kernel sums and stores (stream order makes the partials visible)
      } else if (KS > 1 && emit) {
        const size_t tile_id = (size_t)wk.item * a.row_tiles + wk.tile;
        __threadfence();
        named_barrier(1, kEpiThreads);
        if (threadIdx.x == kEpiFirst) {
          const int old = atomicAdd(a.counters + tile_id, 1);
          const int last = old == KS - 1;
          if (last) a.counters[tile_id] = 0;
          *last_flag = last;
        }
        named_barrier(1, kEpiThreads);
        emit = *last_flag != 0;
        if (emit) __threadfence();
      }
      if (emit) {
        const size_t orow0 = (size_t)(a.out_row0 + wk.t0);
#pragma unroll 1
        for (int c = 0; c < N / 16; ++c) {
          float v[16];
          if (KS > 1) {
            // the loads of two splits are issued before their adds (latency overlap); the adds stay in split
            // order, so the sum is the same whichever split arrived last
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = 0.f;
            for (int s2 = 0; s2 < KS; s2 += 2) {
              float t0v[16], t1v[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                t0v[i] = __ldcg(part + ((size_t)s2 * N + c * 16 + i) * 128 + row);
                t1v[i] = (s2 + 1 < KS) ? __ldcg(part + ((size_t)(s2 + 1) * N + c * 16 + i) * 128 + row) : 0.f;
              }
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                v[i] += t0v[i];
                if (s2 + 1 < KS) v[i] += t1v[i];
              }
            }
          } else {
            uint32_t u[16];
            tmem_ld16(taddr + c * 16, u);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(u[i]);
          }
          if (a.epi == WGEMM_EPI_STORE) {
            const int col = wk.tile * 128 + row;
            if (col < a.out_cols) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int n = c * 16 + i;
                if (n < wk.nt) {
                  const float f = v[i] * a.alpha;
                  const size_t o = (orow0 + n) * a.out_ld + col;
                  if (a.row_dst) {
                    // per-row destination (may be a peer GPU's buffer): the expert-parallel combine's
                    // data movement happens here, one store per output element straight into its source
                    reinterpret_cast<float*>(a.row_dst[orow0 + n])[col] = f;
                  } else if (a.fan_n > 0) {
                    // tensor-parallel all-reduce: the partial goes straight into every rank's slot [me]
                    const int64_t par = a.fan_epoch[0] & 1;
                    const int64_t off = (par * a.fan_n + a.fan_me) * a.fan_slot + o;
                    for (int pe = 0; pe < a.fan_n; ++pe) reinterpret_cast<float*>(a.fan_base[pe])[off] = f;
                  } else if (a.out_dtype == WGEMM_OUT_F32) {
                    float* op = reinterpret_cast<float*>(a.out) + o;
                    *op = a.accumulate ? *op + f : f;
                  } else if (a.out_dtype == WGEMM_OUT_BF16) {
                    reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(f);
                  } else {
                    reinterpret_cast<__half*>(a.out)[o] = __float2half_rn(f);
                  }
                }
              }
            }
          } else {
            // silu(gate) * up: tile rows 0-63 are gate features 64*tile.., rows 64-127 the matching up rows
            if (q >= 2) {
#pragma unroll
              for (int i = 0; i < 16; ++i) xch[(row - 64) * 17 + i] = v[i];
            }
            named_barrier(1, kEpiThreads);
            if (q < 2) {
              const int f = wk.tile * 64 + row;
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int n = c * 16 + i;
                if (n < wk.nt && f < a.out_cols) {
                  const float y = silu_f(v[i]) * xch[row * 17 + i];
                  const size_t o = (orow0 + n) * a.out_ld + f;
                  if (a.out_dtype == WGEMM_OUT_BF16)
                    reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(y);
                  else if (a.out_dtype == WGEMM_OUT_F32)
                    reinterpret_cast<float*>(a.out)[o] = y;
                  else
                    reinterpret_cast<__half*>(a.out)[o] = __float2half_rn(y);
                }
              }
            }
            named_barrier(1, kEpiThreads);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acc_empty + 8 * buf);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem_base, ncols);
}

// ------------------------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int make_tmap_2d_f16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                     uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  auto enc = get_encode();
  if (!enc) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

int wgemm_groups_per_stage(int) { return 1; }

size_t wgemm_smem_bytes(int n_tile, int g2, int w_stage_bytes, int w_stages, int ab_stages) {
  size_t ab = (size_t)ab_stages * (32768 + 2 * n_tile * 128);
  size_t w = (size_t)w_stages * w_stage_bytes;
  size_t bars = 8 * (2 * w_stages + 3 * ab_stages + 5) + 16;
  size_t epi = 64 * 17 * 4 + 128;
  return 1024 + ab + w + bars + epi;
}

template <int N>
static int launch_n(const WGemmArgs& a, const CUtensorMap& map, int grid, size_t smem, cudaStream_t st) {
  auto k = wgemm_kernel<N>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k<<<grid, kThreads, smem, st>>>(a, map);
  return (int)cudaGetLastError();
}

// Split-K epilogue as its own launch: block (tile, chunk of 16 tokens), thread = weight row. The partials are
// summed in split order (the same order, hence the same bits, as the in-kernel reduction) and the epilogue of the
// GEMM is applied. silu(gate) * up: thread r < 64 sums gate row r and up row r + 64 of its tile.
__global__ void __launch_bounds__(128) wgemm_splitk_reduce_kernel(const WGemmArgs a, int N, int KS) {
  const int tile_id = blockIdx.x, c = blockIdx.y, row = threadIdx.x;
  const int item = tile_id / a.row_tiles, tile = tile_id % a.row_tiles;
  int e, t0, nt;
  item_of(a, item, e, t0, nt);
  const float* part = a.workspace + (size_t)tile_id * KS * N * 128;
  const size_t orow0 = (size_t)(a.out_row0 + t0);
  if (a.epi == WGEMM_EPI_STORE) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
    for (int s = 0; s < KS; ++s) {
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = __ldcg(part + ((size_t)s * N + c * 16 + i) * 128 + row);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] += t[i];
    }
    const int col = tile * 128 + row;
    if (col >= a.out_cols) return;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int n = c * 16 + i;
      if (n >= nt) continue;
      const float f = v[i] * a.alpha;
      const size_t o = (orow0 + n) * a.out_ld + col;
      if (a.fan_n > 0) {
        const int64_t par = a.fan_epoch[0] & 1;
        const int64_t off = (par * a.fan_n + a.fan_me) * a.fan_slot + o;
        for (int pe = 0; pe < a.fan_n; ++pe) reinterpret_cast<float*>(a.fan_base[pe])[off] = f;
      } else if (a.out_dtype == WGEMM_OUT_F32) {
        float* op = reinterpret_cast<float*>(a.out) + o;
        *op = a.accumulate ? *op + f : f;
      } else if (a.out_dtype == WGEMM_OUT_BF16) {
        reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(f);
      } else {
        reinterpret_cast<__half*>(a.out)[o] = __float2half_rn(f);
      }
    }
  } else {
    if (row >= 64) return;
    float g[16], u[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) g[i] = u[i] = 0.f;
    for (int s = 0; s < KS; ++s) {
      float tg[16], tu[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        tg[i] = __ldcg(part + ((size_t)s * N + c * 16 + i) * 128 + row);
        tu[i] = __ldcg(part + ((size_t)s * N + c * 16 + i) * 128 + row + 64);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        g[i] += tg[i];
        u[i] += tu[i];
      }
    }
    const int f = tile * 64 + row;
    if (f >= a.out_cols) return;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int n = c * 16 + i;
      if (n >= nt) continue;
      const float y = silu_f(g[i]) * u[i];
      const size_t o = (orow0 + n) * a.out_ld + f;
      if (a.out_dtype == WGEMM_OUT_BF16)
        reinterpret_cast<__nv_bfloat16*>(a.out)[o] = __float2bfloat16_rn(y);
      else if (a.out_dtype == WGEMM_OUT_F32)
        reinterpret_cast<float*>(a.out)[o] = y;
      else
        reinterpret_cast<__half*>(a.out)[o] = __float2half_rn(y);
    }
  }
}

int wgemm_splitk_reduce(const WGemmArgs& a, int tiles, cudaStream_t st) {
  wgemm_splitk_reduce_kernel<<<dim3(tiles, a.n_tile / 16), 128, 0, st>>>(a, a.n_tile, a.k_splits);
  return (int)cudaGetLastError();
}

int wgemm_launch(const WGemmArgs& a, const CUtensorMap& bmap, int grid, cudaStream_t st) {
  size_t smem = wgemm_smem_bytes(a.n_tile, 1, a.w_stage_bytes, a.w_stages, a.ab_stages);
  switch (a.n_tile) {
    case 16: return launch_n<16>(a, bmap, grid, smem, st);
    case 32: return launch_n<32>(a, bmap, grid, smem, st);
    case 64: return launch_n<64>(a, bmap, grid, smem, st);
    case 128: return launch_n<128>(a, bmap, grid, smem, st);
    default: return -2;
  }
}

}  // namespace fw
