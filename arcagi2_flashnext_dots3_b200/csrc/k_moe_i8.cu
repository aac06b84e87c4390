// Grouped low-bit MoE GEMM for decode-sized expert groups on tcgen05 `kind::i8`, sm_100a (W4/3/2 x A8).
//
// y[t, r] = sum_g  s_w[r, g] * s_x[t, g] * (sum_{k in g} q[r, k] * x8[t, k]  -  z[r, g] * sum_{k in g} x8[t, k])
//
// The same arithmetic as the CUDA-core grouped GEMV (csrc/k_gemv.cu): unsigned 2/3/4-bit codes q with a zero
// point z and an fp16 scale per (row, 128-column group), activations quantized per (token, group) to int8 by
// `gemv_quant`. The integer dot products move from dp4a to the tensor cores: the row threads only widen codes to
// bytes, the MMA does the products. Results equal the GEMV's bit for bit: the integer dots are exact in both, and
// the per-group fp32 folds run in the same order with the same operations.
//
// CTA (160 threads, kCps per SM), persistent over work units (item, 128-row tile), strided by the grid:
//   warp 0     producer: per (unit, group) one stage = the 2 KB activation tile (16 token rows x 128 int8 by
//              2-D TMA in the 128-byte swizzle, the MMA's B operand as is) + the packed weight block (4.5 to
//              8.6 KB, one 1-D bulk copy), 8 stages in flight
//   warps 1-4  one thread per weight row (TMEM lane = row): read the row's code words from the stage, widen
//              them to 128 bytes in the activations' column order and tcgen05.st them as the A operand of a TMEM slot
//              (5 slots of A 32 columns + D 16 columns). The last of the four warps to finish a group (an
//              acquire-release counter per slot, no polling) issues its 4 x tcgen05.mma kind::i8 (M 128 rows,
//              N 16 tokens, K 32, A read from tensor memory) and commits them to the slot's `done` and the
//              stage's `empty`. kLag groups later every warp folds the group's int32 dots into its fp32
//              accumulators with the group's scales (tcgen05.ld); silu(gate) * up or fp32 stores (optionally to
//              per-row destinations, the expert-parallel combine) after the unit's last group.
// Token rows of the activation tile past the item's n belong to other items (or are TMA zero fill); their D
// columns are never read. Every wait is bounded (%globaltimer): a timeout records an error code (75xx), the CTA
// drains its copies and MMAs in flight (bounded), frees its TMEM and returns without storing.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cstdint>
#include <cstdlib>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "ptx.cuh"
#include "lowbit.cuh"
#include "wgemm.h"

namespace fw {
namespace moei8 {

constexpr int kTok = 16;                 // MMA N (the smallest N of an M = 128 MMA); rows past the item's n unused
constexpr int kMaxTok = 8;               // tokens of one item (plans are built with items of at most 8 tokens)
#ifndef FW_MOE_I8_CPS
#define FW_MOE_I8_CPS 4                  // CTAs per SM
#endif
constexpr int kCps = FW_MOE_I8_CPS;
constexpr int kSlots = kCps >= 4 ? 2 : 5;   // TMEM slots, each A (32 columns = 128 int8 per row) + D (16 columns)
constexpr int kSlotCols = 48;
constexpr int kLag = kSlots - 1;         // groups between storing a group's A and folding its dots
constexpr int kTmemCols = kCps >= 4 ? 128 : 256;
constexpr int kStages = kCps >= 4 ? 4 : 8;
constexpr int kBTile = kTok * 128;       // activation tile bytes (1024-aligned start, 128-byte swizzle)
constexpr int kStageBytes = 11264;       // kBTile + the largest packed block (8576), rounded up to 1024
constexpr int kThreads = 160;            // warp 0 producer, warps 1-4 rows
constexpr int kGshBytes = kTok * 64 * 4;
constexpr int kBarBytes = 8 * (2 * kStages + kSlots + 2) + 4 * kSlots + 16;
constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + kGshBytes + kBarBytes;
static_assert(kSlots * kSlotCols <= kTmemCols, "TMEM slots exceed the allocation");
static_assert(kLag < kSlots, "a slot must be folded before it is rewritten");
static_assert(kBTile + 8576 <= kStageBytes && kStageBytes % 1024 == 0, "stage layout");

struct Args {
  const uint8_t* wbase;
  const int64_t* exp_off;
  const int8_t* exp_fmt;
  int row_tiles, kg;
  const int4* items;
  const int* n_items;
  int max_items;
  const float* xs;                       // [P, kg] activation scales
  const int* xsum;                       // [P, kg] activation code sums
  void* out;
  int out_ld, out_cols, epi;
  const int64_t* row_dst;
  int* err;
  unsigned long long timeout_ns;
};

struct Ctx {
  uint32_t base, full0, empty0, done0, gready, gfree, cnt0, tmem;
  float* gsh;
  volatile int* abort_flag;
  int q, lane, r;
  uint64_t lim;
  __device__ uint32_t stage(int s) const { return base + (uint32_t)s * kStageBytes; }
  __device__ uint32_t full(int s) const { return full0 + 8u * s; }
  __device__ uint32_t empty(int s) const { return empty0 + 8u * s; }
  __device__ uint32_t done(int b) const { return done0 + 8u * b; }
};

__device__ __forceinline__ uint32_t block_bytes(int fmt) { return (fmt == 4 ? 16 : fmt == 3 ? 13 : 8) * 512 + 384; }

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int FMT, int M>
__device__ __forceinline__ void widen(const uint32_t* w, uint32_t (&v)[32]) {
  v[M] = lowbit::quad<FMT, M>(w);
  if constexpr (M + 1 < 32) widen<FMT, M + 1>(w, v);
}

__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return;
  }
}

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t addr, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
  return old;
}

// Fold the dots of global group jj (group gg of the unit) into the accumulators with the group's weight scale /
// zero point. Every row warp waits for the group's MMA here: that wait is also what lets it rewrite the slot's
// A columns kSlots - kLag groups later.
__device__ __forceinline__ bool fold(const Args& a, const Ctx& c, int jj, int gg, int t0, int n, float sw, int z,
                                     float (&acc)[kMaxTok]) {
  float sx[kMaxTok];
  int xsm[kMaxTok];
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) {
    sx[t] = 0.f;
    xsm[t] = 0;
    if (t < n) {
      sx[t] = __ldg(a.xs + (int64_t)(t0 + t) * a.kg + gg);
      xsm[t] = __ldg(a.xsum + (int64_t)(t0 + t) * a.kg + gg);
    }
  }
  const int slot = jj % kSlots;
  if (!mbar_wait_warp(c.done(slot), (uint32_t)(jj / kSlots) & 1u, a.err, 7502, c.abort_flag, c.lim)) return false;
  tc_fence_after();
  uint32_t d[8];
  tmem_ld8(c.tmem + ((uint32_t)(c.q * 32) << 16) + (uint32_t)(slot * kSlotCols + 32), d);
  tmem_ld_wait();
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t)
    if (t < n) acc[t] = fmaf(sw * sx[t], (float)((int)d[t] - z * xsm[t]), acc[t]);
  return true;
}

// Row threads: one work unit (expert e, row tile, tokens t0..t0+n-1). j = global group counter of this CTA;
// last = the last group whose MMA this warp issued (drained on an abort).
template <int FMT>
__device__ __forceinline__ bool row_unit(const Args& a, const Ctx& c, int t0, int n, int tile, int& j, int& ek,
                                         int& last) {
  constexpr int NW = lowbit::NWords<FMT>::value;
  constexpr uint32_t idesc = umma_idesc_i8_us(128, kTok);
  const int G = a.kg;
  float acc[kMaxTok];
#pragma unroll
  for (int t = 0; t < kMaxTok; ++t) acc[t] = 0.f;
  float sw_h[kLag];
  int z_h[kLag];
#pragma unroll
  for (int k = 0; k < kLag; ++k) {
    sw_h[k] = 0.f;
    z_h[k] = 0;
  }
  for (int g = 0; g < G; ++g, ++j) {
    const int s = j % kStages;
    if (!mbar_wait_warp(c.full(s), (uint32_t)(j / kStages) & 1u, a.err, 7501, c.abort_flag, c.lim)) return false;
    const uint32_t pk = c.stage(s) + kBTile;
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = lds32(pk + (uint32_t)((i * 128 + c.r) * 4));
    unsigned short sbits;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sbits) : "r"(pk + NW * 512 + 2 * c.r));
    uint32_t zb;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(zb) : "r"(pk + NW * 512 + 256 + c.r));
    __syncwarp();
    if (c.lane == 0) mbar_arrive(c.empty(s));
    uint32_t v[32];
    widen<FMT, 0>(w, v);
    const int slot = j % kSlots;
    tmem_st32(c.tmem + ((uint32_t)(c.q * 32) << 16) + (uint32_t)(slot * kSlotCols), v);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (c.lane == 0 && (atom_add_acq_rel(c.cnt0 + 4u * slot, 1u) & 3u) == 3u) {
      // the fourth warp of this group: every lane quarter of A is in place (and the stage's B tile landed, which
      // this warp saw through full[s]); issue the group's MMAs
      tc_fence_after();
      const uint64_t bd = umma_desc_sw128(c.stage(s));
      const uint32_t ta = c.tmem + (uint32_t)(slot * kSlotCols);
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_i8_ts(ta + 32, ta + 8 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
      umma_commit(c.done(slot));
      umma_commit(c.empty(s));
      last = j;
    }
    __syncwarp();
    if (g >= kLag && !fold(a, c, j - kLag, g - kLag, t0, n, sw_h[kLag - 1], z_h[kLag - 1], acc)) return false;
#pragma unroll
    for (int k = kLag - 1; k > 0; --k) {
      sw_h[k] = sw_h[k - 1];
      z_h[k] = z_h[k - 1];
    }
    sw_h[0] = __half2float(__ushort_as_half(sbits));
    z_h[0] = (int)zb;
  }
  // the unit's last min(G, kLag) groups: history index d - 1 holds group G - d
#pragma unroll
  for (int d = kLag; d >= 1; --d)
    if (d <= G && !fold(a, c, j - d, G - d, t0, n, sw_h[d - 1], z_h[d - 1], acc)) return false;
  const int row = tile * 128 + c.r;
  if (a.epi == WGEMM_EPI_STORE) {
    if (row < a.out_cols) {
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) {
        if (t < n) {
          float* dst = a.row_dst ? reinterpret_cast<float*>(a.row_dst[t0 + t])
                                 : reinterpret_cast<float*>(a.out) + (int64_t)(t0 + t) * a.out_ld;
          dst[row] = acc[t];
        }
      }
    }
  } else {
    // silu(gate) * up: tile rows 0..63 are gates, 64..127 the matching ups. The up rows' warps hand their sums
    // to the gate rows' warps through shared memory; two mbarriers (bounded waits, unlike a named barrier, so a
    // warp that aborted earlier cannot strand the others) order the hand-off and the buffer's reuse.
    const uint32_t ph = (uint32_t)ek & 1u;
    if (c.r >= 64) {
      if (!mbar_wait_warp(c.gfree, ph ^ 1u, a.err, 7506, c.abort_flag, c.lim)) return false;
#pragma unroll
      for (int t = 0; t < kMaxTok; ++t) c.gsh[t * 64 + (c.r - 64)] = acc[t];
      __syncwarp();
      if (c.lane == 0) mbar_arrive(c.gready);
    } else {
      if (!mbar_wait_warp(c.gready, ph, a.err, 7507, c.abort_flag, c.lim)) return false;
      const int f = tile * 64 + c.r;
      if (f < a.out_cols) {
#pragma unroll
        for (int t = 0; t < kMaxTok; ++t) {
          if (t < n) {
            const float gt = acc[t], up = c.gsh[t * 64 + c.r];
            reinterpret_cast<__half*>(a.out)[(int64_t)(t0 + t) * a.out_ld + f] =
                __float2half_rn(gt / (1.f + __expf(-gt)) * up);
          }
        }
      }
      __syncwarp();
      if (c.lane == 0) mbar_arrive(c.gfree);
    }
    ++ek;
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, kCps) moe_i8_kernel(const Args a, const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  Ctx c;
  c.base = base;
  c.gsh = reinterpret_cast<float*>(gbase + (size_t)kStages * kStageBytes);
  const uint32_t bars = base + kStages * kStageBytes + kGshBytes;
  c.full0 = bars;
  c.empty0 = bars + 8u * kStages;
  c.done0 = bars + 16u * kStages;
  c.gready = c.done0 + 8u * kSlots;
  c.gfree = c.gready + 8u;
  c.cnt0 = c.gfree + 8u;                 // kSlots arrival counters (u32)
  const uint32_t tmem_slot = c.cnt0 + 4u * kSlots;
  c.abort_flag = reinterpret_cast<volatile int*>(gbase + (tmem_slot + 4 - base));
  const int warp = threadIdx.x >> 5;
  c.lane = threadIdx.x & 31;
  c.q = warp & 3;
  c.r = c.q * 32 + c.lane;
  c.lim = a.timeout_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(c.full(s), 1);
      mbar_init(c.empty(s), 5);          // the four row warps + the MMA commit
    }
    for (int b = 0; b < kSlots; ++b) {
      mbar_init(c.done(b), 1);
      reinterpret_cast<volatile uint32_t*>(gbase + (c.cnt0 - base))[b] = 0u;
    }
    mbar_init(c.gready, 2);              // the two warps of up rows 64..127
    mbar_init(c.gfree, 2);               // the two warps of gate rows 0..63
    *c.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && c.lane == 0) prefetch_tmap(&xmap);
  if (warp == 1) tmem_alloc_dyn(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  c.tmem = *reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));
  pdl_wait();                            // launched early behind gemv_quant: the activations must be complete

  const int total = min(*a.n_items, a.max_items) * a.row_tiles;
  int issued = 0, last = -1;
  if (warp == 0) {
    if (c.lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int j = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int item = u / a.row_tiles, tile = u % a.row_tiles;
        const int4 it = a.items[item];
        if (it.z <= 0) continue;
        const uint32_t bb = block_bytes(a.exp_fmt[it.x]);
        const uint8_t* src = a.wbase + a.exp_off[it.x] + (int64_t)tile * a.kg * bb;
        if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) {   // a bulk copy needs a 16-byte aligned source
          atomicCAS(a.err, 0, 7508);
          *c.abort_flag = 1;
          break;
        }
        for (int g = 0; g < a.kg; ++g, ++j) {
          const int s = j % kStages;
          if (!mbar_wait_sleepy(c.empty(s), ((uint32_t)(j / kStages) & 1u) ^ 1u, a.err, 7503, c.abort_flag, c.lim,
                                2000u)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(c.full(s), kBTile + bb);
          tma_load_2d(c.stage(s), &xmap, g * 128, it.y, c.full(s));
          tma_bulk_g2s(c.stage(s) + kBTile, src + (int64_t)g * bb, bb, c.full(s), pol);
          issued = j + 1;
        }
      }
    }
  } else {
    int j = 0, ek = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int item = u / a.row_tiles, tile = u % a.row_tiles;
      const int4 it = a.items[item];
      const int n = min(it.z, kMaxTok);
      if (it.z <= 0) continue;
      const int fmt = a.exp_fmt[it.x];
      bool ok;
      if (fmt == 4) ok = row_unit<4>(a, c, it.y, n, tile, j, ek, last);
      else if (fmt == 3) ok = row_unit<3>(a, c, it.y, n, tile, j, ek, last);
      else ok = row_unit<2>(a, c, it.y, n, tile, j, ek, last);
      if (!ok) break;
    }
  }
  __syncwarp();
  // After an abort, copies and MMAs still in flight must land before the CTA frees its TMEM and exits.
  if (*c.abort_flag && c.lane == 0) {
    if (warp == 0)
      for (int i = issued > kStages ? issued - kStages : 0; i < issued; ++i)
        drain_wait(c.full(i % kStages), (uint32_t)(i / kStages) & 1u, c.lim);
    if (warp > 0 && last >= 0) drain_wait(c.done(last % kSlots), (uint32_t)(last / kSlots) & 1u, c.lim);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(c.tmem, kTmemCols);
  }
}

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

}  // namespace moei8
}  // namespace fw

namespace {

// Same contract as gemv_grouped (csrc/k_gemv.cu) for plans of items with at most 8 tokens: xq int8 [P, K] with
// P >= 16 rows (callers pad; rows past the plan's pairs are never used), xs fp32 / xsum int32 [P, K/128].
void moe_i8(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, int64_t row_tiles, int64_t kg,
            torch::Tensor items, torch::Tensor n_items, int64_t max_items, torch::Tensor xq, torch::Tensor xs,
            torch::Tensor xsum, torch::Tensor out, int64_t out_cols, int64_t epi, c10::optional<torch::Tensor> row_dst,
            torch::Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(xq.is_cuda() && xq.scalar_type() == torch::kInt8 && xq.dim() == 2 && xq.is_contiguous() &&
                  xq.size(1) == kg * 128, "xq must be contiguous int8 [P, kg*128]");
  TORCH_CHECK(xq.size(0) >= fw::moei8::kTok, "xq needs at least 16 rows (pad the activation buffer)");
  TORCH_CHECK(((uintptr_t)xq.data_ptr()) % 16 == 0 && ((uintptr_t)wbase.data_ptr()) % 16 == 0, "16-byte alignment");
  TORCH_CHECK(xs.scalar_type() == torch::kFloat && xsum.scalar_type() == torch::kInt32 &&
                  xs.numel() >= xq.size(0) * kg && xsum.numel() >= xq.size(0) * kg, "xs fp32 / xsum int32 [P, kg]");
  TORCH_CHECK(items.scalar_type() == torch::kInt32 && items.dim() == 2 && items.size(1) == 4, "items int32 [n, 4]");
  TORCH_CHECK(epi == 0 ? out.scalar_type() == torch::kFloat : out.scalar_type() == torch::kHalf, "out dtype");
  TORCH_CHECK(out.is_contiguous(), "out contiguous");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32, "err int32");
  const c10::cuda::CUDAGuard guard(xq.device());
  fw::moei8::Args a{};
  a.wbase = wbase.data_ptr<uint8_t>();
  a.exp_off = exp_off.data_ptr<int64_t>();
  a.exp_fmt = exp_fmt.data_ptr<int8_t>();
  a.row_tiles = (int)row_tiles;
  a.kg = (int)kg;
  a.items = reinterpret_cast<const int4*>(items.data_ptr<int32_t>());
  a.n_items = n_items.data_ptr<int32_t>();
  a.max_items = (int)max_items;
  a.xs = xs.data_ptr<float>();
  a.xsum = xsum.data_ptr<int>();
  a.out = out.data_ptr();
  a.out_ld = (int)out.size(1);
  a.out_cols = (int)out_cols;
  a.epi = (int)epi;
  a.row_dst = row_dst ? row_dst->data_ptr<int64_t>() : nullptr;
  a.err = err.data_ptr<int32_t>();
  a.timeout_ns = (unsigned long long)timeout_ns;
  CUtensorMap xm;
  {
    auto enc = fw::moei8::encoder();
    TORCH_CHECK(enc, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {(cuuint64_t)(kg * 128), (cuuint64_t)xq.size(0)};
    cuuint64_t strides[1] = {(cuuint64_t)(kg * 128)};
    cuuint32_t box[2] = {128, (cuuint32_t)fw::moei8::kTok};
    cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(&xm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "activation tensor map: ", (int)r);
  }
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  static bool attr = false;
  if (!attr) {
    TORCH_CHECK(cudaFuncSetAttribute(fw::moei8::moe_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)fw::moei8::kSmem) == cudaSuccess, "moe_i8 shared memory attribute");
    attr = true;
  }
  const int64_t work = max_items * row_tiles;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(work, (int64_t)sms * fw::moei8::kCps));
  static const bool pdl = !(getenv("FW_PDL") && atoi(getenv("FW_PDL")) == 0);   // FW_PDL=0: plain launch
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(fw::moei8::kThreads);
  cfg.dynamicSmemBytes = fw::moei8::kSmem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = la;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fw::moei8::moe_i8_kernel, a, xm);
  TORCH_CHECK(e == cudaSuccess, "moe_i8 launch failed: ", cudaGetErrorString(e));
}

}  // namespace

void register_moe_i8(pybind11::module& m) {
  m.def("moe_i8", &moe_i8, "grouped low-bit MoE GEMM on tcgen05 kind::i8 (decode-sized expert groups)");
}
