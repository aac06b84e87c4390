// DSA indexer logits on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//     s[t, j] = sum_h w[t, h] * relu(q[t, h] . k[j]),   j <= pos(t),  -FLT_MAX beyond
// For one query row the head dots are a GEMM with the keys as M: D [128 keys x iH heads] = K_tile [128 x iD] .
// Q^T, so every epilogue thread owns one key (its TMEM lane) and forms the weighted ReLU sum over the iH columns
// without any cross-thread reduction.
//
// CTA = (row t, range of 8 key tiles); 6 warps:
//   warp 4      TMA producer: 2-D tiled loads (128-byte swizzle) of 128 keys x 64 dims of the slot's bf16 index
//               keys into a 4-stage ring
//   warp 5      MMA issuer (one thread): iD / 16 MMAs per tile (M = 128 keys, N = iH, bf16) into one of two
//               TMEM accumulators
//   warps 0-3   epilogue: tcgen05.ld of the key's iH scores, relu, weights, sum, masked store
// Every wait is bounded (%globaltimer); on a timeout the CTA records an error code, drains its copies and MMAs
// and releases TMEM.
//
// Replaces the reference's indexer logits (dotsnote/engine/arcstats_pkg/arcstats/dsa_sm89.py:44-97 and the
// sharded key write + logits of shard_indexer.py:42-145); math of dotsnote/training/finetune/student.py:209-240.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cfloat>
#include "ptx.cuh"
#include "wgemm.h"

namespace {

using namespace fw;

constexpr int KT = 128;        // keys per tile (MMA M)
constexpr int TPC = 8;         // tiles per CTA
constexpr int NS = 4;          // TMA stages
constexpr int kThreads = 192;

struct DsaArgs {
  const float* iq;             // [T, iH, iD]
  const float* iw;             // [T, iH]
  int iH, iD, max_len;
  const int *slots, *positions;
  int n_tok;
  float* scores;               // [T, ld]
  int ld;
  int* err;
  uint64_t timeout_ns;
};

__host__ __device__ inline uint32_t dsa_smem(int iH, int iD) {
  const uint32_t q = (iD / 64) * iH * 128, stage = (iD / 64) * KT * 128;
  return 1024 + q + NS * stage + iH * 4 + (2 * NS + 4) * 8 + 16;
}

__global__ void __launch_bounds__(kThreads, 1) dsa_tc_kernel(const DsaArgs a, const __grid_constant__ CUtensorMap kmap) {
  extern __shared__ uint8_t smem_dyn[];
  const uint32_t base = (smem_u32(smem_dyn) + 1023) & ~1023u;
  uint8_t* gbase = smem_dyn + (base - smem_u32(smem_dyn));
  const int iH = a.iH, iD = a.iD, nkb = iD / 64;
  const uint32_t q_bytes = nkb * iH * 128, stage_bytes = nkb * KT * 128;
  const uint32_t sQ = base, sS = base + q_bytes;
  float* w_sm = reinterpret_cast<float*>(gbase + q_bytes + NS * stage_bytes);
  const uint32_t bars = base + q_bytes + NS * stage_bytes + iH * 4;
  const uint32_t full0 = bars, empty0 = bars + NS * 8, accf0 = bars + 2 * NS * 8, acce0 = accf0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + q_bytes + NS * stage_bytes + iH * 4 + (2 * NS + 4) * 8);
  volatile int* abort_w = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = blockIdx.x, b = row / a.n_tok;
  const int pos = a.positions[b] + row % a.n_tok, slot = a.slots[b];
  const int tile0 = blockIdx.y * TPC;
  const int n_valid_tiles = (pos + KT) / KT;                  // tiles holding keys 0..pos
  const int nt = max(0, min(TPC, n_valid_tiles - tile0));
  float* srow = a.scores + (int64_t)row * a.ld;

  if (nt == 0) {  // the whole range lies past the row's position
    for (int j = tile0 * KT + tid; j < min(a.ld, (tile0 + TPC) * KT); j += kThreads) srow[j] = -FLT_MAX;
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(accf0 + 8 * k, 1);
      mbar_init(acce0 + 8 * k, 4);
    }
    *abort_w = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc<128>(smem_u32(tmem_slot));
  // Q (bf16, K-major, 128-byte swizzle) and the head weights
  if (warp < 4) {
    const float* q = a.iq + (int64_t)row * iH * iD;
    for (int i = tid; i < iH * iD / 8; i += 128) {
      const int h = i / (iD / 8), d0 = (i % (iD / 8)) * 8;
      const float4 f0 = *reinterpret_cast<const float4*>(q + (int64_t)h * iD + d0);
      const float4 f1 = *reinterpret_cast<const float4*>(q + (int64_t)h * iD + d0 + 4);
      __nv_bfloat162 p0 = __floats2bfloat162_rn(f0.x, f0.y), p1 = __floats2bfloat162_rn(f0.z, f0.w),
                     p2 = __floats2bfloat162_rn(f1.x, f1.y), p3 = __floats2bfloat162_rn(f1.z, f1.w);
      const uint32_t addr = sQ + (d0 / 64) * iH * 128 + h * 128 + ((((d0 & 63) >> 3) ^ (h & 7)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(*reinterpret_cast<uint32_t*>(&p0)),
                   "r"(*reinterpret_cast<uint32_t*>(&p1)), "r"(*reinterpret_cast<uint32_t*>(&p2)),
                   "r"(*reinterpret_cast<uint32_t*>(&p3))
                   : "memory");
    }
    for (int i = tid; i < iH; i += 128) w_sm[i] = a.iw[(int64_t)row * iH + i];
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tmap(&kmap);
      int issued = 0;
      for (int i = 0; i < nt; ++i) {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(empty0 + 8 * s, ((i / NS) - 1) & 1, a.err, 7201, abort_w, a.timeout_ns)) break;
        mbar_arrive_expect_tx(full0 + 8 * s, stage_bytes);
        const int y = slot * a.max_len + (tile0 + i) * KT;
        for (int kb = 0; kb < nkb; ++kb) tma_load_2d(sS + s * stage_bytes + kb * KT * 128, &kmap, kb * 64, y, full0 + 8 * s);
        issued = i + 1;
      }
      volatile int no_abort = 0;
      for (int i = max(0, issued - NS); i < issued; ++i)
        mbar_wait(full0 + 8 * (i % NS), (i / NS) & 1, a.err, 7202, &no_abort, a.timeout_ns);
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(128, iH, 1);   // bf16 x bf16 -> fp32
      int done = 0;
      for (int i = 0; i < nt; ++i) {
        const int s = i % NS, ab = i & 1;
        if (!mbar_wait(full0 + 8 * s, (i / NS) & 1, a.err, 7203, abort_w, a.timeout_ns)) break;
        if (i >= 2 && !mbar_wait(acce0 + 8 * ab, ((i >> 1) - 1) & 1, a.err, 7204, abort_w, a.timeout_ns)) break;
        tc_fence_after();
        const uint64_t kd0 = umma_desc_sw128(sS + s * stage_bytes), qd0 = umma_desc_sw128(sQ);
        for (int kb = 0; kb < nkb; ++kb)
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)
            umma_f16(tmem + ab * iH, kd0 + (uint64_t)((kb * KT * 128) >> 4) + 2 * k4,
                     qd0 + (uint64_t)((kb * iH * 128) >> 4) + 2 * k4, idesc, (kb | k4) ? 1u : 0u);
        umma_commit(empty0 + 8 * s);
        umma_commit(accf0 + 8 * ab);
        done = i + 1;
      }
      volatile int no_abort = 0;
      if (done > 0) mbar_wait(accf0 + 8 * ((done - 1) & 1), ((done - 1) >> 1) & 1, a.err, 7205, &no_abort, a.timeout_ns);
    }
    __syncwarp();
  } else {
    // epilogue: lane = key within the tile
    for (int i = 0; i < nt; ++i) {
      const int ab = i & 1;
      const bool ok = mbar_wait_warp(accf0 + 8 * ab, (i >> 1) & 1, a.err, 7206, abort_w, a.timeout_ns);
      if (!ok) break;
      tc_fence_after();
      float acc = 0.f;
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + ab * iH;
      for (int c = 0; c < iH; c += 16) {
        uint32_t r[16];
        tmem_ld16(ta + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = fmaf(w_sm[c + k], fmaxf(__uint_as_float(r[k]), 0.f), acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce0 + 8 * ab);
      const int j = (tile0 + i) * KT + warp * 32 + lane;
      if (j < a.ld) srow[j] = j <= pos ? acc : -FLT_MAX;
    }
    // tiles of this range past the row's position
    for (int j = (tile0 + nt) * KT + tid; j < min(a.ld, (tile0 + TPC) * KT); j += 128) srow[j] = -FLT_MAX;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

bool dsa_tc_supported(int64_t iH, int64_t iD) { return iH % 16 == 0 && iH >= 16 && iH <= 64 && iD % 64 == 0 && iD <= 256; }

void d3_dsa_scores_tc(torch::Tensor iq, torch::Tensor iw, torch::Tensor keys, torch::Tensor slots,
                      torch::Tensor positions, int64_t n_tok, torch::Tensor scores, torch::Tensor err,
                      int64_t timeout_ns) {
  TORCH_CHECK(iq.dim() == 3 && iq.scalar_type() == torch::kFloat && iq.is_contiguous(), "iq fp32 [T, iH, iD]");
  const int T = iq.size(0), iH = iq.size(1), iD = iq.size(2);
  TORCH_CHECK(dsa_tc_supported(iH, iD), "tensor-core DSA needs iH % 16 == 0 (<= 64) and iD % 64 == 0");
  TORCH_CHECK(iw.scalar_type() == torch::kFloat && iw.is_contiguous() && iw.size(0) == T && iw.size(1) == iH, "iw");
  TORCH_CHECK(keys.scalar_type() == torch::kBFloat16 && keys.is_contiguous() && keys.dim() == 3 && keys.size(2) == iD,
              "keys bf16 [S, max_len, iD]");
  TORCH_CHECK(scores.scalar_type() == torch::kFloat && scores.is_contiguous() && scores.size(0) == T, "scores");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.numel() >= 2, "err word");
  if (!T) return;
  const c10::cuda::CUDAGuard guard(iq.device());
  DsaArgs a{};
  a.iq = iq.data_ptr<float>();
  a.iw = iw.data_ptr<float>();
  a.iH = iH;
  a.iD = iD;
  a.max_len = keys.size(1);
  a.slots = slots.data_ptr<int32_t>();
  a.positions = positions.data_ptr<int32_t>();
  a.n_tok = n_tok;
  a.scores = scores.data_ptr<float>();
  a.ld = scores.size(1);
  a.err = err.data_ptr<int32_t>();
  a.timeout_ns = (uint64_t)timeout_ns;
  CUtensorMap kmap;
  // the 16-bit copy is bitwise: the fp16 map serves bf16 keys
  const int rc = make_tmap_2d_f16(&kmap, keys.data_ptr(), (uint64_t)keys.size(0) * keys.size(1), iD, iD, 64, KT, true);
  TORCH_CHECK(rc == 0, "cuTensorMapEncodeTiled failed: ", rc);
  const uint32_t smem = dsa_smem(iH, iD);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dsa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr = true;
  }
  const int ranges = (a.ld + TPC * KT - 1) / (TPC * KT);
  dsa_tc_kernel<<<dim3(T, ranges), kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(a, kmap);
}

}  // namespace

void register_dsa(pybind11::module& m) {
  m.def("d3_dsa_scores_tc", &d3_dsa_scores_tc);
  m.def("d3_dsa_tc_supported", &dsa_tc_supported);
}
