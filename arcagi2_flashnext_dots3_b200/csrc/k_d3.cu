// Dots3-Note-shaped model kernels (MLA attention with DSA / sliding-window layers, sigmoid-routed MoE).
//
//   d3_add_rms     : h += y (optional), out = rms(h) * w  (residual add fused with the next pre-norm)
//   d3_mla_prep    : after the fused [q_a | kv_a | g | idx_k | idx_w] GEMM: q latent RMSNorm (fp16 out), kv latent
//                    RMSNorm + rope-key RMSNorm + interleaved RoPE written as one FP8 row of the paged latent
//                    cache, indexer key LayerNorm + RoPE into the per-slot index-key cache, indexer head weights
//   d3_mla_qsplit  : after the fused [q_b | idx_q] GEMM: q_nope as [H, T, dn] (input of the per-head absorption
//                    GEMM), RoPE'd q_pe [T, H, dr], RoPE'd indexer queries [T, iH, iD]
//   d3_dsa_scores  : DSA indexer logits s[t, j] = sum_h w[t, h] * relu(q[t, h] . k[j]) for j <= pos(t)
//   d3_mla_attn    : latent-space attention (MQA over the shared latent rows): scores q_lat . c_j + q_pe . r_j,
//                    online softmax, o_lat = sum p_j c_j; rows = DSA top-k list, all causal rows, or the window
//   d3_mla_out     : o [H, T, dv] * sigmoid(gate [T, H]) -> fp16 [T, H * dv] (input of o_proj)
//   d3_route       : sigmoid scores, top-k of score + correction bias, renormalized weights * route scale
//
// Reference behavior: dotsnote/training/finetune/student.py:209-259 (MLA, DSA mask), :322-343 (MoE routing);
// the serving kernels it replaces: dotsnote/engine/arcstats_pkg/arcstats/csrc/offload_attn.cu (sparse MLA decode
// over FP8 576-byte latent rows), csrc/swa_attn.cu (window-513 MLA decode over 1088-byte rows),
// arcstats/dsa_sm89.py:44-97 (indexer logits), arcstats/lowbit_fuse.py:20 (fused sigmoid router).
// These run on CUDA cores; every launch has a host-side shape check.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cfloat>

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()
#define CK(x) TORCH_CHECK(x)

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x == 256 (scratch: 8 floats).
__device__ __forceinline__ float bsum(float v, float* red) {
  v = wsum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return wsum(t);
}

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return (float)*p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ldf<__half>(const __half* p) { return __half2float(*p); }

template <typename T>
__device__ __forceinline__ void stf(T* p, float v) { *p = (T)v; }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ void stf<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <>
__device__ __forceinline__ void stf<__nv_fp8_e4m3>(__nv_fp8_e4m3* p, float v) { *p = __nv_fp8_e4m3(v); }

// ------------------------------------------------------------------------------------------ add + rms
template <typename OT>
__global__ void __launch_bounds__(256) add_rms_kernel(float* h, const float* y, const float* w, int n, float eps,
                                                      OT* out) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float* hr = h + row * n;
  const float* yr = y ? y + row * n : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = hr[i];
    if (yr) {
      v += yr[i];
      hr[i] = v;
    }
    ss += v * v;
  }
  const float r = rsqrtf(bsum(ss, red) / n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) stf(out + row * n + i, hr[i] * r * w[i]);
}

// Same, for n % 4 == 0 and n <= 4 * 256 * NV: float4 accesses, the row kept in registers between the two passes.
template <typename OT, int NV>
__global__ void __launch_bounds__(256) add_rms_vec_kernel(float* h, const float* y, const float* w, int n, float eps,
                                                          OT* out) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float4* hr = reinterpret_cast<float4*>(h + row * n);
  const float4* yr = y ? reinterpret_cast<const float4*>(y + row * n) : nullptr;
  const int n4 = n >> 2;
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * 256;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < n4) {
      v[k] = hr[i];
      if (yr) {
        const float4 u = yr[i];
        v[k].x += u.x; v[k].y += u.y; v[k].z += u.z; v[k].w += u.w;
        hr[i] = v[k];
      }
      ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    }
  }
  const float r = rsqrtf(bsum(ss, red) / n + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * 256;
    if (i < n4) {
      const float4 g = w4[i];
      OT* o = out + row * n + 4 * i;
      stf(o, v[k].x * r * g.x);
      stf(o + 1, v[k].y * r * g.y);
      stf(o + 2, v[k].z * r * g.z);
      stf(o + 3, v[k].w * r * g.w);
    }
  }
}

// ------------------------------------------------------------------------------------------ MLA prep
struct PrepArgs {
  const float* P;
  int ldP;
  int qr, kvr, dr, H, iD, iH;       // iD == 0: no indexer (SWA layer)
  int off_g, off_ik, off_iw;
  const float *q_ln, *kv_ln, *kr_ln, *ik_w, *ik_b;
  float qs, kvs, eps;
  const float* rope;                // [max_pos, dr/2, 2] (cos, sin)
  int rope_len;
  __nv_fp8_e4m3* cache;             // [n_blocks, bs, kvr + dr]
  const int* block_table;
  int max_blocks, bs;
  void* idx_cache;                  // [S, max_len / idx_stride, iD] (bf16 or fp32)
  int idx_bf16, idx_max_len;
  int idx_stride, idx_off;          // sharded index: this rank stores positions p = idx_off (mod idx_stride)
  const int *slots, *positions;
  int n_tok;
  __half* qc_out;                   // [T, qr]
  float* gate_out;                  // [T, H]
  float* iw_out;                    // [T, iH]
};

__global__ void __launch_bounds__(256) mla_prep_kernel(PrepArgs a) {
  __shared__ float red[8];
  __shared__ float kp[256];         // normalized rope key before rotation (dr <= 256)
  __shared__ float ikb[512];        // indexer key (iD <= 512)
  const int row = blockIdx.x, b = row / a.n_tok;
  const int pos = a.positions[b] + row % a.n_tok, slot = a.slots[b];
  const float* P = a.P + (int64_t)row * a.ldP;
  const float* rp = a.rope + (int64_t)min(pos, a.rope_len - 1) * a.dr;
  // q latent
  float ss = 0.f;
  for (int i = threadIdx.x; i < a.qr; i += blockDim.x) ss += P[i] * P[i];
  float r = rsqrtf(bsum(ss, red) / a.qr + a.eps) * a.qs;
  for (int i = threadIdx.x; i < a.qr; i += blockDim.x)
    a.qc_out[(int64_t)row * a.qr + i] = __float2half_rn(P[i] * r * a.q_ln[i]);
  // kv latent -> FP8 cache row
  const float* kv = P + a.qr;
  ss = 0.f;
  for (int i = threadIdx.x; i < a.kvr; i += blockDim.x) ss += kv[i] * kv[i];
  r = rsqrtf(bsum(ss, red) / a.kvr + a.eps) * a.kvs;
  const int blk = a.block_table[(int64_t)slot * a.max_blocks + pos / a.bs];
  __nv_fp8_e4m3* crow = a.cache + ((int64_t)blk * a.bs + pos % a.bs) * (a.kvr + a.dr);
  for (int i = threadIdx.x; i < a.kvr; i += blockDim.x) crow[i] = __nv_fp8_e4m3(kv[i] * r * a.kv_ln[i]);
  // rope key: rms, weight, interleaved rotation
  const float* kr = kv + a.kvr;
  ss = 0.f;
  for (int i = threadIdx.x; i < a.dr; i += blockDim.x) ss += kr[i] * kr[i];
  r = rsqrtf(bsum(ss, red) / a.dr + a.eps);
  for (int i = threadIdx.x; i < a.dr; i += blockDim.x) kp[i] = kr[i] * r * a.kr_ln[i];
  __syncthreads();
  for (int i = threadIdx.x; i < a.dr / 2; i += blockDim.x) {
    const float c = rp[2 * i], s = rp[2 * i + 1], x1 = kp[2 * i], x2 = kp[2 * i + 1];
    crow[a.kvr + 2 * i] = __nv_fp8_e4m3(x1 * c - x2 * s);
    crow[a.kvr + 2 * i + 1] = __nv_fp8_e4m3(x2 * c + x1 * s);
  }
  for (int i = threadIdx.x; i < a.H; i += blockDim.x) a.gate_out[(int64_t)row * a.H + i] = P[a.off_g + i];
  if (a.iD == 0) return;
  // indexer key: LayerNorm (eps 1e-6) with weight and bias, RoPE on the first dr dims
  const float* ik = P + a.off_ik;
  float s1 = 0.f;
  for (int i = threadIdx.x; i < a.iD; i += blockDim.x) s1 += ik[i];
  const float mean = bsum(s1, red) / a.iD;
  float s2 = 0.f;
  for (int i = threadIdx.x; i < a.iD; i += blockDim.x) s2 += (ik[i] - mean) * (ik[i] - mean);
  const float inv = rsqrtf(bsum(s2, red) / a.iD + 1e-6f);
  for (int i = threadIdx.x; i < a.iD; i += blockDim.x) ikb[i] = (ik[i] - mean) * inv * a.ik_w[i] + a.ik_b[i];
  __syncthreads();
  const bool keep_key = pos >= a.idx_off && (pos - a.idx_off) % a.idx_stride == 0;
  const int64_t ibase = ((int64_t)slot * a.idx_max_len + (pos - a.idx_off) / a.idx_stride) * a.iD;
  for (int i = threadIdx.x; i < a.iD && keep_key; i += blockDim.x) {
    float v = ikb[i];
    if (i < a.dr) {
      const int p2 = i >> 1;
      const float c = rp[2 * p2], s = rp[2 * p2 + 1];
      v = (i & 1) ? ikb[i] * c + ikb[i - 1] * s : ikb[i] * c - ikb[i + 1] * s;
    }
    if (a.idx_bf16) reinterpret_cast<__nv_bfloat16*>(a.idx_cache)[ibase + i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(a.idx_cache)[ibase + i] = v;
  }
  const float wsc = rsqrtf((float)a.iD) * rsqrtf((float)a.iH);
  for (int i = threadIdx.x; i < a.iH; i += blockDim.x) a.iw_out[(int64_t)row * a.iH + i] = P[a.off_iw + i] * wsc;
}

// ------------------------------------------------------------------------------------------ q split
// grid (rows, head groups of 8 then index-head groups of 8): enough blocks to cover the SMs at decode sizes
__global__ void __launch_bounds__(256) mla_qsplit_kernel(const float* Q, int ldQ, int H, int dn, int dr, int iH,
                                                         int iD, const float* rope, int rope_len,
                                                         const int* positions, int n_tok, int T,
                                                         __nv_bfloat16* q_nope, float* q_pe, float* iq) {
  const int row = blockIdx.x;
  const int pos = positions[row / n_tok] + row % n_tok;
  const float* rp = rope + (int64_t)min(pos, rope_len - 1) * dr;
  const float* q = Q + (int64_t)row * ldQ;
  const int hd = dn + dr, hgroups = (H + 7) / 8;
  if ((int)blockIdx.y < hgroups) {
    const int h0 = blockIdx.y * 8, nh = min(8, H - h0);
    for (int i = threadIdx.x; i < nh * hd; i += blockDim.x) {
      const int hl = i / hd, d = i - hl * hd, h = h0 + hl;
      const float* qh = q + (int64_t)h * hd;
      if (d < dn) {
        q_nope[((int64_t)h * T + row) * dn + d] = __float2bfloat16_rn(qh[d]);
      } else {
        const int e = d - dn, p2 = e >> 1;
        const float c = rp[2 * p2], sn = rp[2 * p2 + 1];
        const float v = (e & 1) ? qh[d] * c + qh[d - 1] * sn : qh[d] * c - qh[d + 1] * sn;
        q_pe[((int64_t)row * H + h) * dr + e] = v;
      }
    }
    return;
  }
  if (!iq) return;
  const int g0 = (blockIdx.y - hgroups) * 8, ng = min(8, iH - g0);
  const float* qi = q + (int64_t)H * hd + (int64_t)g0 * iD;
  for (int i = threadIdx.x; i < ng * iD; i += blockDim.x) {
    const int e = i % iD;
    float v = qi[i];
    if (e < dr) {
      const int p2 = e >> 1;
      const float c = rp[2 * p2], sn = rp[2 * p2 + 1];
      v = (e & 1) ? qi[i] * c + qi[i - 1] * sn : qi[i] * c - qi[i + 1] * sn;
    }
    iq[(int64_t)row * iH * iD + (int64_t)g0 * iD + i] = v;
  }
}

// ------------------------------------------------------------------------------------------ DSA scores
// grid (rows, chunks of 256 keys); one key per thread, the key row held in registers, query heads and weights
// broadcast from shared memory.
template <typename KT, int ID>
__global__ void __launch_bounds__(256) dsa_scores_kernel(const float* iq, const float* iw, int iH, const KT* keys,
                                                         int max_len, const int* slots, const int* positions, int n_tok,
                                                         float* scores, int ld) {
  extern __shared__ float qs[];  // [iH][ID] then [iH] weights
  const int row = blockIdx.x, b = row / n_tok;
  const int pos = positions[b] + row % n_tok;
  const int j = blockIdx.y * blockDim.x + threadIdx.x;
  if ((int)(blockIdx.y * blockDim.x) > pos) {
    if (j < ld) scores[(int64_t)row * ld + j] = -FLT_MAX;
    return;
  }
  for (int i = threadIdx.x; i < iH * ID; i += blockDim.x) qs[i] = iq[(int64_t)row * iH * ID + i];
  for (int i = threadIdx.x; i < iH; i += blockDim.x) qs[iH * ID + i] = iw[(int64_t)row * iH + i];
  __syncthreads();
  if (j >= ld) return;
  float out = -FLT_MAX;
  if (j <= pos && j < max_len) {
    const KT* kr = keys + ((int64_t)slots[b] * max_len + j) * ID;
    float k[ID];
#pragma unroll
    for (int d = 0; d < ID; ++d) k[d] = ldf(kr + d);
    float acc = 0.f;
    for (int h = 0; h < iH; ++h) {
      const float* qh = qs + h * ID;
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < ID; ++d) dot = fmaf(qh[d], k[d], dot);
      acc = fmaf(qs[iH * ID + h], fmaxf(dot, 0.f), acc);
    }
    out = acc;
  }
  scores[(int64_t)row * ld + j] = out;
}

// ------------------------------------------------------------------------------------------ latent attention
struct AttnArgs {
  const __nv_bfloat16* q_lat;  // [H, T, kvr]
  const float* q_pe;           // [T, H, dr]
  const __nv_fp8_e4m3* cache;  // [n_blocks, bs, kvr + dr]
  const int* block_table;
  int max_blocks, bs;
  const int *slots, *positions;
  int n_tok, T, H, kvr, dr;
  const int* sel;              // [T, topk] row positions (first entry -1 = no list), or null
  int topk;
  int window;                  // > 0: rows pos-window+1 .. pos
  float scale;
  __nv_bfloat16* o_lat;        // [H, T, kvr]
};

constexpr int kChunk = 256;

template <int HG, int CPT>  // heads per CTA, latent columns per thread (kvr <= 256 * CPT)
__global__ void __launch_bounds__(256) mla_attn_kernel(AttnArgs a) {
  extern __shared__ float sm[];
  const int D = a.kvr + a.dr;
  float* qsm = sm;                       // [HG][D]
  float* psm = qsm + HG * D;             // [HG][kChunk]
  float* corr = psm + HG * kChunk;       // [HG]
  float* msm = corr + HG;                // [HG] running max
  float* lsm = msm + HG;                 // [HG] running sum
  int* rows = reinterpret_cast<int*>(lsm + HG);  // [kChunk] cache row index
  const int t = blockIdx.x, h0 = blockIdx.y * HG, b = t / a.n_tok;
  const int pos = a.positions[b] + t % a.n_tok, slot = a.slots[b];
  for (int i = threadIdx.x; i < HG * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    qsm[i] = d < a.kvr ? __bfloat162float(a.q_lat[((int64_t)(h0 + h) * a.T + t) * a.kvr + d])
                       : a.q_pe[((int64_t)t * a.H + h0 + h) * a.dr + d - a.kvr];
  }
  if (threadIdx.x < HG) {
    msm[threadIdx.x] = -FLT_MAX;
    lsm[threadIdx.x] = 0.f;
  }
  // row source
  const int* sel = a.sel ? a.sel + (int64_t)t * a.topk : nullptr;
  const bool sparse = sel && sel[0] >= 0;
  int lo = 0, n;
  if (sparse) {
    n = a.topk;
  } else {
    lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
    n = pos - lo + 1;
  }
  float acc[HG][CPT];
#pragma unroll
  for (int h = 0; h < HG; ++h)
#pragma unroll
    for (int c = 0; c < CPT; ++c) acc[h][c] = 0.f;
  __syncthreads();
  const int64_t rowB = a.kvr + a.dr;
  for (int c0 = 0; c0 < n; c0 += kChunk) {
    // phase A: one row per thread, HG scores
    const int i = c0 + threadIdx.x;
    int crow = -1;
    if (i < n) {
      const int p = sparse ? sel[i] : lo + i;
      if (p >= 0 && p <= pos) {
        const int blk = a.block_table[(int64_t)slot * a.max_blocks + p / a.bs];
        crow = blk * a.bs + p % a.bs;
      }
    }
    rows[threadIdx.x] = crow;
    float s[HG];
#pragma unroll
    for (int h = 0; h < HG; ++h) s[h] = 0.f;
    if (crow >= 0) {
      const uint4* src = reinterpret_cast<const uint4*>(a.cache + (int64_t)crow * rowB);
      for (int d0 = 0; d0 < D; d0 += 16) {
        const uint4 v = src[d0 >> 4];
        const __nv_fp8_e4m3* e8 = reinterpret_cast<const __nv_fp8_e4m3*>(&v);
        float kf[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) kf[u] = (float)e8[u];
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          const float* q = qsm + h * D + d0;
          float d = 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u) d = fmaf(q[u], kf[u], d);
          s[h] += d;
        }
      }
    }
#pragma unroll
    for (int h = 0; h < HG; ++h) psm[h * kChunk + threadIdx.x] = crow >= 0 ? s[h] * a.scale : -FLT_MAX;
    __syncthreads();
    // phase B: per-head online softmax update (warp h)
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    for (int h = w; h < HG; h += 8) {
      float m = -FLT_MAX;
      for (int k = l; k < kChunk; k += 32) m = fmaxf(m, psm[h * kChunk + k]);
      m = wmax(m);
      const float mo = msm[h], mn = fmaxf(mo, m);
      float sum = 0.f;
      for (int k = l; k < kChunk; k += 32) {
        const float sv = psm[h * kChunk + k];
        const float pv = sv == -FLT_MAX ? 0.f : __expf(sv - mn);
        psm[h * kChunk + k] = pv;
        sum += pv;
      }
      sum = wsum(sum);
      if (l == 0) {
        const float cf = mo == -FLT_MAX ? 0.f : __expf(mo - mn);
        corr[h] = cf;
        msm[h] = mn;
        lsm[h] = lsm[h] * cf + sum;
      }
    }
    __syncthreads();
    // phase C: P.V over this chunk, thread owns columns threadIdx.x + 256 * c
#pragma unroll
    for (int h = 0; h < HG; ++h)
#pragma unroll
      for (int c = 0; c < CPT; ++c) acc[h][c] *= corr[h];
    const int nr = min(kChunk, n - c0);
    for (int k = 0; k < nr; ++k) {
      const int cr = rows[k];
      if (cr < 0) continue;
      const __nv_fp8_e4m3* src = a.cache + (int64_t)cr * rowB;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const int col = threadIdx.x + 256 * c;
        if (col < a.kvr) {
          const float v = (float)src[col];
#pragma unroll
          for (int h = 0; h < HG; ++h) acc[h][c] = fmaf(psm[h * kChunk + k], v, acc[h][c]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int h = 0; h < HG; ++h) {
    const float inv = lsm[h] > 0.f ? 1.f / lsm[h] : 0.f;
#pragma unroll
    for (int c = 0; c < CPT; ++c) {
      const int col = threadIdx.x + 256 * c;
      if (col < a.kvr) a.o_lat[((int64_t)(h0 + h) * a.T + t) * a.kvr + col] = __float2bfloat16_rn(acc[h][c] * inv);
    }
  }
}

// grid (rows, head groups of 8); sigmoid(gate) once per head, 8 elements per thread when dv % 8 == 0
__global__ void mla_out_kernel(const __nv_bfloat16* o, const float* gate, int H, int T, int dv, __half* out) {
  __shared__ float gs[8];
  const int t = blockIdx.x, h0 = blockIdx.y * 8, nh = min(8, H - h0);
  if ((int)threadIdx.x < nh) gs[threadIdx.x] = 1.f / (1.f + __expf(-gate[(int64_t)t * H + h0 + threadIdx.x]));
  __syncthreads();
  if (dv % 8 == 0) {
    const int per = dv / 8;
    for (int i = threadIdx.x; i < nh * per; i += blockDim.x) {
      const int hl = i / per, d0 = (i - hl * per) * 8, h = h0 + hl;
      const uint4 v = *reinterpret_cast<const uint4*>(o + ((int64_t)h * T + t) * dv + d0);
      const float g = gs[hl];
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      uint32_t r[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[k]));
        const __half2 hh = __floats2half2_rn(f.x * g, f.y * g);
        r[k] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(out + (int64_t)t * H * dv + (int64_t)h * dv + d0) = make_uint4(r[0], r[1], r[2], r[3]);
    }
    return;
  }
  for (int i = threadIdx.x; i < nh * dv; i += blockDim.x) {
    const int hl = i / dv, d = i % dv, h = h0 + hl;
    out[(int64_t)t * H * dv + (int64_t)h * dv + d] =
        __float2half_rn(__bfloat162float(o[((int64_t)h * T + t) * dv + d]) * gs[hl]);
  }
}

// ------------------------------------------------------------------------------------------ routing
// One warp per token: lanes hold E/32 scores; k rounds of warp argmax (ties: lower expert id).
__global__ void route_kernel(const float* logits, int ld, int E, const float* bias, int k, float scale, int T,
                             int32_t* ids, float* w) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* lg = logits + (int64_t)warp * ld;
  constexpr int kMax = 16;  // E <= 512
  float sc[kMax], key[kMax];
#pragma unroll
  for (int i = 0; i < kMax; ++i) {
    const int e = lane + 32 * i;
    float v = e < E ? lg[e] : 0.f;
    v = v != v ? 0.f : v;
    sc[i] = e < E ? 1.f / (1.f + __expf(-v)) : 0.f;
    key[i] = e < E ? sc[i] + bias[e] : -FLT_MAX;
  }
  float tot = 0.f;
  for (int r = 0; r < k; ++r) {
    float best = -FLT_MAX;
    int be = 1 << 30;
#pragma unroll
    for (int i = 0; i < kMax; ++i) {
      const int e = lane + 32 * i;
      if (key[i] > best || (key[i] == best && e < be)) {
        best = key[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ob > best || (ob == best && oe < be)) {
        best = ob;
        be = oe;
      }
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kMax; ++i)
      if (lane + 32 * i == be) {
        s = sc[i];
        key[i] = -FLT_MAX;
      }
    s = wsum(s);
    if (lane == 0) {
      ids[(int64_t)warp * k + r] = min(be, E - 1);
      w[(int64_t)warp * k + r] = s;
    }
    tot += s;
  }
  __syncwarp();
  if (lane == 0)
    for (int r = 0; r < k; ++r) w[(int64_t)warp * k + r] *= scale / fmaxf(tot, 1e-20f);
}

// ------------------------------------------------------------------------------------------ bindings
void d3_add_rms(torch::Tensor h, c10::optional<torch::Tensor> y, torch::Tensor w, double eps, torch::Tensor out) {
  CK(h.is_cuda() && h.scalar_type() == torch::kFloat && h.is_contiguous() && h.dim() == 2);
  const int T = h.size(0), n = h.size(1);
  CK(w.numel() == n && out.size(0) == T && out.size(1) == n && out.is_contiguous());
  if (y) CK(y->scalar_type() == torch::kFloat && y->is_contiguous() && y->sizes() == h.sizes());
  if (!T) return;
  const float* yp = y ? y->data_ptr<float>() : nullptr;
  if (n % 4 == 0 && n <= 4 * 256 * 8) {
    const int nv = (n / 4 + 255) / 256;
#define ARV(OT, PTR)                                                                                   \
  if (nv <= 2) add_rms_vec_kernel<OT, 2><<<T, 256, 0, STREAM>>>(h.data_ptr<float>(), yp, w.data_ptr<float>(), n, \
                                                               (float)eps, PTR);                        \
  else if (nv <= 4) add_rms_vec_kernel<OT, 4><<<T, 256, 0, STREAM>>>(h.data_ptr<float>(), yp, w.data_ptr<float>(), \
                                                                    n, (float)eps, PTR);                \
  else add_rms_vec_kernel<OT, 8><<<T, 256, 0, STREAM>>>(h.data_ptr<float>(), yp, w.data_ptr<float>(), n, (float)eps, PTR);
    if (out.scalar_type() == torch::kHalf) {
      ARV(__half, (__half*)out.data_ptr())
    } else {
      CK(out.scalar_type() == torch::kFloat);
      ARV(float, out.data_ptr<float>())
    }
#undef ARV
    return;
  }
  if (out.scalar_type() == torch::kHalf)
    add_rms_kernel<__half><<<T, 256, 0, STREAM>>>(h.data_ptr<float>(), yp, w.data_ptr<float>(), n, (float)eps,
                                                 (__half*)out.data_ptr());
  else {
    CK(out.scalar_type() == torch::kFloat);
    add_rms_kernel<float><<<T, 256, 0, STREAM>>>(h.data_ptr<float>(), yp, w.data_ptr<float>(), n, (float)eps,
                                                out.data_ptr<float>());
  }
}

void d3_mla_prep(torch::Tensor P, std::vector<int64_t> dims, std::vector<int64_t> offs, torch::Tensor q_ln,
                 torch::Tensor kv_ln, torch::Tensor kr_ln, c10::optional<torch::Tensor> ik_w,
                 c10::optional<torch::Tensor> ik_b, std::vector<double> scal, torch::Tensor rope, torch::Tensor cache,
                 torch::Tensor block_table, c10::optional<torch::Tensor> idx_cache, torch::Tensor slots,
                 torch::Tensor positions, int64_t n_tok, torch::Tensor qc_out, torch::Tensor gate_out,
                 c10::optional<torch::Tensor> iw_out) {
  CK(dims.size() == 6 && (offs.size() == 3 || offs.size() == 5) && scal.size() == 3);
  PrepArgs a{};
  a.P = P.data_ptr<float>();
  a.ldP = P.size(1);
  a.qr = dims[0]; a.kvr = dims[1]; a.dr = dims[2]; a.H = dims[3]; a.iD = dims[4]; a.iH = dims[5];
  a.off_g = offs[0]; a.off_ik = offs[1]; a.off_iw = offs[2];
  a.idx_stride = offs.size() == 5 ? (int)offs[3] : 1;
  a.idx_off = offs.size() == 5 ? (int)offs[4] : 0;
  CK(a.idx_stride >= 1 && a.idx_off >= 0 && a.idx_off < a.idx_stride);
  CK(a.dr <= 256 && a.dr % 2 == 0 && a.iD <= 512);
  CK(cache.scalar_type() == at::kFloat8_e4m3fn && cache.size(2) == a.kvr + a.dr);
  CK(rope.size(1) == a.dr / 2 && rope.size(2) == 2);
  a.q_ln = q_ln.data_ptr<float>(); a.kv_ln = kv_ln.data_ptr<float>(); a.kr_ln = kr_ln.data_ptr<float>();
  a.qs = scal[0]; a.kvs = scal[1]; a.eps = scal[2];
  a.rope = rope.data_ptr<float>(); a.rope_len = rope.size(0);
  a.cache = reinterpret_cast<__nv_fp8_e4m3*>(cache.data_ptr());
  a.block_table = block_table.data_ptr<int32_t>(); a.max_blocks = block_table.size(1); a.bs = cache.size(1);
  if (a.iD) {
    CK(idx_cache && ik_w && ik_b && iw_out);
    a.ik_w = ik_w->data_ptr<float>(); a.ik_b = ik_b->data_ptr<float>();
    a.idx_cache = idx_cache->data_ptr(); a.idx_bf16 = idx_cache->scalar_type() == torch::kBFloat16;
    a.idx_max_len = idx_cache->size(1);
    CK(idx_cache->size(2) == a.iD);
    a.iw_out = iw_out->data_ptr<float>();
  }
  a.slots = slots.data_ptr<int32_t>(); a.positions = positions.data_ptr<int32_t>(); a.n_tok = n_tok;
  CK(qc_out.scalar_type() == torch::kHalf && qc_out.size(1) == a.qr);
  a.qc_out = (__half*)qc_out.data_ptr(); a.gate_out = gate_out.data_ptr<float>();
  const int T = P.size(0);
  if (T) mla_prep_kernel<<<T, 256, 0, STREAM>>>(a);
}

void d3_mla_qsplit(torch::Tensor Q, int64_t H, int64_t dn, int64_t dr, int64_t iH, int64_t iD, torch::Tensor rope,
                   torch::Tensor positions, int64_t n_tok, torch::Tensor q_nope, torch::Tensor q_pe,
                   c10::optional<torch::Tensor> iq) {
  const int T = Q.size(0);
  CK(q_nope.scalar_type() == torch::kBFloat16 && q_nope.size(0) == H && q_nope.size(1) == T && q_nope.size(2) == dn);
  CK(q_pe.size(0) == T && q_pe.size(1) == H && q_pe.size(2) == dr && rope.size(1) == dr / 2);
  if (!T) return;
  const int gy = (int)((H + 7) / 8 + (iq ? (iH + 7) / 8 : 0));
  mla_qsplit_kernel<<<dim3(T, gy), 256, 0, STREAM>>>(Q.data_ptr<float>(), Q.size(1), H, dn, dr, iH, iD, rope.data_ptr<float>(),
                                          rope.size(0), positions.data_ptr<int32_t>(), n_tok, T,
                                          (__nv_bfloat16*)q_nope.data_ptr(), q_pe.data_ptr<float>(),
                                          iq ? iq->data_ptr<float>() : nullptr);
}

template <int ID>
void launch_dsa(const torch::Tensor& iq, const torch::Tensor& iw, const torch::Tensor& keys, const torch::Tensor& slots,
                const torch::Tensor& positions, int n_tok, torch::Tensor& scores) {
  const int rows = iq.size(0), iH = iq.size(1), ld = scores.size(1);
  const size_t sm = (size_t)(iH * ID + iH) * sizeof(float);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(dsa_scores_kernel<__nv_bfloat16, ID>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(dsa_scores_kernel<float, ID>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    attr = true;
  }
  CK(sm <= 160 * 1024);
  dim3 grid(rows, (ld + 255) / 256);
  if (keys.scalar_type() == torch::kBFloat16)
    dsa_scores_kernel<__nv_bfloat16, ID><<<grid, 256, sm, STREAM>>>(
        iq.data_ptr<float>(), iw.data_ptr<float>(), iH, (const __nv_bfloat16*)keys.data_ptr(), keys.size(1),
        slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), n_tok, scores.data_ptr<float>(), ld);
  else
    dsa_scores_kernel<float, ID><<<grid, 256, sm, STREAM>>>(
        iq.data_ptr<float>(), iw.data_ptr<float>(), iH, keys.data_ptr<float>(), keys.size(1),
        slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), n_tok, scores.data_ptr<float>(), ld);
}

void d3_dsa_scores(torch::Tensor iq, torch::Tensor iw, torch::Tensor keys, torch::Tensor slots, torch::Tensor positions,
                   int64_t n_tok, torch::Tensor scores) {
  CK(iq.dim() == 3 && iq.scalar_type() == torch::kFloat && iw.size(1) == iq.size(1));
  if (!iq.size(0)) return;
  switch (iq.size(2)) {
    case 64: launch_dsa<64>(iq, iw, keys, slots, positions, n_tok, scores); break;
    case 128: launch_dsa<128>(iq, iw, keys, slots, positions, n_tok, scores); break;
    default: CK(false && "index_dim must be 64 or 128");
  }
}

template <int HG, int CPT>
void launch_attn(const AttnArgs& a) {
  const size_t sm = (size_t)(HG * (a.kvr + a.dr) + HG * kChunk + 3 * HG) * 4 + kChunk * 4;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(mla_attn_kernel<HG, CPT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  CK(sm <= 200 * 1024);
  mla_attn_kernel<HG, CPT><<<dim3(a.T, a.H / HG), 256, sm, STREAM>>>(a);
}

void d3_mla_attn(torch::Tensor q_lat, torch::Tensor q_pe, torch::Tensor cache, torch::Tensor block_table,
                 torch::Tensor slots, torch::Tensor positions, int64_t n_tok, c10::optional<torch::Tensor> sel,
                 int64_t window, double scale, torch::Tensor o_lat) {
  AttnArgs a{};
  a.H = q_lat.size(0); a.T = q_lat.size(1); a.kvr = q_lat.size(2); a.dr = q_pe.size(2);
  CK(q_lat.scalar_type() == torch::kBFloat16 && o_lat.scalar_type() == torch::kBFloat16 && o_lat.sizes() == q_lat.sizes());
  CK(cache.scalar_type() == at::kFloat8_e4m3fn && cache.size(2) == a.kvr + a.dr && (a.kvr + a.dr) % 16 == 0);
  CK(q_pe.size(0) == a.T && q_pe.size(1) == a.H);
  if (!a.T) return;
  a.q_lat = (const __nv_bfloat16*)q_lat.data_ptr(); a.q_pe = q_pe.data_ptr<float>();
  a.cache = (const __nv_fp8_e4m3*)cache.data_ptr(); a.block_table = block_table.data_ptr<int32_t>();
  a.max_blocks = block_table.size(1); a.bs = cache.size(1);
  a.slots = slots.data_ptr<int32_t>(); a.positions = positions.data_ptr<int32_t>(); a.n_tok = n_tok;
  a.sel = sel ? sel->data_ptr<int32_t>() : nullptr; a.topk = sel ? sel->size(1) : 0;
  a.window = window; a.scale = scale; a.o_lat = (__nv_bfloat16*)o_lat.data_ptr();
  const int cpt = (a.kvr + 255) / 256;
  CK(cpt <= 4);
  const int hg = a.H % 8 == 0 ? 8 : a.H % 4 == 0 ? 4 : a.H % 2 == 0 ? 2 : 1;
#define L_(HG)                                   \
  if (hg == HG) {                                \
    if (cpt == 1) launch_attn<HG, 1>(a);         \
    else if (cpt == 2) launch_attn<HG, 2>(a);    \
    else launch_attn<HG, 4>(a);                  \
    return;                                      \
  }
  L_(8) L_(4) L_(2) L_(1)
#undef L_
}

void d3_mla_out(torch::Tensor o, torch::Tensor gate, torch::Tensor out) {
  const int H = o.size(0), T = o.size(1), dv = o.size(2);
  CK(o.scalar_type() == torch::kBFloat16 && out.scalar_type() == torch::kHalf && out.size(1) == H * dv);
  CK(o.is_contiguous() && out.is_contiguous());
  if (T) mla_out_kernel<<<dim3(T, (H + 7) / 8), 256, 0, STREAM>>>((const __nv_bfloat16*)o.data_ptr(), gate.data_ptr<float>(),
                                                                 H, T, dv, (__half*)out.data_ptr());
}

void d3_route(torch::Tensor logits, int64_t E, torch::Tensor bias, int64_t k, double scale, torch::Tensor ids,
              torch::Tensor w) {
  const int T = logits.size(0);
  CK(E <= 512 && k <= E && logits.size(1) >= E && ids.scalar_type() == torch::kInt32);
  if (T) route_kernel<<<(T * 32 + 255) / 256, 256, 0, STREAM>>>(logits.data_ptr<float>(), logits.size(1), E,
                                                               bias.data_ptr<float>(), k, scale, T,
                                                               ids.data_ptr<int32_t>(), w.data_ptr<float>());
}

}  // namespace

void register_d3(pybind11::module& m) {
  m.def("d3_add_rms", &d3_add_rms);
  m.def("d3_mla_prep", &d3_mla_prep);
  m.def("d3_mla_qsplit", &d3_mla_qsplit);
  m.def("d3_dsa_scores", &d3_dsa_scores);
  m.def("d3_mla_attn", &d3_mla_attn);
  m.def("d3_mla_out", &d3_mla_out);
  m.def("d3_route", &d3_route);
}
