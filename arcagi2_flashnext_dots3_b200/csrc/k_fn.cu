// CUDA-core kernels of the Flash-Next-shaped engine step (everything that is not a weight-streaming GEMM):
// hyper-connection norms/activations/mixing, Gated DeltaNet conv + recurrent update, attention prep with paged
// KV writes, the block indexer (scores + radix top-k), split-K sparse GQA decode attention, MoE routing
// (softmax top-k), expert plan (stable expert sort + tile items), token scatter, weighted combine fused with the
// shared expert and the hyper-connection injection, and greedy argmax.
//
// Math references (student_fn.py = flashnext/training/student/student_fn.py): rms1p :58, GatedResidual :232,
// GDN :251, QSA :295-378, MoE :461-563. Each kernel has a torch twin in ops/fn_ops.py used as its test oracle.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cfloat>
#include <type_traits>
#include <atomic>
#include <cub/block/block_scan.cuh>
#include "ptx.cuh"
#include "kernels.h"

namespace {

#define CK(x) TORCH_CHECK(x)
#define STREAM at::cuda::getCurrentCUDAStream()

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum (blockDim.x multiple of 32, <= 1024). `sh` needs 32 floats.
__device__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  float t = lane < nw ? sh[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

template <typename T>
__device__ __forceinline__ float ldf(const T* p) { return (float)*p; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ldf<__half>(const __half* p) { return __half2float(*p); }
template <>
__device__ __forceinline__ float ldf<__nv_fp8_e4m3>(const __nv_fp8_e4m3* p) { return (float)(*p); }

template <typename T>
__device__ __forceinline__ void stf(T* p, float v) { *p = (T)v; }
template <>
__device__ __forceinline__ void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ void stf<__half>(__half* p, float v) { *p = __float2half_rn(v); }
template <>
__device__ __forceinline__ void stf<__nv_fp8_e4m3>(__nv_fp8_e4m3* p, float v) { *p = __nv_fp8_e4m3(v); }

// 8 consecutive cache elements -> fp32.
__device__ __forceinline__ void load8f(const __nv_fp8_e4m3* p, float (&o)[8]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const uint32_t w[2] = {u.x, u.y};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)((w[j] >> (16 * hh)) & 0xFFFF), __NV_E4M3);
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h2));
      o[4 * j + 2 * hh] = f.x;
      o[4 * j + 2 * hh + 1] = f.y;
    }
  }
}
// 8 e4m3 values held in a uint2 -> 8 floats (pairs converted by the hardware e4m3x2 -> f16x2 conversion)
__device__ __forceinline__ void fp8x8_to_f32(const uint2 raw, float (&o)[8]) {
  const __nv_fp8x2_e4m3* p2 = reinterpret_cast<const __nv_fp8x2_e4m3*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = static_cast<float2>(p2[j]);
    o[2 * j] = f.x;
    o[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ void load8f(const __nv_bfloat16* p, float (&o)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(b[i]);
    o[2 * i] = f.x;
    o[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8f(const float* p, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

// ============================================================================================ embedding
template <typename IT>
__global__ void embed_hc_kernel(const IT* ids, const __nv_bfloat16* table, float* out, int H, int hc, int64_t V) {
  const int t = blockIdx.x;
  const int64_t id = min(max((int64_t)ids[t], (int64_t)0), V - 1);  // out-of-range ids never index past the table
  const __nv_bfloat16* row = table + id * H;
  float* o = out + (int64_t)t * hc * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = __bfloat162float(row[i]);
    for (int s = 0; s < hc; ++s) o[s * H + i] = v;
  }
}

void embed_hc(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t hc) {
  CK(table.scalar_type() == torch::kBFloat16 && table.is_contiguous());
  CK(out.scalar_type() == torch::kFloat && out.is_contiguous());
  const int T = ids.size(0), H = table.size(1);
  if (!T) return;
  if (ids.scalar_type() == torch::kInt64)
    embed_hc_kernel<<<T, 256, 0, STREAM>>>(ids.data_ptr<int64_t>(), (const __nv_bfloat16*)table.data_ptr(),
                                           out.data_ptr<float>(), H, hc, table.size(0));
  else
    embed_hc_kernel<<<T, 256, 0, STREAM>>>(ids.data_ptr<int32_t>(), (const __nv_bfloat16*)table.data_ptr(),
                                           out.data_ptr<float>(), H, hc, table.size(0));
}

// ===================================================================================== hyper-connections
// hn[t, s*H+i] = h * rsqrt(mean_s(h^2) + eps) * (1 + w[s*H+i]), one block per (token, stream).
// One warp per (token, stream): the stream's H values stay in registers (float4 loads, H % 128 == 0, H <= 4096),
// one pass over memory, no block barrier.
template <int V4>
__global__ void hc_prenorm_warp_kernel(const float* h, const float* w, __half* out, int H, int S, int rows, float eps) {
  const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (wid >= rows) return;
  const int s = wid % S;
  const float4* x = reinterpret_cast<const float4*>(h + (int64_t)wid * H);
  const float4* ww = reinterpret_cast<const float4*>(w + (int64_t)s * H);
  float4 v[V4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V4; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < H / 4 ? x[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / H + eps);
  __half2* o = reinterpret_cast<__half2*>(out + (int64_t)wid * H);
#pragma unroll
  for (int j = 0; j < V4; ++j) {
    const int i = lane + 32 * j;
    if (i < H / 4) {
      const float4 a = ww[i];
      o[2 * i] = __floats2half2_rn(v[j].x * r * (1.f + a.x), v[j].y * r * (1.f + a.y));
      o[2 * i + 1] = __floats2half2_rn(v[j].z * r * (1.f + a.z), v[j].w * r * (1.f + a.w));
    }
  }
}

// One block of four warps per (token, stream) row, each warp a quarter of the row in registers (float4 loads): four
// times the warps of the warp-per-row form on a decode batch's few hundred rows.
template <int V4>
__global__ void __launch_bounds__(128) hc_prenorm_split_kernel(const float* h, const float* w, __half* out, int H,
                                                               int S, float eps) {
  __shared__ float red[4];
  const int row = blockIdx.x, s = row % S, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q4 = H / 16;                 // float4 of one quarter
  const float4* x = reinterpret_cast<const float4*>(h + (int64_t)row * H) + warp * q4;
  const float4* ww = reinterpret_cast<const float4*>(w + (int64_t)s * H) + warp * q4;
  float4 v[V4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V4; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < q4 ? x[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const float r = rsqrtf((red[0] + red[1] + red[2] + red[3]) / H + eps);
  __half2* o = reinterpret_cast<__half2*>(out + (int64_t)row * H) + warp * q4 * 2;
#pragma unroll
  for (int j = 0; j < V4; ++j) {
    const int i = lane + 32 * j;
    if (i < q4) {
      const float4 a = ww[i];
      o[2 * i] = __floats2half2_rn(v[j].x * r * (1.f + a.x), v[j].y * r * (1.f + a.y));
      o[2 * i + 1] = __floats2half2_rn(v[j].z * r * (1.f + a.z), v[j].w * r * (1.f + a.w));
    }
  }
}

__global__ void hc_prenorm_kernel(const float* h, const float* w, __half* out, int H, float eps) {
  __shared__ float sh[32];
  const int t = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const float* x = h + ((int64_t)t * S + s) * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) ss += x[i] * x[i];
  ss = block_sum(ss, sh);
  const float r = rsqrtf(ss / H + eps);
  __half* o = out + ((int64_t)t * S + s) * H;
  const float* ww = w + (int64_t)s * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) o[i] = __float2half_rn(x[i] * r * (1.f + ww[i]));
}

void hc_prenorm(torch::Tensor h, torch::Tensor w, torch::Tensor out, int64_t H, double eps) {
  const int T = h.size(0);
  const int hc = h.size(1) / H;
  if (!T) return;
  const int rows = T * hc;
  if (H % 64 == 0 && H <= 4096 && rows <= 4096) {   // decode-sized batches: four warps per row
    if (H <= 2048)
      hc_prenorm_split_kernel<4><<<rows, 128, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                           (__half*)out.data_ptr(), H, hc, (float)eps);
    else
      hc_prenorm_split_kernel<8><<<rows, 128, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                           (__half*)out.data_ptr(), H, hc, (float)eps);
    return;
  }
  if (H % 128 == 0 && H <= 4096) {
    const int blocks = (rows * 32 + 255) / 256;
    if (H <= 1024)
      hc_prenorm_warp_kernel<8><<<blocks, 256, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                            (__half*)out.data_ptr(), H, hc, rows, (float)eps);
    else if (H <= 2560)
      hc_prenorm_warp_kernel<20><<<blocks, 256, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                             (__half*)out.data_ptr(), H, hc, rows, (float)eps);
    else
      hc_prenorm_warp_kernel<32><<<blocks, 256, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                             (__half*)out.data_ptr(), H, hc, rows, (float)eps);
    return;
  }
  hc_prenorm_kernel<<<dim3(T, hc), 256, 0, STREAM>>>(h.data_ptr<float>(), w.data_ptr<float>(),
                                                     (__half*)out.data_ptr(), H, (float)eps);
}

__global__ void hc_act_kernel(const float* z, int ldz, __half* a, float* inj, int rank_pad, int hc, int with_inj) {
  const int t = blockIdx.x;
  const float inv = 1.f / hc;
  for (int i = threadIdx.x; i < rank_pad; i += blockDim.x)
    a[(int64_t)t * rank_pad + i] = __float2half_rn(silu(z[(int64_t)t * ldz + i] * inv));
  if (with_inj && threadIdx.x < hc)
    inj[t * hc + threadIdx.x] = 2.f * sigm(z[(int64_t)t * ldz + rank_pad + threadIdx.x] * inv);
}

void hc_act(torch::Tensor z, torch::Tensor a, torch::Tensor inj, int64_t rank_pad, int64_t hc, bool with_inj) {
  const int T = z.size(0);
  if (!T) return;
  hc_act_kernel<<<T, 128, 0, STREAM>>>(z.data_ptr<float>(), z.size(1), (__half*)a.data_ptr(), inj.data_ptr<float>(),
                                       rank_pad, hc, with_inj);
}

__global__ void hc_mix_kernel(const float* u, const __half* hn, __half* out, int hc, int H) {
  const int t = blockIdx.x;
  const float inv = 1.f / hc;
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H; i += blockDim.x * gridDim.y) {
    float acc = 0.f;
    for (int s = 0; s < hc; ++s) {
      const int64_t o = ((int64_t)t * hc + s) * H + i;
      acc += sigm(u[o]) * __half2float(hn[o]);
    }
    out[(int64_t)t * H + i] = __float2half_rn(acc * inv);
  }
}

// Four columns per thread (16-byte fp32 and 8-byte fp16 accesses): the per-token elementwise kernels of a decode
// step move a few MB each and are bound by instructions per byte and latency, not by bandwidth.
__device__ __forceinline__ float4 h4_to_f4(uint2 v) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ uint2 f4_to_h4(float4 v) {
  __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 r;
  r.x = *reinterpret_cast<uint32_t*>(&a);
  r.y = *reinterpret_cast<uint32_t*>(&b);
  return r;
}

__device__ __forceinline__ void fma4(float4& acc, float a, float4 v) {
  acc.x = fmaf(a, v.x, acc.x);
  acc.y = fmaf(a, v.y, acc.y);
  acc.z = fmaf(a, v.z, acc.z);
  acc.w = fmaf(a, v.w, acc.w);
}

__global__ void hc_mix4_kernel(const float4* u, const uint2* hn, uint2* out, int hc, int H4) {
  const int t = blockIdx.x;
  const float inv = 1.f / hc;
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H4; i += blockDim.x * gridDim.y) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < hc; ++s) {
      const int64_t o = ((int64_t)t * hc + s) * H4 + i;
      const float4 uv = u[o], hv = h4_to_f4(hn[o]);
      acc.x += sigm(uv.x) * hv.x;
      acc.y += sigm(uv.y) * hv.y;
      acc.z += sigm(uv.z) * hv.z;
      acc.w += sigm(uv.w) * hv.w;
    }
    out[(int64_t)t * H4 + i] = f4_to_h4(make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
  }
}

inline bool vec4_ok(int64_t H, std::initializer_list<const void*> ptrs) {
  if (H % 4) return false;
  for (const void* p : ptrs)
    if (reinterpret_cast<uintptr_t>(p) % 16) return false;
  return true;
}

void hc_mix(torch::Tensor u, torch::Tensor hn, torch::Tensor out, int64_t hc, int64_t H) {
  const int T = u.size(0);
  if (!T) return;
  if (vec4_ok(H, {u.data_ptr(), hn.data_ptr(), out.data_ptr()})) {
    const int H4 = H / 4;
    hc_mix4_kernel<<<dim3(T, (H4 + 127) / 128), 128, 0, STREAM>>>(
        (const float4*)u.data_ptr(), (const uint2*)hn.data_ptr(), (uint2*)out.data_ptr(), hc, H4);
    return;
  }
  hc_mix_kernel<<<dim3(T, (H + 255) / 256), 256, 0, STREAM>>>(u.data_ptr<float>(), (const __half*)hn.data_ptr(), (__half*)out.data_ptr(),
                                       hc, H);
}

__global__ void hc_residual_kernel(float* h, const float* y, const float* inj, int hc, int H) {
  const int t = blockIdx.x;
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H; i += blockDim.x * gridDim.y) {
    const float v = y[(int64_t)t * H + i];
    for (int s = 0; s < hc; ++s) h[((int64_t)t * hc + s) * H + i] += v * inj[t * hc + s];
  }
}

__global__ void hc_residual4_kernel(float4* h, const float4* y, const float* inj, int hc, int H4) {
  const int t = blockIdx.x;
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H4; i += blockDim.x * gridDim.y) {
    const float4 v = y[(int64_t)t * H4 + i];
    for (int s = 0; s < hc; ++s) {
      float4& d = h[((int64_t)t * hc + s) * H4 + i];
      float4 a = d;
      fma4(a, inj[t * hc + s], v);
      d = a;
    }
  }
}

void hc_residual(torch::Tensor h, torch::Tensor y, torch::Tensor inj) {
  const int T = h.size(0), hc = inj.size(1), H = y.size(1);
  if (!T) return;
  if (vec4_ok(H, {h.data_ptr(), y.data_ptr()})) {
    const int H4 = H / 4;
    hc_residual4_kernel<<<dim3(T, (H4 + 127) / 128), 128, 0, STREAM>>>(
        (float4*)h.data_ptr(), (const float4*)y.data_ptr(), inj.data_ptr<float>(), hc, H4);
    return;
  }
  hc_residual_kernel<<<dim3(T, (H + 255) / 256), 256, 0, STREAM>>>(h.data_ptr<float>(), y.data_ptr<float>(), inj.data_ptr<float>(), hc, H);
}

// ======================================================================================= Gated DeltaNet
// Causal depthwise conv over [conv_state | new tokens] + SiLU for every channel; updates conv_state in place.
// Rows of proj: seq b token j at b*n_tok + j. One thread per (seq, channel).
// n_commit (optional, per sequence): only the state after the first n_commit[b] tokens is written back (speculative
// verification computes every token's output but commits the accepted prefix in a later pass).
__global__ void gdn_conv_kernel(const float* proj, int ldp, const float* conv_w, float* conv_state, const int* slots,
                                float* out, int C, int kc, int n_tok, int B, const int* n_commit) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * C) return;
  const int b = idx / C, c = idx % C;
  const int s = slots[b];
  const int m = n_commit ? n_commit[b] : n_tok;
  float* st = conv_state + ((int64_t)s * C + c) * (kc - 1);
  float hist[8];  // kc - 1 <= 7
  for (int j = 0; j < kc - 1; ++j) hist[j] = st[j];
  float w[8];
  for (int j = 0; j < kc; ++j) w[j] = conv_w[c * kc + j];
  for (int t = 0; t < n_tok; ++t) {
    const float x = proj[((int64_t)b * n_tok + t) * ldp + c];
    float acc = w[kc - 1] * x;
    for (int j = 0; j < kc - 1; ++j) acc += w[j] * hist[j];
    for (int j = 0; j < kc - 2; ++j) hist[j] = hist[j + 1];
    hist[kc - 2] = x;
    out[((int64_t)b * n_tok + t) * C + c] = silu(acc);
    if (t + 1 == m)
      for (int j = 0; j < kc - 1; ++j) st[j] = hist[j];
  }
}

// Prefill form of the convolution (no commit count): one thread per (sequence, token, channel); the kc-1 inputs
// before a token come from this step's rows or the conv state, which gdn_conv_state_kernel rewrites afterwards.
// Same products in the same order as gdn_conv_kernel.
__global__ void gdn_conv_par_kernel(const float* proj, int ldp, const float* conv_w, const float* conv_state,
                                    const int* slots, float* out, int C, int kc, int n_tok, int B) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * n_tok * C) return;
  const int c = idx % C;
  const int64_t bt = idx / C;
  const int t = bt % n_tok, b = bt / n_tok;
  const float* st = conv_state + ((int64_t)slots[b] * C + c) * (kc - 1);
  const float* w = conv_w + (int64_t)c * kc;
  float acc = w[kc - 1] * proj[((int64_t)b * n_tok + t) * ldp + c];
  for (int j = 0; j < kc - 1; ++j) {
    const int tp = t - (kc - 1) + j;
    const float v = tp >= 0 ? proj[((int64_t)b * n_tok + tp) * ldp + c] : st[kc - 1 + tp];
    acc += w[j] * v;
  }
  out[((int64_t)b * n_tok + t) * C + c] = silu(acc);
}

// The conv state after a prefill step: the last kc-1 inputs (entry j reads entry j + n_tok of the old state when
// the step is shorter than the window, so ascending j never reads an entry it already wrote).
__global__ void gdn_conv_state_kernel(const float* proj, int ldp, float* conv_state, const int* slots, int C, int kc,
                                      int n_tok, int B) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * C) return;
  const int b = idx / C, c = idx % C;
  float* st = conv_state + ((int64_t)slots[b] * C + c) * (kc - 1);
  for (int j = 0; j < kc - 1; ++j) {
    const int tp = n_tok - (kc - 1) + j;
    st[j] = tp >= 0 ? proj[((int64_t)b * n_tok + tp) * ldp + c] : st[j + n_tok];
  }
}

// Gated delta rule for one (sequence, value head) over n_tok tokens; DK = DV = 128, 256 threads:
// thread (j = tid & 127, half = tid >> 7) keeps S[64*half .. 64*half+63][j] in registers.
template <typename ST>
__global__ void __launch_bounds__(256) gdn_recur_kernel(const float* qkv, const float* proj, int ldp, ST* ssm,
                                                        const int* slots, const float* A_log, const float* dt_bias,
                                                        const float* norm_w, __half* out, int nk, int nv, int n_tok,
                                                        float eps, int gate_sigmoid, const int* n_commit) {
  constexpr int DK = 128, DV = 128;
  __shared__ float q_s[DK], k_s[DK], part[2][DV], red[32];
  const int b = blockIdx.x, hv = blockIdx.y;
  const int tid = threadIdx.x, j = tid & 127, half = tid >> 7;
  const int r = nv / nk, hk = hv / r;
  const int s = slots[b];
  const int C = 2 * nk * DK + nv * DV;
  ST* S = ssm + ((int64_t)s * nv + hv) * DK * DV;
  float Sr[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) Sr[i] = ldf(&S[(int64_t)(64 * half + i) * DV + j]);
  const float A = -__expf(A_log[hv]);
  const float dtb = dt_bias[hv];
  const int m = n_commit ? n_commit[b] : n_tok;
  const float scale = rsqrtf((float)DK);
  for (int t = 0; t < n_tok; ++t) {
    const int64_t row = (int64_t)b * n_tok + t;
    const float* x = qkv + row * C;
    const float* pr = proj + row * ldp;
    // q, k of head hk: l2 normalize (eps 1e-6 inside the sqrt)
    float qv = 0.f, kv = 0.f;
    if (tid < DK) {
      qv = x[hk * DK + tid];
      kv = x[nk * DK + hk * DK + tid];
    }
    const float qn = block_sum(tid < DK ? qv * qv : 0.f, red);
    const float kn = block_sum(tid < DK ? kv * kv : 0.f, red);
    if (tid < DK) {
      q_s[tid] = qv * rsqrtf(qn + 1e-6f) * scale;
      k_s[tid] = kv * rsqrtf(kn + 1e-6f);
    }
    const float beta = sigm(pr[C + nv * DV + hv]);
    const float g = A * softplus(pr[C + nv * DV + nv + hv] + dtb);
    const float dec = __expf(g);
    __syncthreads();
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      Sr[i] *= dec;
      acc += Sr[i] * k_s[64 * half + i];
    }
    part[half][j] = acc;
    __syncthreads();
    const float vj = x[2 * nk * DK + hv * DV + j];
    const float u = beta * (vj - (part[0][j] + part[1][j]));
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      Sr[i] += k_s[64 * half + i] * u;
      o += Sr[i] * q_s[64 * half + i];
    }
    __syncthreads();
    part[half][j] = o;
    __syncthreads();
    const float oj = part[0][j] + part[1][j];
    const float ss = block_sum(half == 0 ? oj * oj : 0.f, red);
    if (half == 0) {
      const float on = oj * rsqrtf(ss / DV + eps) * norm_w[j];
      const float z = pr[C + hv * DV + j];
      const float gz = gate_sigmoid ? sigm(z) : silu(z);
      out[row * (nv * DV) + hv * DV + j] = __float2half_rn(on * gz);
    }
    if (t + 1 == m) {
#pragma unroll
      for (int i = 0; i < 64; ++i) stf(&S[(int64_t)(64 * half + i) * DV + j], Sr[i]);
    }
    __syncthreads();
  }
}

// Decode form (one token per sequence, bf16 state) for one (sequence, value head): the 32 KB state arrives by one
// bulk copy into shared memory and leaves by one bulk store, and thread j owns column j of it: a first pass over
// the rows forms (S^T k)_j, a second applies the update and accumulates o_j. The only block-wide steps are the q / k
// norms and the output norm. The arithmetic is gdn_recur_kernel's (its sums over the rows run in one order here
// instead of two halves).
__global__ void __launch_bounds__(128) gdn_decode1_kernel(const float* qkv, const float* proj, int ldp,
                                                          __nv_bfloat16* ssm, const int* slots, const float* A_log,
                                                          const float* dt_bias, const float* norm_w, __half* out,
                                                          int nk, int nv, float eps, int gate_sigmoid,
                                                          const int* n_commit, int* err, uint64_t timeout_ns) {
  constexpr int DK = 128, DV = 128;
  __shared__ __align__(128) __nv_bfloat16 Ss[DK * DV];
  __shared__ float q_s[DK], k_s[DK], red[8];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  const int b = blockIdx.x, hv = blockIdx.y, j = threadIdx.x, warp = j >> 5, lane = j & 31;
  const int hk = hv / (nv / nk);
  __nv_bfloat16* S = ssm + ((int64_t)slots[b] * nv + hv) * DK * DV;
  const uint32_t sbar = fw::smem_u32(&bar), sS = fw::smem_u32(Ss);
  if (j == 0) {
    abort_flag = 0;
    fw::mbar_init(sbar, 1);
    fw::fence_mbar_init();
  }
  __syncthreads();
  if (j == 0) {
    fw::mbar_arrive_expect_tx(sbar, DK * DV * 2);
    fw::tma_bulk_g2s(sS, S, DK * DV * 2, sbar, fw::l2_policy_evict_first());
  }
  const int C = 2 * nk * DK + nv * DV;
  const float* x = qkv + (int64_t)b * C;
  const float* pr = proj + (int64_t)b * ldp;
  const float qv = x[hk * DK + j], kv = x[nk * DK + hk * DK + j];
  float q2 = qv * qv, k2 = kv * kv;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    q2 += __shfl_xor_sync(0xffffffffu, q2, o);
    k2 += __shfl_xor_sync(0xffffffffu, k2, o);
  }
  if (lane == 0) {
    red[warp] = q2;
    red[4 + warp] = k2;
  }
  __syncthreads();
  const float qn = red[0] + red[1] + red[2] + red[3], kn = red[4] + red[5] + red[6] + red[7];
  q_s[j] = qv * rsqrtf(qn + 1e-6f) * rsqrtf((float)DK);
  k_s[j] = kv * rsqrtf(kn + 1e-6f);
  const float beta = sigm(pr[C + nv * DV + hv]);
  const float g = -__expf(A_log[hv]) * softplus(pr[C + nv * DV + nv + hv] + dt_bias[hv]);
  const float dec = __expf(g);
  const float vj = x[2 * nk * DK + hv * DV + j];
  if (j == 0 && !fw::mbar_wait(sbar, 0, err, 6601, &abort_flag, timeout_ns)) abort_flag = 1;
  __syncthreads();                       // q_s, k_s written; the state landed (or the wait gave up)
  const bool ok = !abort_flag;
  float o = 0.f;
  if (ok) {
    float acc = 0.f;
#pragma unroll 8
    for (int r = 0; r < DK; ++r) acc += __bfloat162float(Ss[r * DV + j]) * dec * k_s[r];
    const float u = beta * (vj - acc);
#pragma unroll 8
    for (int r = 0; r < DK; ++r) {
      const float sv = __bfloat162float(Ss[r * DV + j]) * dec + k_s[r] * u;
      o += sv * q_s[r];
      Ss[r * DV + j] = __float2bfloat16_rn(sv);
    }
  }
  float o2 = o * o;
#pragma unroll
  for (int w = 16; w; w >>= 1) o2 += __shfl_xor_sync(0xffffffffu, o2, w);
  __syncthreads();                       // every thread is past its reads of red
  if (lane == 0) red[warp] = o2;
  fw::fence_proxy_async_smem();          // the updated state is visible to the bulk store
  __syncthreads();
  if (ok) {
    const float ss = red[0] + red[1] + red[2] + red[3];
    const float on = o * rsqrtf(ss / DV + eps) * norm_w[j];
    const float z = pr[C + hv * DV + j];
    const float gz = gate_sigmoid ? sigm(z) : silu(z);
    out[(int64_t)b * (nv * DV) + hv * DV + j] = __float2half_rn(on * gz);
  }
  const int m = n_commit ? n_commit[b] : 1;
  if (j == 0 && ok && m >= 1) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(S), "r"(sS), "r"(DK * DV * 2)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
}

void gdn_step(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor ssm,
              torch::Tensor A_log, torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor slots, torch::Tensor out,
              int64_t nk, int64_t nv, int64_t dk, int64_t dv, int64_t n_tok, double eps, int64_t gate_sigmoid,
              c10::optional<torch::Tensor> n_commit, c10::optional<torch::Tensor> err_word, int64_t timeout_ns) {
  CK(dk == 128 && dv == 128);
  const int* ncm = nullptr;
  if (n_commit) {
    CK(n_commit->scalar_type() == torch::kInt32 && n_commit->numel() * n_tok == proj.size(0));
    ncm = n_commit->data_ptr<int32_t>();
  }
  CK(proj.scalar_type() == torch::kFloat && proj.is_contiguous());
  CK(slots.scalar_type() == torch::kInt32);
  const int rows = proj.size(0);
  if (!rows) return;
  const int B = rows / n_tok;
  const int C = 2 * nk * dk + nv * dv;
  const int kc = conv_w.size(1);
  CK(kc >= 2 && kc <= 8);
  auto qkv = torch::empty({rows, C}, proj.options());
  const int64_t nthr = (int64_t)B * C;
  if (!ncm && n_tok >= 16) {             // prefill: every (token, channel) in parallel, then the state
    const int64_t nall = nthr * n_tok;
    gdn_conv_par_kernel<<<(nall + 255) / 256, 256, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1),
                                                                conv_w.data_ptr<float>(), conv_state.data_ptr<float>(),
                                                                slots.data_ptr<int32_t>(), qkv.data_ptr<float>(), C,
                                                                kc, n_tok, B);
    gdn_conv_state_kernel<<<(nthr + 255) / 256, 256, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1),
                                                                  conv_state.data_ptr<float>(),
                                                                  slots.data_ptr<int32_t>(), C, kc, n_tok, B);
  } else {
    gdn_conv_kernel<<<(nthr + 255) / 256, 256, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1),
                                                            conv_w.data_ptr<float>(), conv_state.data_ptr<float>(),
                                                            slots.data_ptr<int32_t>(), qkv.data_ptr<float>(), C, kc,
                                                            n_tok, B, ncm);
  }
  dim3 grid(B, nv);
  // FW_GDN_DECODE1=0: the general kernel for one-token steps too (FN decode: 22.67 vs 23.06 ms per step)
  static const bool decode1 = !(getenv("FW_GDN_DECODE1") && atoi(getenv("FW_GDN_DECODE1")) == 0);
  if (decode1 && n_tok == 1 && ssm.scalar_type() == torch::kBFloat16 && err_word) {
    gdn_decode1_kernel<<<grid, 128, 0, STREAM>>>(
        qkv.data_ptr<float>(), proj.data_ptr<float>(), proj.size(1), (__nv_bfloat16*)ssm.data_ptr(),
        slots.data_ptr<int32_t>(), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), norm_w.data_ptr<float>(),
        (__half*)out.data_ptr(), nk, nv, (float)eps, gate_sigmoid, ncm, err_word->data_ptr<int32_t>(),
        (uint64_t)timeout_ns);
    return;
  }
  if (ssm.scalar_type() == torch::kBFloat16)
    gdn_recur_kernel<__nv_bfloat16><<<grid, 256, 0, STREAM>>>(
        qkv.data_ptr<float>(), proj.data_ptr<float>(), proj.size(1), (__nv_bfloat16*)ssm.data_ptr(),
        slots.data_ptr<int32_t>(), A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), norm_w.data_ptr<float>(),
        (__half*)out.data_ptr(), nk, nv, n_tok, (float)eps, gate_sigmoid, ncm);
  else
    gdn_recur_kernel<float><<<grid, 256, 0, STREAM>>>(
        qkv.data_ptr<float>(), proj.data_ptr<float>(), proj.size(1), ssm.data_ptr<float>(), slots.data_ptr<int32_t>(),
        A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), norm_w.data_ptr<float>(), (__half*)out.data_ptr(), nk,
        nv, n_tok, (float)eps, gate_sigmoid, ncm);
}

// The GDN causal convolution of a prefill step (every token in parallel, then the state), for the chunked
// prefill in k_gdn_chunk.cu. qkv: [rows, C] fp32 output.
void gdn_conv_prefill_impl(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor slots,
                           torch::Tensor qkv, int64_t n_tok) {
  const int rows = proj.size(0);
  const int B = rows / n_tok, C = qkv.size(1), kc = conv_w.size(1);
  CK(kc >= 2 && kc <= 8 && proj.is_contiguous() && qkv.is_contiguous());
  const int64_t nthr = (int64_t)B * C, nall = nthr * n_tok;
  gdn_conv_par_kernel<<<(nall + 255) / 256, 256, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1),
                                                              conv_w.data_ptr<float>(), conv_state.data_ptr<float>(),
                                                              slots.data_ptr<int32_t>(), qkv.data_ptr<float>(), C, kc,
                                                              n_tok, B);
  gdn_conv_state_kernel<<<(nthr + 255) / 256, 256, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1),
                                                                conv_state.data_ptr<float>(), slots.data_ptr<int32_t>(),
                                                                C, kc, n_tok, B);
}

// ============================================================================================ attention
// RMSNorm(1+w) + partial RoPE (neox half split on the first rd dims) of one head vector held by `nthr` threads,
// dims d = tid, tid + nthr, ... ; x in smem.
__device__ void norm_rope_head(float* x, int D, const float* w, float eps, const float* cs_cos, const float* cs_sin,
                               int rd, float* red) {
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) ss += x[d] * x[d];
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / D + eps);
  __syncthreads();
  float tmp[4];
  int n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) {
    const float v = x[d] * r * (1.f + w[d]);
    float o = v;
    if (d < rd) {
      const int h2 = rd / 2;
      const float other = d < h2 ? -(x[d + h2] * r * (1.f + w[d + h2])) : x[d - h2] * r * (1.f + w[d - h2]);
      o = v * cs_cos[d] + other * cs_sin[d];
    }
    tmp[n] = o;
  }
  __syncthreads();
  n = 0;
  for (int d = threadIdx.x; d < D; d += blockDim.x, ++n) x[d] = tmp[n];
  __syncthreads();
}

// One block per (row, head): blockIdx.y < Hq a query head (norm+rope) -> q plus its gate copy, then the KV heads
// (norm+rope) -> k cache with v -> v cache, then the indexer query heads (norm+rope) -> iq. 256 threads, D <= 1024.
// The heads are independent, so each gets its own block (a block per row walked the 16-20 heads of a row in
// series, two block-wide reductions each, and left most SMs idle at decode batch).
template <typename KT>
__global__ void qsa_prep_kernel(const float* proj, int ldp, const float* qn, const float* kn, const float* iqn,
                                const float* rope, int rope_len, KT* kc, KT* vc, const int* block_table, int max_blocks,
                                int bs, const int* slots, const int* positions, float* q_out, float* gate_out,
                                float* iq_out, int Hq, int KV, int D, int iH, int iD, int n_tok, float eps,
                                int rdq) {
  extern __shared__ float xs[];
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int b = row / n_tok;
  const int p = positions[b] + row % n_tok;
  const int s = slots[b];
  const float* P = proj + (int64_t)row * ldp;
  const float* cs_c = rope + (int64_t)p * rdq;
  const float* cs_s = rope + (int64_t)rope_len * rdq + (int64_t)p * rdq;
  int h = blockIdx.y;
  if (h < Hq) {                                   // query head + gate
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      xs[d] = P[h * 2 * D + d];
      gate_out[(int64_t)row * Hq * D + h * D + d] = P[h * 2 * D + D + d];
    }
    __syncthreads();
    norm_rope_head(xs, D, qn, eps, cs_c, cs_s, rdq, red);
    for (int d = threadIdx.x; d < D; d += blockDim.x) q_out[((int64_t)row * Hq + h) * D + d] = xs[d];
    return;
  }
  h -= Hq;
  if (h < KV) {                                   // key head (norm+rope) and value head into the paged caches
    const int blk = block_table[(int64_t)s * max_blocks + p / bs];
    const int64_t coff = ((int64_t)blk * bs + (p % bs)) * KV * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) xs[d] = P[Hq * 2 * D + h * D + d];
    __syncthreads();
    norm_rope_head(xs, D, kn, eps, cs_c, cs_s, rdq, red);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      stf(&kc[coff + h * D + d], xs[d]);
      stf(&vc[coff + h * D + d], P[Hq * 2 * D + KV * D + h * D + d]);
    }
    return;
  }
  h -= KV;                                        // indexer query head
  const int ib = Hq * 2 * D + 2 * KV * D;
  for (int d = threadIdx.x; d < iD; d += blockDim.x) xs[d] = P[ib + h * iD + d];
  __syncthreads();
  norm_rope_head(xs, iD, iqn, eps, cs_c, cs_s, rdq, red);
  for (int d = threadIdx.x; d < iD; d += blockDim.x) iq_out[((int64_t)row * iH + h) * iD + d] = xs[d];
}

// One block per sequence: compressed indexer keys of every block that completes within this step, from the ring
// of the previous raw keys plus this step's rows; then the ring is refreshed. Sequential per sequence (no race).
// The ring holds RL >= r raw keys indexed by position mod RL; the extra RL - r entries keep the keys of accepted
// positions intact while speculative steps write (and later rewrite) up to RL - r rejected positions ahead.
template <typename CT>
__global__ void qsa_compress_kernel(const float* proj, int ldp, int kr_off, float* ring, CT* comp, int max_comp,
                                    const float* ikn, const float* rope, int rope_len, int rdq, const int* slots,
                                    const int* positions, int r, int RL, int iD, int n_tok, float eps) {
  extern __shared__ float sm[];
  float* old = sm;             // [RL][iD]
  float* xs = sm + RL * iD;    // [iD]
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int s = slots[b];
  const int p0 = positions[b];
  float* rg = ring + (int64_t)s * RL * iD;
  for (int i = threadIdx.x; i < RL * iD; i += blockDim.x) old[i] = rg[i];
  __syncthreads();
  for (int t = 0; t < n_tok; ++t) {
    const int p = p0 + t;
    if ((p + 1) % r) continue;
    const int cb = (p + 1) / r - 1;
    const int st = cb * r;
    for (int d = threadIdx.x; d < iD; d += blockDim.x) {
      float acc = 0.f;
      for (int q = st; q <= p; ++q) {
        const float v = q >= p0 ? proj[((int64_t)b * n_tok + (q - p0)) * ldp + kr_off + d] : old[(q % RL) * iD + d];
        acc += v;
      }
      xs[d] = acc / r;
    }
    __syncthreads();
    norm_rope_head(xs, iD, ikn, eps, rope + (int64_t)st * rdq, rope + (int64_t)rope_len * rdq + (int64_t)st * rdq,
                   rdq, red);
    if (cb < max_comp)
      for (int d = threadIdx.x; d < iD; d += blockDim.x) stf(&comp[((int64_t)s * max_comp + cb) * iD + d], xs[d]);
    __syncthreads();
  }
  // refresh the ring with the last min(RL, n_tok) raw keys of this step
  const int first = max(0, n_tok - RL);
  for (int t = first; t < n_tok; ++t) {
    const int p = p0 + t;
    for (int d = threadIdx.x; d < iD; d += blockDim.x)
      rg[(p % RL) * iD + d] = proj[((int64_t)b * n_tok + t) * ldp + kr_off + d];
  }
}

// Prefill form: one block per (sequence, compressed block completing in this step), the blocks independent; the
// raw-key ring is read as it was at the step start and refreshed by qsa_ring_kernel afterwards. Same sums in the
// same order as qsa_compress_kernel.
template <typename CT>
__global__ void qsa_compress_par_kernel(const float* proj, int ldp, int kr_off, const float* ring, CT* comp,
                                        int max_comp, const float* ikn, const float* rope, int rope_len, int rdq,
                                        const int* slots, const int* positions, int r, int RL, int iD, int n_tok,
                                        float eps) {
  extern __shared__ float xs[];  // [iD]
  __shared__ float red[32];
  const int b = blockIdx.x;
  const int s = slots[b];
  const int p0 = positions[b];
  const int cb = (p0 + r) / r - 1 + blockIdx.y;   // first block whose last position is >= p0, then the next ones
  if ((cb + 1) * r > p0 + n_tok) return;          // completes in a later step
  const int st = cb * r, p = st + r - 1;
  const float* rg = ring + (int64_t)s * RL * iD;
  for (int d = threadIdx.x; d < iD; d += blockDim.x) {
    float acc = 0.f;
    for (int q = st; q <= p; ++q) {
      const float v = q >= p0 ? proj[((int64_t)b * n_tok + (q - p0)) * ldp + kr_off + d] : rg[(q % RL) * iD + d];
      acc += v;
    }
    xs[d] = acc / r;
  }
  __syncthreads();
  norm_rope_head(xs, iD, ikn, eps, rope + (int64_t)st * rdq, rope + (int64_t)rope_len * rdq + (int64_t)st * rdq, rdq,
                 red);
  if (cb < max_comp)
    for (int d = threadIdx.x; d < iD; d += blockDim.x) stf(&comp[((int64_t)s * max_comp + cb) * iD + d], xs[d]);
}

// Refresh the raw-key ring with the last min(RL, n_tok) raw keys of the step (one block per sequence).
__global__ void qsa_ring_kernel(const float* proj, int ldp, int kr_off, float* ring, const int* slots,
                                const int* positions, int RL, int iD, int n_tok) {
  const int b = blockIdx.x;
  float* rg = ring + (int64_t)slots[b] * RL * iD;
  const int p0 = positions[b];
  for (int t = max(0, n_tok - RL); t < n_tok; ++t)
    for (int d = threadIdx.x; d < iD; d += blockDim.x)
      rg[((p0 + t) % RL) * iD + d] = proj[((int64_t)b * n_tok + t) * ldp + kr_off + d];
}

void qsa_prep(torch::Tensor proj, torch::Tensor qn, torch::Tensor kn, torch::Tensor iqn, torch::Tensor ikn,
              torch::Tensor rope, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
              torch::Tensor slots, torch::Tensor positions, torch::Tensor kr_ring, torch::Tensor comp_cache,
              torch::Tensor q, torch::Tensor gate, torch::Tensor iq, int64_t Hq, int64_t KV, int64_t D, int64_t iH,
              int64_t iD, int64_t ratio, int64_t n_tok, double eps) {
  const int rows = proj.size(0);
  if (!rows) return;
  CK(proj.is_contiguous() && proj.scalar_type() == torch::kFloat);
  CK(slots.scalar_type() == torch::kInt32 && positions.scalar_type() == torch::kInt32);
  const int rd = rope.size(2), rope_len = rope.size(1);
  CK(D <= 1024 && iD <= 1024 && rd <= D && rd <= iD);
  const int bs = k_cache.size(1), max_blocks = block_table.size(1);
  dim3 grid(rows, Hq + KV + iH);
  const size_t sm = std::max(D, iD) * sizeof(float);
#define PREP(KT)                                                                                                 \
  qsa_prep_kernel<KT><<<grid, 256, sm, STREAM>>>(                                                                \
      proj.data_ptr<float>(), proj.size(1), qn.data_ptr<float>(), kn.data_ptr<float>(), iqn.data_ptr<float>(),   \
      rope.data_ptr<float>(), rope_len, (KT*)k_cache.data_ptr(), (KT*)v_cache.data_ptr(),                        \
      block_table.data_ptr<int32_t>(), max_blocks, bs, slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), \
      q.data_ptr<float>(), gate.data_ptr<float>(), iq.data_ptr<float>(), Hq, KV, D, iH, iD, n_tok, (float)eps, rd)
  if (k_cache.scalar_type() == torch::kFloat8_e4m3fn) PREP(__nv_fp8_e4m3);
  else if (k_cache.scalar_type() == torch::kBFloat16) PREP(__nv_bfloat16);
  else PREP(float);
#undef PREP
  const int B = rows / n_tok;
  const int kr_off = Hq * 2 * D + 2 * KV * D + iH * iD;
  const int RL = kr_ring.size(1);
  CK(RL >= ratio);
  const size_t smc = (RL * iD + iD) * sizeof(float);
  if (n_tok >= 2 * ratio) {              // prefill: the completing blocks in parallel, then the ring
    dim3 g2(B, n_tok / ratio + 1);
#define COMP_PAR(CT)                                                                                               \
  qsa_compress_par_kernel<CT><<<g2, 128, iD * sizeof(float), STREAM>>>(                                            \
      proj.data_ptr<float>(), proj.size(1), kr_off, kr_ring.data_ptr<float>(), (CT*)comp_cache.data_ptr(),         \
      comp_cache.size(1), ikn.data_ptr<float>(), rope.data_ptr<float>(), rope_len, rd, slots.data_ptr<int32_t>(),  \
      positions.data_ptr<int32_t>(), ratio, RL, iD, n_tok, (float)eps)
    if (comp_cache.scalar_type() == torch::kBFloat16) COMP_PAR(__nv_bfloat16);
    else COMP_PAR(float);
#undef COMP_PAR
    qsa_ring_kernel<<<B, 128, 0, STREAM>>>(proj.data_ptr<float>(), proj.size(1), kr_off, kr_ring.data_ptr<float>(),
                                           slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), RL, iD, n_tok);
    return;
  }
  if (comp_cache.scalar_type() == torch::kBFloat16)
    qsa_compress_kernel<__nv_bfloat16><<<B, 128, smc, STREAM>>>(
        proj.data_ptr<float>(), proj.size(1), kr_off, kr_ring.data_ptr<float>(), (__nv_bfloat16*)comp_cache.data_ptr(),
        comp_cache.size(1), ikn.data_ptr<float>(), rope.data_ptr<float>(), rope_len, rd, slots.data_ptr<int32_t>(),
        positions.data_ptr<int32_t>(), ratio, RL, iD, n_tok, (float)eps);
  else
    qsa_compress_kernel<float><<<B, 128, smc, STREAM>>>(
        proj.data_ptr<float>(), proj.size(1), kr_off, kr_ring.data_ptr<float>(), comp_cache.data_ptr<float>(),
        comp_cache.size(1), ikn.data_ptr<float>(), rope.data_ptr<float>(), rope_len, rd, slots.data_ptr<int32_t>(),
        positions.data_ptr<int32_t>(), ratio, RL, iD, n_tok, (float)eps);
}

// Indexer scores s[row, blk] = sum_h relu(iq[row,h] . comp[blk]) / sqrt(iD) for complete blocks, -inf beyond.
// grid (rows, chunks of 256 blocks); 256 threads, one block key per thread; IH = index heads (accumulators in
// registers), the key row read 8 elements at a time, the query broadcast from shared memory.
template <typename CT, int IH>
__global__ void __launch_bounds__(256) qsa_scores_kernel(const float* iq, const CT* comp, int max_comp,
                                                         const int* slots, const int* positions, float* scores,
                                                         int ld_scores, int iD, int r, int n_tok) {
  extern __shared__ float qs[];  // [IH][iD]
  const int row = blockIdx.x;
  const int b = row / n_tok;
  const int p = positions[b] + row % n_tok;
  const int nc = (p + 1) / r;
  const int blk = blockIdx.y * blockDim.x + threadIdx.x;
  if (blockIdx.y * blockDim.x >= nc) return;
  for (int i = threadIdx.x; i < IH * iD; i += blockDim.x) qs[i] = iq[(int64_t)row * IH * iD + i];
  __syncthreads();
  if (blk >= ld_scores) return;
  float out = -FLT_MAX;
  if (blk < nc && blk < max_comp) {
    const CT* kb = comp + ((int64_t)slots[b] * max_comp + blk) * iD;
    float acc[IH];
#pragma unroll
    for (int h = 0; h < IH; ++h) acc[h] = 0.f;
    for (int d0 = 0; d0 < iD; d0 += 8) {
      float kf[8];
      load8f(kb + d0, kf);
#pragma unroll
      for (int h = 0; h < IH; ++h) {
        const float4 qa = *reinterpret_cast<const float4*>(qs + h * iD + d0);
        const float4 qb = *reinterpret_cast<const float4*>(qs + h * iD + d0 + 4);
        acc[h] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                  qb.z * kf[6] + qb.w * kf[7];
      }
    }
    float sum = 0.f;
#pragma unroll
    for (int h = 0; h < IH; ++h) sum += fmaxf(acc[h], 0.f);
    out = sum * rsqrtf((float)iD);
  }
  scores[(int64_t)row * ld_scores + blk] = out;
}

__device__ __forceinline__ uint32_t f2ord(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exact top-k (k <= n) of one row by 4-pass 8-bit radix select on order-preserving keys; writes the indices of
// the k largest (ties at the threshold broken by lower index) into sel[row, 0..k). 512 threads.
__global__ void topk_rows_kernel(const float* scores, int ld, const int* n_valid_row, int n_fixed, int k, int* sel,
                                 int* sparse_flag, const int* positions, int r, int n_tok) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_kleft, s_cnt_gt, s_eq_taken;
  const int row = blockIdx.x;
  int n;
  if (positions) {
    const int p = positions[row / n_tok] + row % n_tok;
    n = (p + 1) / r;
  } else {
    n = n_valid_row ? n_valid_row[row] : n_fixed;
  }
  n = min(n, ld);
  int* out = sel + (int64_t)row * k;
  if (n <= k) {
    for (int i = threadIdx.x; i < k; i += blockDim.x) out[i] = -1;
    if (sparse_flag && threadIdx.x == 0) sparse_flag[row] = 0;
    return;
  }
  if (sparse_flag && threadIdx.x == 0) sparse_flag[row] = 1;
  const float* x = scores + (int64_t)row * ld;
  uint32_t prefix = 0, mask = 0;
  uint32_t kleft = k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t u = f2ord(x[i]);
      if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= kleft) break;
        acc += hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_kleft = kleft - acc;
    }
    __syncthreads();
    prefix = s_prefix;
    kleft = s_kleft;
    mask |= 255u << shift;
    __syncthreads();
  }
  // prefix = threshold key; take all > threshold, then the first `kleft` equal ones by index
  if (threadIdx.x == 0) {
    s_cnt_gt = 0;
    s_eq_taken = 0;
  }
  __syncthreads();
  const uint32_t thr = prefix;
  const uint32_t n_gt = k - kleft;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t u = f2ord(x[i]);
    if (u > thr) {
      const uint32_t slot = atomicAdd(&s_cnt_gt, 1u);
      out[slot] = i;
    }
  }
  __syncthreads();
  // equal elements in index order (sequential chunks keep the lowest indices)
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const bool eq = i < n && f2ord(x[i]) == thr;
    const unsigned ballot = __ballot_sync(0xffffffffu, eq);
    __shared__ uint32_t wcnt[32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) wcnt[w] = __popc(ballot);
    __syncthreads();
    uint32_t before = 0;
    for (int ww = 0; ww < w; ++ww) before += wcnt[ww];
    const uint32_t rank = s_eq_taken + before + __popc(ballot & ((1u << lane) - 1));
    if (eq && rank < kleft) out[n_gt + rank] = i;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t tot = 0;
      for (int ww = 0; ww < (int)(blockDim.x >> 5); ++ww) tot += wcnt[ww];
      s_eq_taken += tot;
    }
    __syncthreads();
    if (s_eq_taken >= kleft) break;
  }
}

template <int IH>
void launch_scores_ih(const float* iq, const void* comp, bool bf16, int max_comp, const int* slots, const int* pos,
                      float* scores, int ld, int rows, int chunks, int iD, int r, int n_tok, cudaStream_t st) {
  const size_t sm = (size_t)IH * iD * sizeof(float);
  if (bf16)
    qsa_scores_kernel<__nv_bfloat16, IH><<<dim3(rows, chunks), 256, sm, st>>>(
        iq, static_cast<const __nv_bfloat16*>(comp), max_comp, slots, pos, scores, ld, iD, r, n_tok);
  else
    qsa_scores_kernel<float, IH><<<dim3(rows, chunks), 256, sm, st>>>(iq, static_cast<const float*>(comp), max_comp,
                                                                      slots, pos, scores, ld, iD, r, n_tok);
}

// Index-head counts with compiled kernels (FN: 20; tests: 2, 4; Dots3: 64).
bool launch_scores(const float* iq, const void* comp, bool bf16, int max_comp, const int* slots, const int* pos,
                   float* scores, int ld, int rows, int chunks, int iH, int iD, int r, int n_tok, cudaStream_t st) {
  switch (iH) {
    case 1: launch_scores_ih<1>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 2: launch_scores_ih<2>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 4: launch_scores_ih<4>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 8: launch_scores_ih<8>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 16: launch_scores_ih<16>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 20: launch_scores_ih<20>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    case 32: launch_scores_ih<32>(iq, comp, bf16, max_comp, slots, pos, scores, ld, rows, chunks, iD, r, n_tok, st); return true;
    default: return false;
  }
}

void qsa_select(torch::Tensor iq, torch::Tensor comp, torch::Tensor slots, torch::Tensor positions, torch::Tensor sel,
                torch::Tensor sparse, int64_t nblk, int64_t r, int64_t n_tok) {
  const int rows = iq.size(0);
  if (!rows) return;
  const int iH = iq.size(1), iD = iq.size(2);
  CK(iH == 1 || iH == 2 || iH == 4 || iH == 8 || iH == 16 || iH == 20 || iH == 32);
  const int max_comp = comp.size(1);
  const int chunks = (max_comp + 255) / 256;
  auto scores = torch::empty({rows, chunks * 256}, iq.options());
  CK(iD % 8 == 0);
  launch_scores(iq.data_ptr<float>(), comp.data_ptr(), comp.scalar_type() == torch::kBFloat16, max_comp,
                slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), scores.data_ptr<float>(), chunks * 256, rows,
                chunks, iH, iD, r, n_tok, STREAM);
  topk_rows_kernel<<<rows, 512, 0, STREAM>>>(scores.data_ptr<float>(), chunks * 256, nullptr, 0, nblk,
                                             sel.data_ptr<int32_t>(), sparse.data_ptr<int32_t>(),
                                             positions.data_ptr<int32_t>(), r, n_tok);
}

// Generic exact top-k over rows (the sharded-indexer local select and merge use it too).
void topk_rows(torch::Tensor scores, torch::Tensor n_valid, int64_t k, torch::Tensor sel) {
  const int rows = scores.size(0);
  if (!rows) return;
  topk_rows_kernel<<<rows, 512, 0, STREAM>>>(scores.data_ptr<float>(), scores.size(1),
                                             n_valid.numel() ? n_valid.data_ptr<int32_t>() : nullptr, scores.size(1),
                                             k, sel.data_ptr<int32_t>(), nullptr, nullptr, 1, 1);
}

// Split-K sparse GQA decode attention on CUDA cores. Block = (row, kv head, split), 4 warps; the G <= 8 query
// heads of the kv head share every loaded key. Per chunk of 32 keys a warp: each lane scores its own key
// against all G heads (q broadcast from shared memory, the key row read 8 elements at a time), the warp runs
// the online softmax of every head with shuffles, then each lane accumulates P.V for its D/32 dims. The four
// warps' (m, l, acc) are merged in shared memory and written as this split's partial.
template <typename KT, int D>
__global__ void __launch_bounds__(128) attn_split_kernel(const float* q, const KT* kc, const KT* vc,
                                                         const int* block_table, int max_blocks, int bs,
                                                         const int* slots, const int* positions, const int* sel,
                                                         const int* sparse, int nblk, int r, int KV, int G, int n_tok,
                                                         int n_split, float* part_o, float* part_ml) {
  constexpr int NI = D / 32;
  extern __shared__ float sm[];
  float* qs = sm;                       // [8][D]
  float* mrg = qs + 8 * D;              // [4 warps][8 heads][D + 2]
  const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int b = row / n_tok;
  const int p = positions[b] + row % n_tok;
  const int s = slots[b];
  const int Hq = KV * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool is_sparse = sparse[row] != 0;
  const int tail0 = ((p + 1) / r) * r;
  const int n_keys = is_sparse ? nblk * r + (p + 1 - tail0) : p + 1;
  const int per = (n_keys + n_split - 1) / n_split;
  const int k0 = split * per, k1 = min(n_keys, k0 + per);
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x)
    qs[i] = i < G * D ? q[((int64_t)row * Hq + kvh * G) * D + i] : 0.f;
  __syncthreads();
  const float scale = rsqrtf((float)D);
  float m[8], l[8], acc[8][NI];
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    m[h] = -FLT_MAX;
    l[h] = 0.f;
#pragma unroll
    for (int i = 0; i < NI; ++i) acc[h][i] = 0.f;
  }
  for (int c0 = k0 + warp * 32; c0 < k1; c0 += 128) {
    const int mk = c0 + lane;
    const bool valid = mk < k1;
    int64_t off = 0;
    if (valid) {
      int tok = mk;
      if (is_sparse) tok = mk < nblk * r ? sel[(int64_t)row * nblk + mk / r] * r + mk % r : tail0 + (mk - nblk * r);
      const int blk = block_table[(int64_t)s * max_blocks + tok / bs];
      off = (((int64_t)blk * bs + tok % bs) * KV + kvh) * D;
    }
    float sc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) sc[h] = 0.f;
    if (valid) {
#pragma unroll 4
      for (int d0 = 0; d0 < D; d0 += 8) {
        float kf[8];
        load8f(kc + off + d0, kf);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(qs + h * D + d0);
          const float4 qb = *reinterpret_cast<const float4*>(qs + h * D + d0 + 4);
          sc[h] += qa.x * kf[0] + qa.y * kf[1] + qa.z * kf[2] + qa.w * kf[3] + qb.x * kf[4] + qb.y * kf[5] +
                   qb.z * kf[6] + qb.w * kf[7];
        }
      }
    }
    float pr[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      const float sh = valid ? sc[h] * scale : -FLT_MAX;
      const float mn = fmaxf(m[h], warp_max(sh));
      pr[h] = valid ? __expf(sh - mn) : 0.f;
      const float corr = __expf(m[h] - mn);
      l[h] = l[h] * corr + warp_sum(pr[h]);
      m[h] = mn;
#pragma unroll
      for (int i = 0; i < NI; ++i) acc[h][i] *= corr;
    }
    // P.V, 8 keys at a time: the 8 value rows are loaded before any is used, so their latencies overlap
    const int n_here = min(32, k1 - c0);
    for (int k8 = 0; k8 < n_here; k8 += 8) {
      float vf[8][NI];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int kk = k8 + u;
        const int64_t ok = __shfl_sync(0xffffffffu, off, kk & 31);
        if (kk < n_here) {
          if constexpr (NI == 8) {
            load8f(vc + ok + lane * 8, vf[u]);
          } else {
#pragma unroll
            for (int i = 0; i < NI; ++i) vf[u][i] = ldf(&vc[ok + lane * NI + i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < NI; ++i) vf[u][i] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float pk = __shfl_sync(0xffffffffu, pr[h], (k8 + u) & 31);
#pragma unroll
          for (int i = 0; i < NI; ++i) acc[h][i] += pk * vf[u][i];
        }
      }
    }
  }
  // merge the 4 warps
  float* mw = mrg + warp * 8 * (D + 2);
#pragma unroll
  for (int h = 0; h < 8; ++h) {
#pragma unroll
    for (int i = 0; i < NI; ++i) mw[h * (D + 2) + lane * NI + i] = acc[h][i];
    if (lane == 0) {
      mw[h * (D + 2) + D] = m[h];
      mw[h * (D + 2) + D + 1] = l[h];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mrg[(w * 8 + h) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* mh = mrg + (w * 8 + h) * (D + 2);
      const float f = mh[D] > -FLT_MAX ? __expf(mh[D] - M) : 0.f;
      L += mh[D + 1] * f;
      O += mh[d] * f;
    }
    const int64_t base = ((int64_t)row * Hq + kvh * G + h) * n_split + split;
    part_o[base * D + d] = O;
    if (d == 0) {
      part_ml[base * 2] = M;
      part_ml[base * 2 + 1] = L;
    }
  }
}

// Split-K sparse GQA decode attention, version 2 (D = 128 or 256). A warp streams its keys 4 at a time with the
// lanes spread over the head dimension (lane l owns dims [l*NI, l*NI+NI): every key and value row is one
// coalesced 128/256-byte read), the G <= 8 query heads in registers. The 8 heads x 4 keys partial dot products
// are reduced with a butterfly transpose-reduce (31 shuffles leave lane j with the full score of head j/4, key
// j%4); each 4-lane group keeps the online-softmax state of its head, and the probabilities are broadcast back
// for the P.V update of every lane's dims. Same partial-output contract as attn_split_kernel.
template <typename KT, int D>
__global__ void __launch_bounds__(128) attn_split_v2_kernel(const float* q, const KT* kc, const KT* vc,
                                                            const int* block_table, int max_blocks, int bs,
                                                            const int* slots, const int* positions, const int* sel,
                                                            const int* sparse, int nblk, int r, int KV, int G,
                                                            int n_tok, int n_split, float* part_o, float* part_ml) {
  constexpr int NI = D / 32;
  constexpr bool kPipe = std::is_same<KT, __nv_fp8_e4m3>::value && NI == 8;  // raw 8-byte prefetch path
  extern __shared__ float sm[];
  float* mrg = sm;                                            // [4 warps][8 heads][D + 2]
  int* krow = reinterpret_cast<int*>(mrg + 4 * 8 * (D + 2));  // cache row of every key of this split
  const int row = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int b = row / n_tok;
  const int p = positions[b] + row % n_tok;
  const int s = slots[b];
  const int Hq = KV * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool is_sparse = sparse[row] != 0;
  const int tail0 = ((p + 1) / r) * r;
  const int n_keys = is_sparse ? nblk * r + (p + 1 - tail0) : p + 1;
  const int per = (n_keys + n_split - 1) / n_split;
  const int k0 = split * per, k1 = min(n_keys, k0 + per);
  // prologue: resolve every key of the split to its cache row once (index-select + block table lookups)
  for (int mk = k0 + threadIdx.x; mk < k1; mk += blockDim.x) {
    int tok = mk;
    if (is_sparse) tok = mk < nblk * r ? sel[(int64_t)row * nblk + mk / r] * r + mk % r : tail0 + (mk - nblk * r);
    const int blk = block_table[(int64_t)s * max_blocks + tok / bs];
    krow[mk - k0] = blk * bs + tok % bs;
  }
  const float scale = rsqrtf((float)D);
  float qr[8][NI], acc[8][NI];
#pragma unroll
  for (int h = 0; h < 8; ++h)
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      qr[h][i] = h < G ? q[((int64_t)row * Hq + kvh * G + h) * D + lane * NI + i] * scale : 0.f;
      acc[h][i] = 0.f;
    }
  __syncthreads();
  float m_g = -FLT_MAX, l_g = 0.f;      // softmax state of head lane/4, kept by its 4-lane group
  auto offset = [&](int mk) -> int64_t {
    const int kr = krow[min(mk, k1 - 1) - k0];
    return ((int64_t)kr * KV + kvh) * D + lane * NI;
  };
  uint2 kraw[4], vraw[4];
  if constexpr (kPipe) {
    const int c0 = k0 + warp * 4;
    if (c0 < k1) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t o = offset(c0 + u);
        kraw[u] = *reinterpret_cast<const uint2*>(kc + o);
        vraw[u] = *reinterpret_cast<const uint2*>(vc + o);
      }
    }
  }
  // each warp takes every 4th chunk of 4 keys
  for (int c0 = k0 + warp * 4; c0 < k1; c0 += 16) {
    bool ok[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) ok[u] = c0 + u < k1;
    float kf[4][NI], vf[4][NI];
    if constexpr (kPipe) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        fp8x8_to_f32(kraw[u], kf[u]);
        fp8x8_to_f32(vraw[u], vf[u]);
      }
      const int cn = c0 + 16;
      if (cn < k1) {  // the next chunk's rows are in flight during this chunk's math
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t o = offset(cn + u);
          kraw[u] = *reinterpret_cast<const uint2*>(kc + o);
          vraw[u] = *reinterpret_cast<const uint2*>(vc + o);
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t o = offset(c0 + u);
        if constexpr (NI == 8) {
          load8f(kc + o, kf[u]);
          load8f(vc + o, vf[u]);
        } else {
#pragma unroll
          for (int i = 0; i < NI; ++i) {
            kf[u][i] = ldf(&kc[o + i]);
            vf[u][i] = ldf(&vc[o + i]);
          }
        }
      }
    }
    // partial dots: v[h*4 + u]
    float v[32];
#pragma unroll
    for (int h = 0; h < 8; ++h)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float d = 0.f;
#pragma unroll
        for (int i = 0; i < NI; ++i) d = fmaf(qr[h][i], kf[u][i], d);
        v[h * 4 + u] = d;
      }
    // butterfly transpose-reduce: after the round with offset o the lane keeps the half selected by (lane & o)
#pragma unroll
    for (int o = 16, n = 16; o >= 1; o >>= 1, n >>= 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < n; ++i) {
        const float send = upper ? v[i] : v[i + n];
        const float keep = upper ? v[i + n] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    const int hg = lane >> 2, ug = lane & 3;
    const bool valid = ok[ug] && hg < G;
    const float sc = valid ? v[0] : -FLT_MAX;
    float cm = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 1));
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
    const float mn = fmaxf(m_g, cm);
    const float pr = valid ? __expf(sc - mn) : 0.f;
    const float corr = m_g == -FLT_MAX ? 0.f : __expf(m_g - mn);
    float ps = pr + __shfl_xor_sync(0xffffffffu, pr, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_g = l_g * corr + ps;
    m_g = mn;
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      const float ch = __shfl_sync(0xffffffffu, corr, 4 * h);
#pragma unroll
      for (int i = 0; i < NI; ++i) acc[h][i] *= ch;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float pk = __shfl_sync(0xffffffffu, pr, 4 * h + u);
#pragma unroll
        for (int i = 0; i < NI; ++i) acc[h][i] = fmaf(pk, vf[u][i], acc[h][i]);
      }
    }
  }
  float* mw = mrg + warp * 8 * (D + 2);
#pragma unroll
  for (int h = 0; h < 8; ++h) {
#pragma unroll
    for (int i = 0; i < NI; ++i) mw[h * (D + 2) + lane * NI + i] = acc[h][i];
  }
  if ((lane & 3) == 0) {
    mw[(lane >> 2) * (D + 2) + D] = m_g;
    mw[(lane >> 2) * (D + 2) + D + 1] = l_g;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    float M = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, mrg[(w * 8 + h) * (D + 2) + D]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* mh = mrg + (w * 8 + h) * (D + 2);
      const float f = mh[D] > -FLT_MAX ? __expf(mh[D] - M) : 0.f;
      L += mh[D + 1] * f;
      O += mh[d] * f;
    }
    const int64_t base = ((int64_t)row * Hq + kvh * G + h) * n_split + split;
    part_o[base * D + d] = O;
    if (d == 0) {
      part_ml[base * 2] = M;
      part_ml[base * 2 + 1] = L;
    }
  }
}

// Merge the splits of each (row, head) and apply the sigmoid output gate; out fp16 [rows, Hq*D].
__global__ void attn_combine_kernel(const float* part_o, const float* part_ml, const float* gate, __half* out, int Hq,
                                    int D, int n_split) {
  const int row = blockIdx.x, h = blockIdx.y;
  const int64_t base = ((int64_t)row * Hq + h) * n_split;
  float M = -FLT_MAX;
  for (int i = 0; i < n_split; ++i) M = fmaxf(M, part_ml[(base + i) * 2]);
  float L = 0.f;
  for (int i = 0; i < n_split; ++i) {
    const float mi = part_ml[(base + i) * 2];
    if (mi > -FLT_MAX) L += part_ml[(base + i) * 2 + 1] * __expf(mi - M);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int i = 0; i < n_split; ++i) {
      const float mi = part_ml[(base + i) * 2];
      if (mi > -FLT_MAX) o += part_o[(base + i) * D + d] * __expf(mi - M);
    }
    o = L > 0.f ? o / L : 0.f;
    const int64_t oi = (int64_t)row * Hq * D + h * D + d;
    out[oi] = __float2half_rn(o * sigm(gate[oi]));
  }
}

void attn_decode(torch::Tensor q, torch::Tensor gate, torch::Tensor k_cache, torch::Tensor v_cache,
                 torch::Tensor block_table, torch::Tensor slots, torch::Tensor positions, torch::Tensor sel,
                 torch::Tensor sparse, torch::Tensor out, int64_t KV, int64_t r, int64_t n_tok) {
  const int rows = q.size(0), Hq = q.size(1), D = q.size(2);
  if (!rows) return;
  const int G = Hq / KV;
  CK(G <= 8 && Hq % KV == 0);
  CK(D == 64 || D == 128 || D == 256);
  const int nblk = sel.size(1);
  // enough blocks for the machine: rows * KV * split >= ~2 waves
  int n_split = std::max(1, std::min(32, (int)((4 * 148 + rows * KV - 1) / (rows * KV))));
  auto part_o = torch::empty({rows, Hq, n_split, D}, q.options());
  auto part_ml = torch::empty({rows, Hq, n_split, 2}, q.options());
  const size_t sm = (8 * D + 4 * 8 * (D + 2)) * sizeof(float);
  dim3 grid(rows, KV, n_split);
  static const bool attn_v2 = !(getenv("FW_ATTN_V1") && atoi(getenv("FW_ATTN_V1")));
  // most keys one split can see (sparse: nblk*r selected + < r tail; dense only while fewer blocks are complete):
  // every key index is resolved to its cache row in shared memory; fall back to v1 if that would not fit
  const int64_t max_keys = std::min<int64_t>((int64_t)block_table.size(1) * k_cache.size(1), (int64_t)(nblk + 1) * r);
  const int64_t max_per = (max_keys + n_split - 1) / n_split + 1;
  const bool v2_fits = 4 * 8 * (D + 2) * 4 + max_per * 4 <= 100 * 1024;
#define ATT(KT, DD)                                                                                                 \
  {                                                                                                                 \
    auto kern = attn_split_kernel<KT, DD>;                                                                         \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                             \
    kern<<<grid, 128, sm, STREAM>>>(q.data_ptr<float>(), (const KT*)k_cache.data_ptr(), (const KT*)v_cache.data_ptr(), \
                                    block_table.data_ptr<int32_t>(), block_table.size(1), k_cache.size(1),          \
                                    slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), sel.data_ptr<int32_t>(), \
                                    sparse.data_ptr<int32_t>(), nblk, r, KV, G, n_tok, n_split,                    \
                                    part_o.data_ptr<float>(), part_ml.data_ptr<float>());                          \
  }
#define ATT2(KT, DD)                                                                                                \
  {                                                                                                                 \
    auto kern = attn_split_v2_kernel<KT, DD>;                                                                      \
    const size_t sm2 = 4 * 8 * (DD + 2) * sizeof(float) + (size_t)max_per * sizeof(int);                          \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);                          \
    kern<<<grid, 128, sm2, STREAM>>>(q.data_ptr<float>(), (const KT*)k_cache.data_ptr(), (const KT*)v_cache.data_ptr(), \
                                     block_table.data_ptr<int32_t>(), block_table.size(1), k_cache.size(1),         \
                                     slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), sel.data_ptr<int32_t>(), \
                                     sparse.data_ptr<int32_t>(), nblk, r, KV, G, n_tok, n_split,                   \
                                     part_o.data_ptr<float>(), part_ml.data_ptr<float>());                         \
  }
#define ATT_D(KT)            \
  if (D == 64) ATT(KT, 64)   \
  else if (D == 128) { if (attn_v2 && v2_fits) ATT2(KT, 128) else ATT(KT, 128) } \
  else { if (attn_v2 && v2_fits) ATT2(KT, 256) else ATT(KT, 256) }
  if (k_cache.scalar_type() == torch::kFloat8_e4m3fn) {
    ATT_D(__nv_fp8_e4m3)
  } else if (k_cache.scalar_type() == torch::kBFloat16) {
    ATT_D(__nv_bfloat16)
  } else {
    ATT_D(float)
  }
#undef ATT_D
#undef ATT2
#undef ATT
  attn_combine_kernel<<<dim3(rows, Hq), 128, 0, STREAM>>>(part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                                          gate.data_ptr<float>(), (__half*)out.data_ptr(), Hq, D,
                                                          n_split);
}

// ================================================================================================== MoE
// softmax over E logits, top-k (ties -> lower id), renormalize. One block (256 threads) per token.
__global__ void moe_route_kernel(const float* logits, int ld, int32_t* ids, float* w, int E, int k) {
  extern __shared__ float pr[];
  __shared__ float red_v[32];
  __shared__ int red_i[32];
  __shared__ float s_sum;
  const int t = blockIdx.x;
  const float* x = logits + (int64_t)t * ld;
  float mx = -FLT_MAX;
  for (int e = threadIdx.x; e < E; e += blockDim.x) mx = fmaxf(mx, x[e]);
  mx = warp_max(mx);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) red_v[wid] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < nw ? red_v[threadIdx.x] : -FLT_MAX;
    v = warp_max(v);
    if (threadIdx.x == 0) red_v[0] = v;
  }
  __syncthreads();
  mx = red_v[0];
  __syncthreads();
  float sum = 0.f;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    float v = __expf(x[e] - mx);
    if (!(v >= 0.f)) v = 0.f;  // NaN logits must still yield valid expert ids below
    pr[e] = v;
    sum += v;
  }
  __shared__ float sh[32];
  sum = block_sum(sum, sh);
  if (threadIdx.x == 0) s_sum = 0.f;
  __syncthreads();
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float v = pr[e];
      if (v > bv || (v == bv && e < bi)) {
        bv = v;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      red_v[wid] = bv;
      red_i[wid] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float v = red_v[0];
      int i = red_i[0];
      for (int q = 1; q < nw; ++q)
        if (red_v[q] > v || (red_v[q] == v && red_i[q] < i)) {
          v = red_v[q];
          i = red_i[q];
        }
      ids[t * k + j] = i;
      w[t * k + j] = v / sum;
      wsum += v / sum;
      pr[i] = -2.f;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    for (int j = 0; j < k; ++j) w[t * k + j] /= wsum;
  }
}

// One warp per token for E <= 32 * EPL experts: lane l holds the probabilities of experts l, l + 32, ... in
// registers, so the k selection rounds are shuffles only (the block-per-token kernel above spends two block
// barriers per round). Same selection rule: highest probability first, ties to the lower expert id; weights
// renormalized over the selected experts.
template <int EPL>
__global__ void __launch_bounds__(256) moe_route_warp_kernel(const float* logits, int ld, int T, int32_t* ids,
                                                             float* w, int E, int k) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* x = logits + (int64_t)t * ld;
  float p[EPL];
  float mx = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? x[e] : -FLT_MAX;
    mx = fmaxf(mx, p[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    float v = e < E ? __expf(p[i] - mx) : -1.f;
    if (e < E && !(v >= 0.f)) v = 0.f;   // NaN logits must still yield valid expert ids below
    p[i] = v;
    sum += e < E ? v : 0.f;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  float wsum = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (p[i] > bv || (p[i] == bv && e < bi)) {
        bv = p[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i == bi) p[i] = -2.f;
    if (lane == 0) {
      ids[t * k + j] = bi;
      w[t * k + j] = bv / sum;
    }
    wsum += bv / sum;
  }
  if (lane == 0)
    for (int j = 0; j < k; ++j) w[t * k + j] /= wsum;
}

void moe_route(torch::Tensor logits, torch::Tensor ids, torch::Tensor w, int64_t E, int64_t k) {
  const int T = logits.size(0);
  if (!T) return;
  const int ld = logits.size(1);
  // threads per block of the warp-per-token kernel (FW_ROUTE_TPB), FW_ROUTE_OLD=1: the block-per-token kernel
  static const int tpb = getenv("FW_ROUTE_TPB") ? atoi(getenv("FW_ROUTE_TPB")) : 64;
  static const bool old_k = getenv("FW_ROUTE_OLD") && atoi(getenv("FW_ROUTE_OLD"));
  const int grid = (T + tpb / 32 - 1) / (tpb / 32);
  if (old_k)
    moe_route_kernel<<<T, 256, E * sizeof(float), STREAM>>>(logits.data_ptr<float>(), ld, ids.data_ptr<int32_t>(),
                                                            w.data_ptr<float>(), E, k);
  else if (E <= 128)
    moe_route_warp_kernel<4><<<grid, tpb, 0, STREAM>>>(logits.data_ptr<float>(), ld, T, ids.data_ptr<int32_t>(),
                                                       w.data_ptr<float>(), E, k);
  else if (E <= 256)
    moe_route_warp_kernel<8><<<grid, tpb, 0, STREAM>>>(logits.data_ptr<float>(), ld, T, ids.data_ptr<int32_t>(),
                                                       w.data_ptr<float>(), E, k);
  else if (E <= 512)
    moe_route_warp_kernel<16><<<grid, tpb, 0, STREAM>>>(logits.data_ptr<float>(), ld, T, ids.data_ptr<int32_t>(),
                                                        w.data_ptr<float>(), E, k);
  else
    moe_route_kernel<<<T, 256, E * sizeof(float), STREAM>>>(logits.data_ptr<float>(), ld, ids.data_ptr<int32_t>(),
                                                            w.data_ptr<float>(), E, k);
}

// Stable expert sort of the T*k pairs and the tile item list, in one block of 1024 threads.
__global__ void __launch_bounds__(1024) moe_plan_kernel(const int32_t* ids, int P, int32_t* pair_pos, int4* items,
                                                        int32_t* n_items, int E, int n_tile, int max_items) {
  extern __shared__ int smi[];
  int* count = smi;             // [E]
  int* start = count + E;       // [E]
  int* wcnt = start + E;        // [32][E]
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) count[e] = 0;
  __syncthreads();
  // expert ids are clamped into [0, E): a bad id can only misroute a token, never index out of bounds
  for (int i = threadIdx.x; i < P; i += blockDim.x) atomicAdd(&count[min(max(ids[i], 0), E - 1)], 1);
  __syncthreads();
  {
    // thread e owns expert e (E <= 1024): exclusive scans give its first row and its first item
    using Scan = cub::BlockScan<int, 1024>;
    __shared__ typename Scan::TempStorage scan_tmp;
    const int e = threadIdx.x;
    const int c = e < E ? count[e] : 0;
    const int nch = (c + n_tile - 1) / n_tile;
    int row0, item0, total_items;
    Scan(scan_tmp).ExclusiveSum(c, row0);
    __syncthreads();
    Scan(scan_tmp).ExclusiveSum(nch, item0, total_items);
    if (e < E) {
      start[e] = row0;
      for (int q = 0; q < nch; ++q)
        if (item0 + q < max_items) items[item0 + q] = make_int4(e, row0 + q * n_tile, min(n_tile, c - q * n_tile), 0);
    }
    if (threadIdx.x == 0) *n_items = min(total_items, max_items);
  }
  __syncthreads();
  // running per-expert offset in start[]; chunks of 1024 pairs keep the flat order stable
  for (int base = 0; base < P; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int e = i < P ? min(max(ids[i], 0), E - 1) : -1;
    for (int q = threadIdx.x; q < 32 * E; q += blockDim.x) wcnt[q] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(same & ((1u << lane) - 1));
    if (i < P && rank_w == 0) wcnt[w * E + e] = __popc(same);
    __syncthreads();
    if (i < P) {
      int before = 0;
      for (int ww = 0; ww < w; ++ww) before += wcnt[ww * E + e];
      pair_pos[i] = start[e] + before + rank_w;
    }
    __syncthreads();
    for (int q = threadIdx.x; q < E; q += blockDim.x) {
      int tot = 0;
      for (int ww = 0; ww < 32; ++ww) tot += wcnt[ww * E + q];
      start[q] += tot;
    }
    __syncthreads();
  }
}

void moe_plan(torch::Tensor ids, torch::Tensor pair_pos, torch::Tensor items, torch::Tensor n_items, int64_t E,
              int64_t n_tile) {
  const int P = ids.numel();
  const size_t sm = (2 * E + 32 * E) * sizeof(int);
  CK(E <= 1024 && sm <= 200 * 1024);
  auto kern = moe_plan_kernel;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  kern<<<1, 1024, sm, STREAM>>>(ids.data_ptr<int32_t>(), P, pair_pos.data_ptr<int32_t>(),
                                reinterpret_cast<int4*>(items.data_ptr<int32_t>()), n_items.data_ptr<int32_t>(), E,
                                n_tile, items.size(0));
}

__global__ void moe_scatter_kernel(const uint4* x, const int32_t* pair_pos, uint4* xs, int k, int row_vec) {
  const int pair = blockIdx.x;
  const int t = pair / k;
  const int dst = pair_pos[pair];
  for (int i = threadIdx.x; i < row_vec; i += blockDim.x) xs[(int64_t)dst * row_vec + i] = x[(int64_t)t * row_vec + i];
}

void moe_scatter(torch::Tensor x, torch::Tensor pair_pos, torch::Tensor xs) {
  const int P = pair_pos.numel(), k = pair_pos.size(1);
  if (!P) return;
  const int rb = x.size(1) * x.element_size();
  CK(rb % 16 == 0);
  moe_scatter_kernel<<<P, 128, 0, STREAM>>>((const uint4*)x.data_ptr(), pair_pos.data_ptr<int32_t>(),
                                            (uint4*)xs.data_ptr(), k, rb / 16);
}

__global__ void moe_combine_kernel(float* h, const float* ypair, const int32_t* pair_pos, const float* w,
                                   const float* ysh, const float* sg, int ld_sg, const float* inj, int k, int hc,
                                   int H) {
  const int t = blockIdx.x;
  const float g = sigm(sg[(int64_t)t * ld_sg]);
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H; i += blockDim.x * gridDim.y) {
    float y = g * ysh[(int64_t)t * H + i];
    for (int j = 0; j < k; ++j) y += w[t * k + j] * ypair[(int64_t)pair_pos[t * k + j] * H + i];
    for (int s = 0; s < hc; ++s) h[((int64_t)t * hc + s) * H + i] += y * inj[t * hc + s];
  }
}

__global__ void moe_combine4_kernel(float4* h, const float4* ypair, const int32_t* pair_pos, const float* w,
                                    const float4* ysh, const float* sg, int ld_sg, const float* inj, int k, int hc,
                                    int H4) {
  const int t = blockIdx.x;
  const float g = sigm(sg[(int64_t)t * ld_sg]);
  for (int i = blockIdx.y * blockDim.x + threadIdx.x; i < H4; i += blockDim.x * gridDim.y) {
    const float4 sv = ysh[(int64_t)t * H4 + i];
    float4 y = make_float4(g * sv.x, g * sv.y, g * sv.z, g * sv.w);
    for (int j = 0; j < k; ++j) fma4(y, w[t * k + j], ypair[(int64_t)pair_pos[t * k + j] * H4 + i]);
    for (int s = 0; s < hc; ++s) {
      float4& d = h[((int64_t)t * hc + s) * H4 + i];
      float4 a = d;
      fma4(a, inj[t * hc + s], y);
      d = a;
    }
  }
}

void moe_combine(torch::Tensor h, torch::Tensor ypair, torch::Tensor pair_pos, torch::Tensor w, torch::Tensor ysh,
                 torch::Tensor sg, torch::Tensor inj) {
  const int T = pair_pos.size(0), k = pair_pos.size(1);
  if (!T) return;
  const int H = ysh.size(1), hc = inj.size(1);
  const int ld_sg = sg.dim() == 1 ? sg.stride(0) : sg.stride(0);
  if (vec4_ok(H, {h.data_ptr(), ypair.data_ptr(), ysh.data_ptr()})) {
    const int H4 = H / 4;
    moe_combine4_kernel<<<dim3(T, (H4 + 127) / 128), 128, 0, STREAM>>>(
        (float4*)h.data_ptr(), (const float4*)ypair.data_ptr(), pair_pos.data_ptr<int32_t>(), w.data_ptr<float>(),
        (const float4*)ysh.data_ptr(), sg.data_ptr<float>(), ld_sg, inj.data_ptr<float>(), k, hc, H4);
    return;
  }
  moe_combine_kernel<<<dim3(T, (H + 255) / 256), 256, 0, STREAM>>>(h.data_ptr<float>(), ypair.data_ptr<float>(), pair_pos.data_ptr<int32_t>(),
                                            w.data_ptr<float>(), ysh.data_ptr<float>(), sg.data_ptr<float>(), ld_sg,
                                            inj.data_ptr<float>(), k, hc, H);
}

// ============================================================================================= sampling
__global__ void argmax_kernel(const float* x, int V, int32_t* out) {
  __shared__ float bv_s[32];
  __shared__ int bi_s[32];
  const float* r = x + (int64_t)blockIdx.x * V;
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = r[i];
    if (v > bv) {
      bv = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) {
    bv_s[w] = bv;
    bi_s[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int q = 1; q < (int)(blockDim.x >> 5); ++q)
      if (bv_s[q] > bv_s[0] || (bv_s[q] == bv_s[0] && bi_s[q] < bi_s[0])) {
        bv_s[0] = bv_s[q];
        bi_s[0] = bi_s[q];
      }
    out[blockIdx.x] = bi_s[0];
  }
}

void argmax_rows(torch::Tensor logits, torch::Tensor out) {
  const int R = logits.size(0);
  if (!R) return;
  argmax_kernel<<<R, 1024, 0, STREAM>>>(logits.data_ptr<float>(), logits.size(1), out.data_ptr<int32_t>());
}

}  // namespace

void register_fn(pybind11::module& m) {
  m.def("embed_hc", &embed_hc);
  m.def("hc_prenorm", &hc_prenorm);
  m.def("hc_act", &hc_act);
  m.def("hc_mix", &hc_mix);
  m.def("hc_residual", &hc_residual);
  m.def("gdn_step", &gdn_step);
  m.def("qsa_prep", &qsa_prep);
  m.def("qsa_select", &qsa_select);
  m.def("topk_rows", &topk_rows);
  m.def("attn_decode", &attn_decode);
  m.def("moe_route", &moe_route);
  m.def("moe_plan", &moe_plan);
  m.def("moe_scatter", &moe_scatter);
  m.def("moe_combine", &moe_combine);
  m.def("argmax_rows", &argmax_rows);
}

// =============================================================================== allocation-free entry point
// fw_qsa_select_noalloc: the indexer top-k select (block scores + exact radix top-k) for callers that cannot
// allocate device memory, e.g. code running inside a foreign runtime's memory pool or a plugin host that owns
// every allocation and forbids cudaMalloc/cudaFree from its extensions. It has no counterpart in the reference.
//
// It calls no cudaMalloc, cudaFree or allocating library routine. Its scratch (the fp32 score matrix,
// rows x ceil(max_comp/256)*256 floats) lives in the file-scope array below, at most kNoAllocScoreFloats floats
// (2 MiB); every GPU that loads this library holds that array until the process exits. Larger requests are
// rejected with FW_NOALLOC_TOO_BIG before anything is launched.
//
// * Set-up: the first call on a device (with that device current) looks up the array's device address with
//   cudaGetSymbolAddress and caches it per device; make that first call before any stream capture.
// * Sharing: all calls on a device share the one array and it keeps the last call's contents. Nothing in it has
//   to start at zero (every score a call reads is written by that call first). Calls that overlap on the GPU
//   (different streams without ordering) race on the array: serialize them on one stream.
// * Inputs/outputs are the caller's: iq [rows, iH, iD] fp32, comp [S, max_comp, iD] (bf16 if comp_bf16 else
//   fp32), slots [rows / n_tok] int32, positions [rows / n_tok] int32, sel [rows, nblk] int32, sparse [rows] int32.
// Returns 0 on success, FW_NOALLOC_INVALID / FW_NOALLOC_TOO_BIG, or 1000 + cudaError_t.
namespace {
constexpr size_t kNoAllocScoreFloats = (size_t)1 << 19;
static __device__ __align__(256) float g_noalloc_scores[kNoAllocScoreFloats];
constexpr int kNoAllocMaxDevices = 64;
std::atomic<float*> g_noalloc_ptr[kNoAllocMaxDevices];
}  // namespace

enum { FW_NOALLOC_OK = 0, FW_NOALLOC_INVALID = 1, FW_NOALLOC_TOO_BIG = 2 };

extern "C" __attribute__((visibility("default"))) size_t fw_qsa_select_noalloc_max_floats() {
  return kNoAllocScoreFloats;
}

extern "C" __attribute__((visibility("default"))) int fw_qsa_select_noalloc(
    const float* iq, const void* comp, int comp_bf16, const int* slots, const int* positions, int* sel, int* sparse,
    int rows, int iH, int iD, int max_comp, int nblk, int r, int n_tok, cudaStream_t stream) {
  if (rows == 0) return FW_NOALLOC_OK;
  if (rows < 0 || iH <= 0 || iH > 32 || iD <= 0 || max_comp <= 0 || nblk <= 0 || r <= 0 || n_tok <= 0 ||
      rows % n_tok || !iq || !comp || !slots || !positions || !sel || !sparse)
    return FW_NOALLOC_INVALID;
  // the score kernel reads comp 8 elements at a time (16 bytes of bf16, 32 of fp32); iq is read per float
  const uintptr_t comp_align = comp_bf16 ? 16 : 32;
  if (reinterpret_cast<uintptr_t>(comp) % comp_align) return FW_NOALLOC_INVALID;
  const size_t smem = (size_t)iH * iD * sizeof(float);
  if (smem > 48 * 1024) return FW_NOALLOC_INVALID;
  const int chunks = (max_comp + 255) / 256;
  const size_t need = (size_t)rows * chunks * 256;
  if (need > kNoAllocScoreFloats) return FW_NOALLOC_TOO_BIG;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return 1000 + (int)e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return FW_NOALLOC_INVALID;
  float* scores = g_noalloc_ptr[dev].load();
  if (!scores) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scores);
    if (e != cudaSuccess) return 1000 + (int)e;
    scores = static_cast<float*>(p);
    g_noalloc_ptr[dev].store(scores);
  }
  const int ld = chunks * 256;
  if (iD % 8 || !launch_scores(iq, comp, comp_bf16 != 0, max_comp, slots, positions, scores, ld, rows, chunks, iH, iD,
                               r, n_tok, stream))
    return FW_NOALLOC_INVALID;
  topk_rows_kernel<<<rows, 512, 0, stream>>>(scores, ld, nullptr, 0, nblk, sel, sparse, positions, r, n_tok);
  e = cudaGetLastError();
  return e == cudaSuccess ? FW_NOALLOC_OK : 1000 + (int)e;
}

void gdn_conv_prefill(torch::Tensor proj, torch::Tensor conv_w, torch::Tensor conv_state, torch::Tensor slots,
                      torch::Tensor qkv, int64_t n_tok) {
  gdn_conv_prefill_impl(proj, conv_w, conv_state, slots, qkv, n_tok);
}
