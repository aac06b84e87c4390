// PLE (per-layer n-gram embedding) kernels of the FN-shaped model's engine path.
//
// Math (the reference's student, flashnext/training/student/student_fn.py:380-459): xor-hashed n-gram row ids
// (n-grams restart after every eos), rows of a shared FP8 table times a scale, key/value projections, per-stream
// gate sign(g) sqrt(|g|) of the key against the RMS-normalized residual stream, gated value, RMSNorm, a causal
// depthwise convolution dilated by the n-gram size, and h += gv + silu(conv).
//
//   ple_ids     : one thread per sequence walks its tokens in order (token history + tokens-since-eos per slot)
//   ple_gather  : FP8 table rows -> fp16 embedding rows (the input of the fused key|value GEMM)
//   ple_mix1    : per token: gate, gv and gvn (written to scratch)
//   ple_mix2    : per token: dilated conv over gvn history (earlier tokens of the same chunk, or the per-slot ring
//                 of >= (kc-1)*d rows indexed by position mod ring length), h += gv + silu(conv)
//   ple_ring    : store the chunk's newest gvn rows into the ring (after every reader of this step)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()
#define CK(x) TORCH_CHECK(x)

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float bsum(float v, float* red) {
  v = wsum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < (int)(blockDim.x >> 5) ? red[l] : 0.f;
  return wsum(t);
}

__global__ void ple_ids_kernel(const int32_t* ids, int B, int n_tok, const int32_t* slots, int64_t* hist, int n,
                               const int64_t* mult, const int64_t* offs, const int64_t* sizes, int hpn, int eos,
                               int64_t* rows) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int64_t* hs = hist + (int64_t)slots[b] * n;  // [n-1 previous tokens, newest first][tokens since eos]
  int64_t since = hs[n - 1];
  const int nh = (n - 1) * hpn;
  for (int j = 0; j < n_tok; ++j) {
    const int64_t t = ids[b * n_tok + j];
    int64_t* out = rows + ((int64_t)b * n_tok + j) * nh;
    for (int ng = 2; ng <= n; ++ng) {
      uint64_t mixed = (uint64_t)t * (uint64_t)mult[0];
      for (int q = 1; q < ng; ++q) {
        const int64_t sq = since >= q ? hs[q - 1] : (int64_t)eos;
        mixed ^= (uint64_t)sq * (uint64_t)mult[q];
      }
      for (int h = (ng - 2) * hpn; h < (ng - 1) * hpn; ++h) {
        const int64_t m = (int64_t)mixed, s = sizes[h];
        out[h] = ((m % s) + s) % s + offs[h];
      }
    }
    for (int q = n - 2; q > 0; --q) hs[q] = hs[q - 1];
    if (n > 1) hs[0] = t;
    since = t == eos ? 0 : since + 1;
  }
  hs[n - 1] = since;
}

// Prefill form: one block per sequence, tokens over the threads. Token j's hashes need the n-1 tokens before it
// (this step's ids, or the history for positions before the step) and the length of the eos-free run that ends
// just before it, which a walk back over at most n-1 tokens gives. Thread 0 rewrites the history after a block
// barrier, once every thread has read it. Same hashes as the sequential kernel above.
__global__ void ple_ids_par_kernel(const int32_t* ids, int n_tok, const int32_t* slots, int64_t* hist, int n,
                                   const int64_t* mult, const int64_t* offs, const int64_t* sizes, int hpn, int eos,
                                   int64_t* rows) {
  const int b = blockIdx.x;
  int64_t* hs = hist + (int64_t)slots[b] * n;  // [n-1 previous tokens, newest first][tokens since eos]
  const int64_t since0 = hs[n - 1];
  const int nh = (n - 1) * hpn;
  const int32_t* tk = ids + (int64_t)b * n_tok;
  for (int j = threadIdx.x; j < n_tok; j += blockDim.x) {
    const int64_t t = tk[j];
    int64_t* out = rows + ((int64_t)b * n_tok + j) * nh;
    // tokens since the last eos as the sequential walk would count them at token j (only values up to n-1 matter)
    int run = 0;
    bool hit = false;
    for (int q = 1; q <= min(j, n - 1); ++q) {
      if (tk[j - q] == eos) {
        hit = true;
        break;
      }
      ++run;
    }
    const int64_t since = hit ? run : (j <= n - 1 ? since0 + j : (int64_t)(n - 1));
    for (int ng = 2; ng <= n; ++ng) {
      uint64_t mixed = (uint64_t)t * (uint64_t)mult[0];
      for (int q = 1; q < ng; ++q) {
        const int64_t prev = q <= j ? (int64_t)tk[j - q] : hs[q - j - 1];
        const int64_t sq = since >= q ? prev : (int64_t)eos;
        mixed ^= (uint64_t)sq * (uint64_t)mult[q];
      }
      for (int h = (ng - 2) * hpn; h < (ng - 1) * hpn; ++h) {
        const int64_t m = (int64_t)mixed, s = sizes[h];
        out[h] = ((m % s) + s) % s + offs[h];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t since = since0;
    for (int j = 0; j < n_tok; ++j) since = tk[j] == eos ? 0 : since + 1;
    for (int q = n - 2; q >= 0; --q) hs[q] = q < n_tok ? (int64_t)tk[n_tok - 1 - q] : hs[q - n_tok];
    hs[n - 1] = since;
  }
}

__global__ void ple_gather_kernel(const __nv_fp8_e4m3* table, int64_t n_rows, int dim, const int64_t* rows, int nh,
                                  float scale, __half* emb) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int64_t r = min(max(rows[(int64_t)t * nh + h], (int64_t)0), n_rows - 1);
  const __nv_fp8_e4m3* src = table + r * dim;
  __half* dst = emb + ((int64_t)t * nh + h) * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) dst[i] = __float2half_rn((float)src[i] * scale);
}

// P row = [key (hc*H) | value (H)]; h row (hc*H); writes gv and gvn rows (hc*H each).
__global__ void __launch_bounds__(256) ple_mix1_kernel(const float* P, const float* h, const float* nk,
                                                       const float* nq, const float* nc, int hc, int H, float eps,
                                                       float* gv, float* gvn) {
  __shared__ float red[8];
  __shared__ float sg[16];
  const int t = blockIdx.x;
  const float* key = P + (int64_t)t * (hc + 1) * H;
  const float* val = key + (int64_t)hc * H;
  const float* hr = h + (int64_t)t * hc * H;
  float* gvr = gv + (int64_t)t * hc * H;
  float* gnr = gvn + (int64_t)t * hc * H;
  for (int c = 0; c < hc; ++c) {
    const float* kc = key + c * H;
    const float* hcp = hr + c * H;
    float sk = 0.f, sq = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      sk += kc[i] * kc[i];
      sq += hcp[i] * hcp[i];
    }
    const float rk = rsqrtf(bsum(sk, red) / H + eps);
    const float rq = rsqrtf(bsum(sq, red) / H + eps);
    float dot = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x)
      dot += (kc[i] * rk * (1.f + nk[c * H + i])) * (hcp[i] * rq * (1.f + nq[c * H + i]));
    float g = bsum(dot, red) * rsqrtf((float)H);
    const float mag = sqrtf(fmaxf(fabsf(g), 1e-6f));
    g = g > 0.f ? mag : g < 0.f ? -mag : 0.f;
    if (threadIdx.x == 0) sg[c] = 1.f / (1.f + __expf(-g));
  }
  __syncthreads();
  for (int c = 0; c < hc; ++c) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float v = sg[c] * val[i];
      gvr[c * H + i] = v;
      ss += v * v;
    }
    const float r = rsqrtf(bsum(ss, red) / H + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) gnr[c * H + i] = gvr[c * H + i] * r * (1.f + nc[c * H + i]);
  }
}

__global__ void ple_mix2_kernel(float* h, const float* gv, const float* gvn, const float* ring, const float* conv,
                                int C, int kc, int d, int R, const int32_t* slots, const int32_t* positions,
                                int n_tok) {
  const int t = blockIdx.x, b = t / n_tok, j = t % n_tok;
  const int p = positions[b] + j;
  const float* rg = ring + (int64_t)slots[b] * R * C;
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < C; c += gridDim.y * blockDim.x) {
    float acc = 0.f;
    for (int k = 0; k < kc; ++k) {
      const int back = (kc - 1 - k) * d;
      const int pp = p - back;
      if (pp < 0) continue;
      float x;
      if (back <= j) x = gvn[((int64_t)t - back) * C + c];
      else x = rg[(int64_t)(pp % R) * C + c];
      acc = fmaf(conv[c * kc + k], x, acc);
    }
    h[(int64_t)t * C + c] += gv[(int64_t)t * C + c] + acc / (1.f + __expf(-acc));
  }
}

__global__ void ple_ring_kernel(float* ring, const float* gvn, int C, int R, const int32_t* slots,
                                const int32_t* positions, int n_tok) {
  const int t = blockIdx.x, b = t / n_tok, j = t % n_tok;
  if (n_tok - 1 - j >= R) return;  // only the newest R rows of the chunk survive
  const int p = positions[b] + j;
  float* dst = ring + ((int64_t)slots[b] * R + p % R) * C;
  for (int c = threadIdx.x; c < C; c += blockDim.x) dst[c] = gvn[(int64_t)t * C + c];
}

void ple_ids(torch::Tensor ids, torch::Tensor slots, int64_t n_tok, torch::Tensor hist, torch::Tensor mult,
             torch::Tensor offs, torch::Tensor sizes, int64_t hpn, int64_t eos, torch::Tensor rows) {
  const int B = slots.size(0), n = hist.size(1);
  CK(ids.scalar_type() == torch::kInt32 && hist.scalar_type() == torch::kInt64 && rows.scalar_type() == torch::kInt64);
  CK(rows.size(0) == B * n_tok && rows.size(1) == (n - 1) * hpn && mult.numel() >= n - 1 + 1);
  if (B && n_tok >= 32)   // prefill: tokens in parallel
    ple_ids_par_kernel<<<B, 256, 0, STREAM>>>(ids.data_ptr<int32_t>(), n_tok, slots.data_ptr<int32_t>(),
                                              hist.data_ptr<int64_t>(), n, mult.data_ptr<int64_t>(),
                                              offs.data_ptr<int64_t>(), sizes.data_ptr<int64_t>(), hpn, eos,
                                              rows.data_ptr<int64_t>());
  else if (B)
    ple_ids_kernel<<<(B + 63) / 64, 64, 0, STREAM>>>(ids.data_ptr<int32_t>(), B, n_tok, slots.data_ptr<int32_t>(),
                                                     hist.data_ptr<int64_t>(), n, mult.data_ptr<int64_t>(),
                                                     offs.data_ptr<int64_t>(), sizes.data_ptr<int64_t>(), hpn,
                                                     eos, rows.data_ptr<int64_t>());
}

void ple_gather(torch::Tensor table, torch::Tensor rows, double scale, torch::Tensor emb) {
  const int T = rows.size(0), nh = rows.size(1), dim = table.size(1);
  CK(table.scalar_type() == at::kFloat8_e4m3fn && emb.scalar_type() == torch::kHalf && emb.size(1) == nh * dim);
  if (T) ple_gather_kernel<<<dim3(T, nh), 128, 0, STREAM>>>((const __nv_fp8_e4m3*)table.data_ptr(), table.size(0),
                                                           dim, rows.data_ptr<int64_t>(), nh, (float)scale,
                                                           (__half*)emb.data_ptr());
}

void ple_mix(torch::Tensor h, torch::Tensor P, torch::Tensor nk, torch::Tensor nq, torch::Tensor nc, torch::Tensor conv,
             torch::Tensor ring, torch::Tensor slots, torch::Tensor positions, int64_t n_tok, int64_t hc, int64_t d,
             double eps) {
  const int T = h.size(0), C = h.size(1), H = C / hc, kc = conv.size(1), R = ring.size(1);
  CK(hc <= 16 && P.size(1) == (hc + 1) * H && R >= (kc - 1) * d && ring.size(2) == C);
  CK(h.is_contiguous() && P.is_contiguous() && conv.is_contiguous() && ring.is_contiguous());
  if (!T) return;
  auto gv = torch::empty({T, C}, h.options());
  auto gvn = torch::empty({T, C}, h.options());
  ple_mix1_kernel<<<T, 256, 0, STREAM>>>(P.data_ptr<float>(), h.data_ptr<float>(), nk.data_ptr<float>(),
                                         nq.data_ptr<float>(), nc.data_ptr<float>(), hc, H, (float)eps,
                                         gv.data_ptr<float>(), gvn.data_ptr<float>());
  ple_mix2_kernel<<<dim3(T, (C + 1023) / 1024), 256, 0, STREAM>>>(
      h.data_ptr<float>(), gv.data_ptr<float>(), gvn.data_ptr<float>(), ring.data_ptr<float>(), conv.data_ptr<float>(),
      C, kc, d, R, slots.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), n_tok);
  ple_ring_kernel<<<T, 256, 0, STREAM>>>(ring.data_ptr<float>(), gvn.data_ptr<float>(), C, R, slots.data_ptr<int32_t>(),
                                         positions.data_ptr<int32_t>(), n_tok);
}

}  // namespace

void register_ple(pybind11::module& m) {
  m.def("ple_ids", &ple_ids);
  m.def("ple_gather", &ple_gather);
  m.def("ple_mix", &ple_mix);
}
