// Token sampling for the decode graph: one CTA (1024 threads) per row of logits.
//
//   temperature <= 0            : argmax (ties: lowest id)
//   no top-k / top-p            : exact sampling by Gumbel-max over the whole vocabulary,
//                                 token = argmax_i(x_i / T + g_i), g_i = -log(-log(u_i))
//   top-k and/or top-p          : the top min(k, 1024) logits (radix select, ties by lowest id), sorted, softmax at
//                                 temperature T, cut to the smallest prefix with mass >= p, one inverse-CDF draw
//
// Uniforms u come from a counter-based hash of (seed, step, index): the SplitMix64 output function (Steele, Lea and
// Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) applied to a linear combination of the
// three counters, top 23 bits mapped to (0, 1) (exactly representable in fp32, never 0 or 1). The same hash is implemented on the host (ops/sampling.py), so CPU
// and GPU draw identical samples. The reference samples in vLLM's sampler, and in its vocab-sharded verifier with
// Gumbel-max (dotsnote/engine/arcstats_pkg/arcstats/shard_sample.py:67-119).
//
// Also returns the log-probability of the chosen token under the unmodified model distribution (log_softmax of
// the raw logits), which RL rollouts record as the behaviour policy.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cfloat>
#include <cstdint>

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()
constexpr int kThreads = 1024;
constexpr int kCand = 1024;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ float uniform(uint64_t seed, uint64_t step, uint64_t i) {
  const uint64_t h = mix64(seed * 0x9E3779B97F4A7C15ull + step * 0xD1B54A32D192ED03ull + i * 0x8CB92BA72F3D8DD7ull + 1ull);
  return ((float)(h >> 41) + 0.5f) * (1.0f / 8388608.0f);
}

__device__ __forceinline__ uint32_t f2ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (value, index) max with ties to the lower index, over the block (kThreads threads).
__device__ __forceinline__ void block_argmax(float& v, int& idx, float* sv, int* si) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) {
    sv[w] = v;
    si[w] = idx;
  }
  __syncthreads();
  if (w == 0) {
    v = sv[l];
    idx = si[l];
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (l == 0) {
      sv[0] = v;
      si[0] = idx;
    }
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  __syncthreads();
}

__device__ __forceinline__ float block_sum(float v, float* sv) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sv[w] = v;
  __syncthreads();
  if (w == 0) {
    v = sv[l];
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (l == 0) sv[0] = v;
  }
  __syncthreads();
  v = sv[0];
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const float* logits, int V, int ld, const float* temp,
                                                          const int* top_k, const float* top_p, const int64_t* seed,
                                                          const int64_t* step, int32_t* out, float* out_lp) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ uint32_t hist[256];
  __shared__ float cv[kCand];
  __shared__ int ci[kCand];
  __shared__ uint32_t s_cnt;
  const int row = blockIdx.x;
  const float* x = logits + (int64_t)row * ld;
  // raw max / argmax / log-sum-exp
  float m = -FLT_MAX;
  int am = 1 << 30;
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = x[i];
    if (v > m || (v == m && i < am)) {
      m = v;
      am = i;
    }
  }
  block_argmax(m, am, sv, si);
  float se = 0.f;
  for (int i = threadIdx.x; i < V; i += kThreads) se += __expf(x[i] - m);
  const float lse = m + __logf(block_sum(se, sv));
  const float T = temp[row];
  const int k = top_k[row];
  const float p = top_p[row];
  const uint64_t sd = (uint64_t)seed[row], st = (uint64_t)step[row];
  int tok = am;
  if (T > 0.f && k <= 0 && p >= 1.f) {
    float best = -FLT_MAX;
    int bi = 1 << 30;
    const float inv = 1.f / T;
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float g = x[i] * inv - logf(-logf(uniform(sd, st, (uint64_t)i)));
      if (g > best || (g == best && i < bi)) {
        best = g;
        bi = i;
      }
    }
    block_argmax(best, bi, sv, si);
    tok = bi;
  } else if (T > 0.f) {
    int K = k > 0 ? min(k, kCand) : kCand;
    K = min(K, V);
    // radix select of the K-th largest order key
    uint32_t prefix = 0, mask = 0, kleft = K;
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += kThreads) {
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
        sv[0] = __uint_as_float(prefix | ((uint32_t)d << shift));
        sv[1] = __uint_as_float(kleft - acc);
      }
      __syncthreads();
      prefix = __float_as_uint(sv[0]);
      kleft = __float_as_uint(sv[1]);
      mask |= 255u << shift;
      __syncthreads();
    }
    // candidates: keys above the threshold, then equal keys in index order
    if (threadIdx.x == 0) s_cnt = 0;
    for (int i = threadIdx.x; i < kCand; i += kThreads) {
      cv[i] = -FLT_MAX;
      ci[i] = 1 << 30;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += kThreads) {
      if (f2ord(x[i]) > prefix) {
        const uint32_t s = atomicAdd(&s_cnt, 1u);
        cv[s] = x[i];
        ci[s] = i;
      }
    }
    __syncthreads();
    const uint32_t n_gt = s_cnt;
    // equal keys in index order: per chunk of kThreads ids, warp ballots give each equal key its rank
    __shared__ uint32_t wcnt[32];
    __shared__ uint32_t s_taken;
    if (threadIdx.x == 0) s_taken = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int base = 0; base < V && kleft > 0; base += kThreads) {
      const int i = base + threadIdx.x;
      const bool eq = i < V && f2ord(x[i]) == prefix;
      const unsigned bal = __ballot_sync(0xffffffffu, eq);
      if (lane == 0) wcnt[wid] = __popc(bal);
      __syncthreads();
      uint32_t before = 0, total = 0;
      for (int w = 0; w < kThreads / 32; ++w) {
        if (w < wid) before += wcnt[w];
        total += wcnt[w];
      }
      const uint32_t rank = s_taken + before + __popc(bal & ((1u << lane) - 1u));
      if (eq && rank < kleft) {
        cv[n_gt + rank] = x[i];
        ci[n_gt + rank] = i;
      }
      __syncthreads();
      if (threadIdx.x == 0) s_taken += total;
      __syncthreads();
      if (s_taken >= kleft) break;
    }
    __syncthreads();
    // bitonic sort, descending by value, ascending index on ties
    for (int size = 2; size <= kCand; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const int i = threadIdx.x, j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float a = cv[i], b = cv[j];
          const int ia = ci[i], ib = ci[j];
          const bool a_first = a > b || (a == b && ia < ib);
          if (desc ? !a_first : a_first) {
            cv[i] = b; cv[j] = a;
            ci[i] = ib; ci[j] = ia;
          }
        }
        __syncthreads();
      }
    }
    // softmax at temperature over the K candidates, inclusive prefix sums (sequential per warp of 32, then warps)
    const int i = threadIdx.x;
    float e = i < K ? __expf((cv[i] - cv[0]) / T) : 0.f;
    float incl = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if ((i & 31) >= o) incl += y;
    }
    __shared__ float wtot[32];
    if ((i & 31) == 31) wtot[i >> 5] = incl;
    __syncthreads();
    if (i < 32) {
      float t = wtot[i];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, t, o);
        if (i >= o) t += y;
      }
      wtot[i] = t;  // inclusive over warps
    }
    __syncthreads();
    const float cum = incl + ((i >> 5) ? wtot[(i >> 5) - 1] : 0.f);
    cv[i] = cum;  // reuse: cumulative mass (candidate values are no longer needed)
    __syncthreads();
    const float Z = cv[K - 1];
    // smallest prefix with mass >= p
    if (i == 0) {
      int cut = K - 1;
      if (p < 1.f) {
        for (int j = 0; j < K; ++j)
          if (cv[j] >= p * Z) {
            cut = j;
            break;
          }
      }
      const float u = uniform(sd, st, (uint64_t)V) * cv[cut];
      int pick = cut;
      for (int j = 0; j <= cut; ++j)
        if (cv[j] > u) {
          pick = j;
          break;
        }
      si[0] = ci[pick];
    }
    __syncthreads();
    tok = si[0];
  }
  if (threadIdx.x == 0) {
    out[row] = tok;
    if (out_lp) out_lp[row] = x[tok] - lse;
  }
}

void sample_rows(torch::Tensor logits, torch::Tensor temp, torch::Tensor top_k, torch::Tensor top_p, torch::Tensor seed,
                 torch::Tensor step, torch::Tensor out, c10::optional<torch::Tensor> out_lp) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "logits fp32 [B, V]");
  const int B = logits.size(0);
  TORCH_CHECK(temp.numel() >= B && top_k.numel() >= B && top_p.numel() >= B && seed.numel() >= B && step.numel() >= B,
              "sampling parameter vectors too short");
  TORCH_CHECK(top_k.scalar_type() == torch::kInt32 && seed.scalar_type() == torch::kInt64 &&
              step.scalar_type() == torch::kInt64 && out.scalar_type() == torch::kInt32, "sampling dtypes");
  if (!B) return;
  sample_kernel<<<B, kThreads, 0, STREAM>>>(logits.data_ptr<float>(), logits.size(1), logits.stride(0),
                                            temp.data_ptr<float>(), top_k.data_ptr<int32_t>(), top_p.data_ptr<float>(),
                                            seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(), out.data_ptr<int32_t>(),
                                            out_lp ? out_lp->data_ptr<float>() : nullptr);
}

}  // namespace

void register_sample(pybind11::module& m) { m.def("sample_rows", &sample_rows); }
