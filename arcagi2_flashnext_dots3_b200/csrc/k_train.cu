// Repair-training kernels over the runtime tile-block weight layout (wgemm.h): the trainable quantity is the
// per-(row, 128-column group) scale of every low-bit expert, the integer codes and zero points stay frozen.
//
//   blk_set_scales  : writes fp16(s) into the blocks' scale slots, so the forward expert GEMMs (wgemm, tcgen05)
//                     run on the current trainable scales without re-packing the weights;
//   blk_dequant     : W = s * (q - z) as bf16 [n, R, K] for the selected experts (inputs of the backward GEMMs);
//   blk_scale_grad  : dL/ds[r, g] = sum_c dL/dW[r, 128 g + c] * (q[r, c] - z[r, g]), read straight from the
//                     packed codes (the reference computes the same sum from a dequantized (q - z) tensor,
//                     flashnext/training/student/student_fn.py:129-131 and :178-189).
//
// One CTA of 128 threads per (expert, 128-row tile, 128-column group) block; thread r owns row r of the block.
// Code words are read coalesced (word i of row r at (i * 128 + r) * 4); dense tiles are staged through shared
// memory with an odd word pitch so both the row-per-thread accesses and the coalesced global accesses are free
// of bank conflicts.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "wgemm.h"

namespace {

#define STREAM at::cuda::getCurrentCUDAStream()

struct BlkRef {
  const uint8_t* base;
  int fmt;
};

__device__ __forceinline__ BlkRef block_of(const uint8_t* wbase, const int64_t* exp_off, const int8_t* exp_fmt,
                                           int e, int t, int g, int kg) {
  BlkRef b;
  b.fmt = exp_fmt[e];
  b.base = wbase + exp_off[e] + (int64_t)(t * kg + g) * fw::wgemm_block_bytes(b.fmt);
  return b;
}

// Calls f(col, q) for the 128 columns of row r of an integer-format block (q = raw code).
template <typename F>
__device__ __forceinline__ void for_codes(const BlkRef& b, int r, F&& f) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(b.base);
  const int bits = b.fmt;
  const int ppw = bits == 4 ? 4 : bits == 3 ? 5 : 8;
  const int nw = fw::wgemm_words(bits);
  const uint32_t mask = (1u << bits) - 1u;
  for (int i = 0; i < nw; ++i) {
    const uint32_t v = w[i * 128 + r];
#pragma unroll 8
    for (int k = 0; k < ppw; ++k) {
      const int p = i * ppw + k;
      if (p < 64) {
        f(2 * p, (int)((v >> (bits * k)) & mask));
        f(2 * p + 1, (int)((v >> (16 + bits * k)) & mask));
      }
    }
  }
}

__device__ __forceinline__ int zero_of(const BlkRef& b, int r) {
  return b.base[fw::wgemm_words(b.fmt) * 512 + 256 + r];
}

__global__ void __launch_bounds__(128) blk_set_scales_kernel(uint8_t* wbase, const int64_t* exp_off,
                                                             const int8_t* exp_fmt, const float* s, int E, int R,
                                                             int row_tiles, int kg) {
  const int b = blockIdx.x;
  const int e = b / (row_tiles * kg), rem = b % (row_tiles * kg), t = rem / kg, g = rem % kg;
  if (e >= E) return;
  const int fmt = exp_fmt[e];
  if (fmt > 4) return;
  uint8_t* base = wbase + exp_off[e] + (int64_t)(t * kg + g) * fw::wgemm_block_bytes(fmt);
  const int r = threadIdx.x, row = t * 128 + r;
  const float v = row < R ? s[((int64_t)e * R + row) * kg + g] : 0.f;
  reinterpret_cast<__half*>(base + fw::wgemm_words(fmt) * 512)[r] = __float2half_rn(v);
}

constexpr int kPitchBf16 = 130;  // 65 words per staged row: odd, conflict-free

__global__ void __launch_bounds__(128) blk_dequant_kernel(const uint8_t* wbase, const int64_t* exp_off,
                                                          const int8_t* exp_fmt, const int32_t* sel, int n,
                                                          const float* s, int R, int row_tiles, int kg,
                                                          __nv_bfloat16* out) {
  __shared__ __nv_bfloat16 tile[128 * kPitchBf16];
  const int b = blockIdx.x;
  const int i = b / (row_tiles * kg), rem = b % (row_tiles * kg), t = rem / kg, g = rem % kg;
  if (i >= n) return;
  const int e = sel[i];
  const BlkRef blk = block_of(wbase, exp_off, exp_fmt, e, t, g, kg);
  const int r = threadIdx.x, row = t * 128 + r;
  const int K = kg * 128;
  if (blk.fmt <= 4) {
    const float sc = row < R ? s[((int64_t)i * R + row) * kg + g] : 0.f;
    const float z = (float)zero_of(blk, r);
    __nv_bfloat162* trow = reinterpret_cast<__nv_bfloat162*>(tile + r * kPitchBf16);
    float lo = 0.f;
    for_codes(blk, r, [&](int c, int q) {
      const float w = sc * ((float)q - z);
      if (c & 1) trow[c >> 1] = __floats2bfloat162_rn(lo, w);
      else lo = w;
    });
  }
  __syncthreads();
  // coalesced store: a warp writes 32 consecutive 4-byte words of one row
  const uint32_t* tw = reinterpret_cast<const uint32_t*>(tile);
  for (int idx = threadIdx.x; idx < 128 * 64; idx += 128) {
    const int rr = idx >> 6, cw = idx & 63, grow = t * 128 + rr;
    if (grow < R)
      reinterpret_cast<uint32_t*>(out + ((int64_t)i * R + grow) * K + g * 128)[cw] = tw[rr * (kPitchBf16 / 2) + cw];
  }
}

template <typename T>
__global__ void __launch_bounds__(128) blk_scale_grad_kernel(const uint8_t* wbase, const int64_t* exp_off,
                                                             const int8_t* exp_fmt, const int32_t* sel, int n,
                                                             const T* dW, int R, int row_tiles, int kg, float* ds) {
  extern __shared__ float sm_f[];
  constexpr int kPitch = sizeof(T) == 4 ? 129 : kPitchBf16;  // elements per staged row
  T* tile = reinterpret_cast<T*>(sm_f);
  const int b = blockIdx.x;
  const int i = b / (row_tiles * kg), rem = b % (row_tiles * kg), t = rem / kg, g = rem % kg;
  if (i >= n) return;
  const int K = kg * 128;
  if (sizeof(T) == 4) {
    for (int idx = threadIdx.x; idx < 128 * 128; idx += 128) {
      const int rr = idx >> 7, c = idx & 127, grow = t * 128 + rr;
      tile[rr * kPitch + c] = grow < R ? dW[((int64_t)i * R + grow) * K + g * 128 + c] : T(0);
    }
  } else {
    uint32_t* tw = reinterpret_cast<uint32_t*>(tile);
    for (int idx = threadIdx.x; idx < 128 * 64; idx += 128) {
      const int rr = idx >> 6, cw = idx & 63, grow = t * 128 + rr;
      tw[rr * (kPitch / 2) + cw] =
          grow < R ? reinterpret_cast<const uint32_t*>(dW + ((int64_t)i * R + grow) * K + g * 128)[cw] : 0u;
    }
  }
  __syncthreads();
  const int e = sel[i];
  const BlkRef blk = block_of(wbase, exp_off, exp_fmt, e, t, g, kg);
  const int r = threadIdx.x, row = t * 128 + r;
  if (blk.fmt > 4 || row >= R) return;
  const float z = (float)zero_of(blk, r);
  const T* trow = tile + r * kPitch;
  float acc = 0.f;
  for_codes(blk, r, [&](int c, int q) { acc = fmaf((float)trow[c], (float)q - z, acc); });
  ds[((int64_t)i * R + row) * kg + g] = acc;
}

void check_blocks(const torch::Tensor& wbase, const torch::Tensor& exp_off, const torch::Tensor& exp_fmt) {
  TORCH_CHECK(wbase.is_cuda() && wbase.scalar_type() == torch::kUInt8, "wbase must be CUDA uint8");
  TORCH_CHECK(exp_off.scalar_type() == torch::kInt64 && exp_fmt.scalar_type() == torch::kInt8, "exp_off/fmt dtypes");
}

void blk_set_scales(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, torch::Tensor s,
                    int64_t row_tiles, int64_t kg) {
  check_blocks(wbase, exp_off, exp_fmt);
  TORCH_CHECK(s.is_cuda() && s.scalar_type() == torch::kFloat && s.is_contiguous() && s.dim() == 3, "s fp32 [E,R,KG]");
  const int E = s.size(0), R = s.size(1);
  TORCH_CHECK(s.size(2) == kg && exp_off.size(0) >= E && R <= row_tiles * 128, "scale shape mismatch");
  const c10::cuda::CUDAGuard guard(wbase.device());
  const int grid = E * row_tiles * kg;
  if (grid)
    blk_set_scales_kernel<<<grid, 128, 0, STREAM>>>(wbase.data_ptr<uint8_t>(), exp_off.data_ptr<int64_t>(),
                                                    exp_fmt.data_ptr<int8_t>(), s.data_ptr<float>(), E, R,
                                                    row_tiles, kg);
}

void blk_dequant(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, torch::Tensor sel,
                 torch::Tensor s, int64_t row_tiles, int64_t kg, torch::Tensor out) {
  check_blocks(wbase, exp_off, exp_fmt);
  TORCH_CHECK(sel.is_cuda() && sel.scalar_type() == torch::kInt32, "sel int32");
  TORCH_CHECK(s.scalar_type() == torch::kFloat && s.is_contiguous() && s.dim() == 3, "s fp32 [n,R,KG]");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.dim() == 3, "out bf16 [n,R,K]");
  const int n = sel.size(0), R = s.size(1);
  TORCH_CHECK(s.size(0) == n && s.size(2) == kg && out.size(0) == n && out.size(1) == R && out.size(2) == kg * 128,
              "dequant shapes");
  const c10::cuda::CUDAGuard guard(wbase.device());
  const int grid = n * row_tiles * kg;
  if (grid)
    blk_dequant_kernel<<<grid, 128, 0, STREAM>>>(wbase.data_ptr<uint8_t>(), exp_off.data_ptr<int64_t>(),
                                                 exp_fmt.data_ptr<int8_t>(), sel.data_ptr<int32_t>(), n,
                                                 s.data_ptr<float>(), R, row_tiles, kg,
                                                 reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
}

void blk_scale_grad(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, torch::Tensor sel,
                    torch::Tensor dW, int64_t row_tiles, int64_t kg, torch::Tensor ds) {
  check_blocks(wbase, exp_off, exp_fmt);
  TORCH_CHECK(sel.is_cuda() && sel.scalar_type() == torch::kInt32, "sel int32");
  TORCH_CHECK(dW.is_contiguous() && dW.dim() == 3, "dW [n,R,K] contiguous");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat && ds.is_contiguous() && ds.dim() == 3, "ds fp32 [n,R,KG]");
  const int n = sel.size(0), R = dW.size(1);
  TORCH_CHECK(dW.size(0) == n && dW.size(2) == kg * 128 && ds.size(0) == n && ds.size(1) == R && ds.size(2) == kg,
              "scale-grad shapes");
  const c10::cuda::CUDAGuard guard(wbase.device());
  const int grid = n * row_tiles * kg;
  if (!grid) return;
  if (dW.scalar_type() == torch::kFloat) {
    const int smem = 128 * 129 * 4;
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(blk_scale_grad_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      attr = true;
    }
    blk_scale_grad_kernel<float><<<grid, 128, smem, STREAM>>>(
        wbase.data_ptr<uint8_t>(), exp_off.data_ptr<int64_t>(), exp_fmt.data_ptr<int8_t>(), sel.data_ptr<int32_t>(),
        n, dW.data_ptr<float>(), R, row_tiles, kg, ds.data_ptr<float>());
  } else {
    TORCH_CHECK(dW.scalar_type() == torch::kBFloat16, "dW must be fp32 or bf16");
    blk_scale_grad_kernel<__nv_bfloat16><<<grid, 128, 128 * kPitchBf16 * 2, STREAM>>>(
        wbase.data_ptr<uint8_t>(), exp_off.data_ptr<int64_t>(), exp_fmt.data_ptr<int8_t>(), sel.data_ptr<int32_t>(),
        n, reinterpret_cast<const __nv_bfloat16*>(dW.data_ptr()), R, row_tiles, kg, ds.data_ptr<float>());
  }
}

}  // namespace

void register_train(pybind11::module& m) {
  m.def("blk_set_scales", &blk_set_scales);
  m.def("blk_dequant", &blk_dequant);
  m.def("blk_scale_grad", &blk_scale_grad);
}
