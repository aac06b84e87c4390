// Python bindings of the sm_100a kernels (torch extension `_C`). Every entry point launches on the current
// torch CUDA stream so it can be captured in CUDA graphs, and validates shapes, dtypes and alignment before
// any launch (a bad launch parameter is a host-side exception, never a device fault).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include "wgemm.h"
#include "kernels.h"

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_ALIGN16(t) TORCH_CHECK(((uintptr_t)(t).data_ptr()) % 16 == 0, #t " must be 16-byte aligned")

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Zero-initialised split-K arrival counters, one pool per device; kernels leave every counter at zero.
int* counter_pool(const torch::Device& dev, int64_t need) {
  static std::vector<torch::Tensor> pools(64);
  const int i = dev.index();
  TORCH_CHECK(i >= 0 && i < 64 && need <= (1 << 20), "split-K counter pool too small");
  if (!pools[i].defined()) pools[i] = torch::zeros({1 << 20}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  return pools[i].data_ptr<int32_t>();
}

// y = x @ W^T with W in runtime tile blocks. x: fp16 [rows, K] (token matrix, K-contiguous).
// Returns the number of kernels launched (2 when the split-K partials get their own reduce launch).
int64_t wgemm(torch::Tensor wbase, torch::Tensor exp_off, torch::Tensor exp_fmt, int64_t row_tiles, int64_t kg,
           c10::optional<torch::Tensor> items, c10::optional<torch::Tensor> n_items, int64_t max_items,
           int64_t dense_T, torch::Tensor x, int64_t b_row0, torch::Tensor out, int64_t out_row0,
           int64_t out_cols, int64_t epi, bool accumulate, double alpha, int64_t n_tile, int64_t max_block_bytes,
           torch::Tensor err, int64_t timeout_ns, int64_t k_splits, c10::optional<torch::Tensor> row_dst,
           c10::optional<torch::Tensor> fan_ptrs, int64_t fan_me, int64_t fan_slot,
           c10::optional<torch::Tensor> fan_epoch) {
  CHECK_CUDA(wbase); CHECK_CUDA(x); CHECK_CUDA(out); CHECK_CUDA(err);
  CHECK_CONTIG(x); CHECK_CONTIG(out);
  CHECK_ALIGN16(wbase); CHECK_ALIGN16(x);
  TORCH_CHECK(wbase.scalar_type() == torch::kUInt8, "wbase must be uint8");
  TORCH_CHECK(exp_off.scalar_type() == torch::kInt64 && exp_fmt.scalar_type() == torch::kInt8, "exp_off/fmt dtypes");
  TORCH_CHECK(x.scalar_type() == torch::kHalf && x.dim() == 2, "x must be fp16 [rows, K]");
  TORCH_CHECK(x.size(1) == kg * 128, "x has ", x.size(1), " columns, weights have K=", kg * 128);
  TORCH_CHECK(n_tile == 16 || n_tile == 32 || n_tile == 64 || n_tile == 128, "n_tile must be 16/32/64/128");
  TORCH_CHECK(err.scalar_type() == torch::kInt32, "err must be int32");
  int out_dtype;
  if (out.scalar_type() == torch::kFloat) out_dtype = fw::WGEMM_OUT_F32;
  else if (out.scalar_type() == torch::kBFloat16) out_dtype = fw::WGEMM_OUT_BF16;
  else if (out.scalar_type() == torch::kHalf) out_dtype = fw::WGEMM_OUT_F16;
  else TORCH_CHECK(false, "out must be fp32/bf16/fp16");
  TORCH_CHECK(!accumulate || out_dtype == fw::WGEMM_OUT_F32, "accumulate needs an fp32 output");
  const c10::cuda::CUDAGuard guard(x.device());

  fw::WGemmArgs a{};
  a.wbase = wbase.data_ptr<uint8_t>();
  a.exp_off = exp_off.data_ptr<int64_t>();
  a.exp_fmt = exp_fmt.data_ptr<int8_t>();
  a.row_tiles = (int)row_tiles;
  a.kg = (int)kg;
  a.dense_T = (int)dense_T;
  if (dense_T < 0) {
    TORCH_CHECK(items.has_value() && n_items.has_value(), "grouped mode needs items and n_items");
    TORCH_CHECK(items->scalar_type() == torch::kInt32 && items->is_contiguous(), "items must be int32 [n,4]");
    a.items = reinterpret_cast<const int4*>(items->data_ptr<int32_t>());
    a.n_items = n_items->data_ptr<int32_t>();
    a.max_items = (int)max_items;
  }
  a.n_tile = (int)n_tile;
  a.b_row0 = (int)b_row0;
  a.out = out.data_ptr();
  a.out_ld = (int)out.size(-1);
  a.out_cols = (int)out_cols;
  a.out_row0 = (int)out_row0;
  a.out_dtype = out_dtype;
  a.epi = (int)epi;
  a.accumulate = accumulate ? 1 : 0;
  a.alpha = (float)alpha;
  a.err = err.data_ptr<int32_t>();
  if (row_dst.has_value()) {
    TORCH_CHECK(row_dst->scalar_type() == torch::kInt64 && epi == fw::WGEMM_EPI_STORE && !accumulate,
                "row_dst needs int64 addresses and the plain store epilogue");
    a.row_dst = row_dst->data_ptr<int64_t>();
  }
  a.timeout_ns = (unsigned long long)timeout_ns;
  if (fan_ptrs) {
    TORCH_CHECK(fan_epoch && out_dtype == fw::WGEMM_OUT_F32 && !accumulate && epi == fw::WGEMM_EPI_STORE && !row_dst,
                "fan-out needs the fp32 store epilogue and an epoch tensor");
    TORCH_CHECK(fan_ptrs->is_cuda() && fan_ptrs->scalar_type() == torch::kInt64 && out.numel() <= fan_slot &&
                out.size(-1) == out_cols, "fan-out: device int64 pointers, output of at most one slot, dense rows");
    a.fan_base = reinterpret_cast<const uint64_t*>(fan_ptrs->data_ptr<int64_t>());
    a.fan_n = fan_ptrs->numel();
    a.fan_me = fan_me;
    a.fan_slot = fan_slot;
    a.fan_epoch = fan_epoch->data_ptr<int64_t>();
  }
  static const int dbg = getenv("FW_WGEMM_DBG") ? atoi(getenv("FW_WGEMM_DBG")) : 0;
  a.dbg = dbg;
  static const int sleep_env = getenv("FW_WGEMM_SLEEP_NS") ? atoi(getenv("FW_WGEMM_SLEEP_NS")) : -1;
  a.sleep_ns = sleep_env >= 0 ? (uint32_t)sleep_env : 20000u;

  static const int ab_env = getenv("FW_WGEMM_AB") ? atoi(getenv("FW_WGEMM_AB")) : 0;
  // Pipeline shape: `teams` dequant teams take stages round-robin. Both ring depths must be multiples of the
  // team count (see the kernel's note on parity waits); pick the most teams that leave >= 2 weight stages.
  // CTAs per SM: two smaller pipelines per SM overlap their stage hand-off latencies (FW_WGEMM_CPS overrides)
  static const int cps_env = getenv("FW_WGEMM_CPS") ? atoi(getenv("FW_WGEMM_CPS")) : 0;
  const int cps = cps_env > 0 ? std::min(cps_env, 4) : 1;
  const size_t budget = (232448 / cps) & ~(size_t)1023;
  int teams = 0, ab_stages = 0, w_stages = 0;
  for (int t = fw::kWgemmMaxTeams; t >= 1 && !teams; --t) {
    int P = ab_env > 0 ? ab_env : t;
    if (P % t) continue;
    const size_t fixed = fw::wgemm_smem_bytes((int)n_tile, 1, 0, 0, P) + 8 * 32;
    if (fixed >= budget) continue;
    int S = (int)std::min<size_t>(12, (budget - fixed) / (size_t)max_block_bytes);
    S -= S % t;
    if (S < 2) continue;
    teams = t;
    ab_stages = P;
    w_stages = S;
  }
  TORCH_CHECK(teams > 0, "no pipeline configuration fits in shared memory");
  a.groups_per_stage = 1;
  a.teams = teams;
  a.w_stage_bytes = (int)max_block_bytes;
  a.w_stages = w_stages;
  a.ab_stages = ab_stages;

  // split-K for dense GEMMs that would leave most SMs idle
  int ks = 1;
  if (dense_T >= 0) {
    const int64_t base = ((dense_T + n_tile - 1) / n_tile) * row_tiles;
    if (base < sm_count() * cps)
      ks = (int)std::min<int64_t>({kg, 16, (3 * sm_count() * cps / 2 + base - 1) / base});
    if (k_splits > 0) ks = (int)std::min<int64_t>(k_splits, kg);
  }
  a.k_splits = ks;
  torch::Tensor ws_t;
  // split partials reduced by a second launch over all (tile, 16-token chunk) pairs instead of by the last split
  // of each tile (FW_WGEMM_INKERNEL_REDUCE=1 always keeps the in-kernel reduction)
  static const bool inkernel_reduce = getenv("FW_WGEMM_INKERNEL_REDUCE") && atoi(getenv("FW_WGEMM_INKERNEL_REDUCE"));
  int64_t split_tiles = 0;
  if (ks > 1) {
    split_tiles = ((dense_T + n_tile - 1) / n_tile) * row_tiles;
    ws_t = torch::empty({split_tiles * ks * n_tile * 128}, x.options().dtype(torch::kFloat));
    a.workspace = ws_t.data_ptr<float>();
    // measured: gdn_out (4 splits) 29.5 -> 19.3 us, attn_o 26.0 -> 16.3 us; with 8 splits of a few tiles the extra
    // launch costs more than the in-kernel reduction saves (router 12.9 -> 13.9 us)
    a.ext_reduce = (inkernel_reduce || ks > 4) ? 0 : 1;
    if (!a.ext_reduce) a.counters = counter_pool(x.device(), split_tiles);
  }

  CUtensorMap bmap;
  int rc = fw::make_tmap_2d_f16(&bmap, x.data_ptr(), x.size(0), x.size(1), x.size(1), 64, (uint32_t)n_tile, true);
  TORCH_CHECK(rc == 0, "cuTensorMapEncodeTiled failed: ", rc);
  const int64_t work = (dense_T >= 0 ? (dense_T + n_tile - 1) / n_tile : max_items) * row_tiles * ks;
  if (work <= 0) return 0;
  const int grid = (int)std::min<int64_t>((int64_t)sm_count() * cps, work);
  rc = fw::wgemm_launch(a, bmap, grid, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == 0, "wgemm launch failed: ", cudaGetErrorString((cudaError_t)rc));
  if (a.ext_reduce) {
    rc = fw::wgemm_splitk_reduce(a, (int)split_tiles, at::cuda::getCurrentCUDAStream());
    TORCH_CHECK(rc == 0, "wgemm split-K reduce launch failed: ", cudaGetErrorString((cudaError_t)rc));
    return 2;
  }
  return 1;
}

}  // namespace

void register_kernels(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of arcagi2_flashnext_dots3_b200";
  m.def("wgemm", &wgemm, "weight-dequant tcgen05 GEMM");
  m.def("sm_count", &sm_count);
  register_kernels(m);
}
