// Host/device interface of the weight-dequant tcgen05 GEMM (wgemm.cu).
//
// Runtime weight layout ("tile blocks"). A weight matrix W [R, K] (y = x W^T) is cut into 128-row tiles and
// 128-column groups; block (tile, group) is contiguous and blocks are stored tile-major:
//   words  uint32 [NW][128 rows]  word i of row r at byte (i*128 + r)*4 (conflict-free smem reads)
//   then, for the integer formats, fp16 scale [128] and uint8 zero [128]; for FP8 one fp32 block scale (16 B).
// Word contents per format (two adjacent columns form a "pair", pairs in column order):
//   fmt 4: NW=16, 4 pairs per word, pair k in bits 4k..4k+3 (even column) and 16+4k.. (odd column)
//   fmt 3: NW=13, 5 pairs per word, pair k in bits 3k.. and 16+3k.. (64 pairs use 12.8 words)
//   fmt 2: NW=8,  8 pairs per word, pair k in bits 2k.. and 16+2k..
//   fmt 8: NW=32, 4 e4m3 bytes per word in column order
//   fmt 16: NW=64, 2 fp16 per word in column order
#pragma once
#include <cstdint>
#include <cstddef>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fw {

enum { WGEMM_EPI_STORE = 0, WGEMM_EPI_SILU_MUL = 1 };
enum { WGEMM_OUT_F32 = 0, WGEMM_OUT_BF16 = 1, WGEMM_OUT_F16 = 2 };

__host__ __device__ inline int wgemm_words(int fmt) {
  return fmt == 4 ? 16 : fmt == 3 ? 13 : fmt == 2 ? 8 : fmt == 8 ? 32 : 64;
}

__host__ __device__ inline uint32_t wgemm_block_bytes(int fmt) {
  const int nw = wgemm_words(fmt);
  return (uint32_t)(nw * 512 + (fmt <= 4 ? 384 : fmt == 8 ? 16 : 0));
}

struct WGemmArgs {
  const uint8_t* wbase;     // packed blocks of all experts
  const int64_t* exp_off;   // [E] byte offset of expert e's first block
  const int8_t* exp_fmt;    // [E] format of expert e
  int row_tiles;            // 128-row tiles per expert
  int kg;                   // K / 128
  const int4* items;        // {expert, token start, token count, 0}; unused when dense_T >= 0
  const int* n_items;       // device-side item count
  int max_items;            // host-side bound on the item count
  int dense_T;              // >= 0: one expert, items = consecutive token tiles of dense_T tokens
  int n_tile;               // N (tokens per MMA tile): 16, 32, 64, 128
  int b_row0;               // first row of the token matrix
  // output
  void* out;
  int out_ld;
  int out_cols;             // valid output columns (weight rows, or features for silu_mul)
  int out_row0;
  int out_dtype;
  int epi;
  int accumulate;           // fp32 store only: out += result
  float alpha;
  const int64_t* row_dst;   // optional: fp32 destination address of every output row (store epilogue only)
  // optional fan-out (tensor-parallel all-reduce): every fp32 output element is also stored at
  // fan_base[p] + (parity * fan_n + fan_me) * fan_slot + row * out_ld + col for p < fan_n, parity = epoch & 1
  const uint64_t* fan_base;
  int fan_n, fan_me;
  int64_t fan_slot;
  const int64_t* fan_epoch;
  // split-K (deterministic): k_splits CTAs share one (item, tile); each writes its fp32 partial
  // [N x 128] to workspace, bumps counters[item * row_tiles + tile]; the last one sums the partials in split
  // order, runs the epilogue and resets the counter to zero (so a captured graph can replay).
  int k_splits;
  float* workspace;
  int* counters;
  int ext_reduce;           // 1: splits only park their partials; wgemm_splitk_reduce sums them (in split order)
                            // and runs the epilogue in a second launch spread over every (tile, 16-token chunk)
  // pipeline
  int groups_per_stage;     // 128-column groups per pipeline stage (always 1 in this version)
  int teams;                // active dequant teams (<= 3); w_stages and ab_stages are multiples of it
  int w_stage_bytes;
  int w_stages;
  int ab_stages;
  int* err;
  unsigned long long timeout_ns;
  // diagnostics (FW_WGEMM_DBG): bit 0 = dequant warps skip the math (stage handshakes only),
  // bit 1 = the MMA issuer skips tcgen05.mma (commits only), bit 2 = no generic->async proxy fence after the
  // dequant stores, bit 3 = no weight bulk copies (the weight stage barrier is armed with 0 bytes).
  // Results are garbage when set.
  int dbg;
  uint32_t sleep_ns;        // suspend-time hint of the off-critical-path barrier waits
};

int make_tmap_2d_f16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                     uint32_t box_cols, uint32_t box_rows, bool swizzle128);
size_t wgemm_smem_bytes(int n_tile, int g2, int w_stage_bytes, int w_stages, int ab_stages);
int wgemm_groups_per_stage(int n_tile);
constexpr int kWgemmMaxTeams = 3;
int wgemm_launch(const WGemmArgs& a, const CUtensorMap& bmap, int grid, cudaStream_t st);
int wgemm_splitk_reduce(const WGemmArgs& a, int tiles, cudaStream_t st);

}  // namespace fw
