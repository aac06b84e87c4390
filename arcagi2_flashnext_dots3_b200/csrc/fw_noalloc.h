// Allocation-free C entry point of the `_C` library (defined in k_fn.cu). It has no counterpart in the reference.
//
// For callers that cannot allocate device memory (a host runtime that owns all allocations, a plugin sandbox
// that forbids cudaMalloc/cudaFree): the caller passes inputs and outputs, the scratch lives in a fixed
// file-scope device array of fw_qsa_select_noalloc_max_floats() floats (2 MiB), held by every GPU that loads the
// library until exit. The first call on a device does a one-time set-up (cudaGetSymbolAddress) and should come
// before any stream capture. Calls share the scratch array: calls that overlap on the GPU race, so order them
// on one stream. Oversize requests return FW_NOALLOC_TOO_BIG (2) without launching; bad arguments return
// FW_NOALLOC_INVALID (1); CUDA errors return 1000 + the cudaError_t.
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

extern "C" {
// Indexer top-k: for each row, the `nblk` highest-scoring complete compressed blocks of its sequence
// (score = sum over heads of relu(iq . comp) / sqrt(iD)); rows with at most nblk complete blocks get sparse = 0
// and sel = -1. iq [rows, iH, iD] fp32; comp [S, max_comp, iD] bf16 (comp_bf16 = 1) or fp32; slots, positions
// [rows / n_tok] int32; sel [rows, nblk] int32; sparse [rows] int32. comp must be 16-byte aligned (bf16) or
// 32-byte aligned (fp32), else FW_NOALLOC_INVALID. The entry point cannot see the cache's slot count S, so the
// caller guarantees 0 <= slots[i] < S (blocks at or beyond max_comp are never read).
int fw_qsa_select_noalloc(const float* iq, const void* comp, int comp_bf16, const int* slots, const int* positions,
                          int* sel, int* sparse, int rows, int iH, int iD, int max_comp, int nblk, int r, int n_tok,
                          cudaStream_t stream);
size_t fw_qsa_select_noalloc_max_floats();
}
