// Code extraction of the runtime low-bit weight blocks (formats/runtime.py): a block holds 128 rows x 128
// columns of one (expert, row tile, 128-column group); word i of row r sits at byte (i * 128 + r) * 4, so the 32
// threads of a warp that own 32 consecutive rows read 128 contiguous bytes per word index.
//
//   4-bit: word i = columns 8i..8i+7, pair 4i+k in bits 4k (even column) and 16+4k (odd column)
//   3-bit: 5 pairs per word, pair p in bits 3(p%5) (even column) and 16+3(p%5) (odd column) of word p/5
//   2-bit: 8 pairs per word, pair p in bits 2(p%8) and 16+2(p%8) of word p/8
//
// The int8 activations of the grouped GEMV kernels are stored with the columns of every 8-column block in the order
// [0, 4, 1, 5, 2, 6, 3, 7] (gemv_quant), the order in which the 4-bit words yield their codes with one mask each.
// quad<FMT, M>(w) returns the unsigned codes at positions 4M..4M+3 of that order (M = 0..31) as four bytes: the
// int8 operand layout of both dp4a and the tcgen05 kind::i8 MMA.
#pragma once
#include <cstdint>

namespace fw {
namespace lowbit {

template <int FMT, int M>
__device__ __forceinline__ uint32_t quad(const uint32_t* w) {
  if constexpr (FMT == 4) {
    // word i = columns 8i..8i+7: x & 0x0F0F0F0F = [c0, c4, c1, c5], (x >> 4) & 0x0F0F0F0F = [c2, c6, c3, c7]
    const uint32_t x = w[M / 2];
    return (M & 1) ? (x >> 4) & 0x0F0F0F0Fu : x & 0x0F0F0F0Fu;
  } else {
    // pairs in bits BITS*k (even col) and 16+BITS*k (odd col), PPW pairs per word; block b = M / 2 holds pairs
    // 4b..4b+3 = (c0 c1) (c2 c3) (c4 c5) (c6 c7): even M takes pairs 4b and 4b+2, odd M pairs 4b+1 and 4b+3
    constexpr int BITS = FMT, PPW = FMT == 3 ? 5 : 8;
    constexpr uint32_t MASK = ((1u << BITS) - 1u) * 0x00010001u;
    constexpr int pa = 4 * (M / 2) + (M & 1), pb = pa + 2;
    const uint32_t Pa = (w[pa / PPW] >> (BITS * (pa % PPW))) & MASK;   // [c_a, 0, c_a+1, 0]
    const uint32_t Pb = (w[pb / PPW] >> (BITS * (pb % PPW))) & MASK;
    return __byte_perm(Pa, Pb, 0x6240);
  }
}

// 32-bit code words per row of one block. A block is NW * 512 bytes of codes, then 128 fp16 scales (one per row),
// then 128 uint8 zero points: NW * 512 + 384 bytes.
template <int FMT>
struct NWords {
  static constexpr int value = FMT == 4 ? 16 : FMT == 3 ? 13 : 8;
};

}  // namespace lowbit
}  // namespace fw
