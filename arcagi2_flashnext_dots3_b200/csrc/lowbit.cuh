// Code extraction of the runtime low-bit weight blocks (formats/runtime.py): a block holds 128 rows x 128
// columns of one (expert, row tile, 128-column group); word i of row r sits at byte (i * 128 + r) * 4, so the 32
// threads of a warp that own 32 consecutive rows read 128 contiguous bytes per word index.
//
//   4-bit: word i = columns 8i..8i+7, pair 4i+k in bits 4k (even column) and 16+4k (odd column)
//   3-bit: 5 pairs per word, pair p in bits 3(p%5) (even column) and 16+3(p%5) (odd column) of word p/5
//   2-bit: 8 pairs per word, pair p in bits 2(p%8) and 16+2(p%8) of word p/8
//
// quad<FMT, M>(w) returns the unsigned codes of columns 4M..4M+3 as four bytes in natural column order (M = 0..31),
// the int8 operand layout of both dp4a and the tcgen05 kind::i8 MMA.
#pragma once
#include <cstdint>

namespace fw {
namespace lowbit {

template <int FMT, int M>
__device__ __forceinline__ uint32_t quad(const uint32_t* w) {
  if constexpr (FMT == 4) {
    // word i = columns 8i..8i+7: pairs 4i+k in bits 4k (even col) and 16+4k (odd col)
    const uint32_t x = w[M / 2];
    const uint32_t A = x & 0x0F0F0F0Fu;          // [c0, c4, c1, c5]
    const uint32_t B = (x >> 4) & 0x0F0F0F0Fu;   // [c2, c6, c3, c7]
    return (M & 1) ? __byte_perm(A, B, 0x7531) : __byte_perm(A, B, 0x6420);
  } else {
    // pairs in bits BITS*k (even col) and 16+BITS*k (odd col), PPW pairs per word
    constexpr int BITS = FMT, PPW = FMT == 3 ? 5 : 8;
    constexpr uint32_t MASK = ((1u << BITS) - 1u) * 0x00010001u;
    constexpr int p0 = 2 * M, p1 = 2 * M + 1;
    const uint32_t P0 = (w[p0 / PPW] >> (BITS * (p0 % PPW))) & MASK;   // [c_{2p0}, 0, c_{2p0+1}, 0]
    const uint32_t P1 = (w[p1 / PPW] >> (BITS * (p1 % PPW))) & MASK;
    return __byte_perm(P0, P1, 0x6420);
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
