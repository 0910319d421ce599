// Device panel layouts of the quantized weights (the B200 counterpart of malkin's ISA panels, gemm_avx512.cpp:17-24)
// and of the quantized activations. Shared by the host repack (repack.cpp) and the kernels.
//
// A panel is 16 weight rows. Within a panel, one k-unit (Q8_0: a 32-value block; Q4_K / Q6_K: a 256-value
// super-block) is one contiguous chunk, laid out so that lane L (g = L / 4, c = L % 4) of a warp reads its
// mma.sync m16n8k32 A fragment {A[g][4c..4c+3], A[g+8][4c..4c+3], A[g][16+4c..], A[g+8][16+4c..]} of every
// 32-value block with one coalesced load. Chunks are [panel][k-unit] in memory, so a warp streams its panel
// front to back. Bytes per chunk equal the GGUF bytes of the same 16 x k-unit weights (34 / 144 / 210 per row).
//
// Q8_0 chunk (544 B):   [0,512) int8 fragments, lane L at 16 L;
//                       [512,544) 8 words, word g = fp16 (d[g], d[g+8]).
// Q4_K chunk (2304 B):  [0,2048) per 32-value block j: 256 B, lane L at 256 j + 8 L: word0 = row g, word1 = row g+8,
//                       byte i low nibble = q[row][32j+4c+i], high nibble = q[row][32j+16+4c+i];
//                       [2048,2304) per g: the 16 GGUF head bytes (d, dmin, 12 packed scale bytes) of row g,
//                       then of row g+8.
// Q6_K chunk (3360 B):  [0,2048) low nibbles as Q4_K (6-bit q stored +32);
//                       [2048,3072) per block j: 128 B, lane L at 2048 + 128 j + 4 L: byte i holds the 2-bit highs of
//                       (A[g][4c+i], A[g+8][4c+i], A[g][16+4c+i], A[g+8][16+4c+i]) in bits (0-1, 2-3, 4-5, 6-7);
//                       [3072,3328) per g: 16 int8 scales of row g, then of row g+8;
//                       [3328,3360) 8 words, word g = fp16 (d[g], d[g+8]).
//
// Quantized activations of n tokens x K (K / 32 blocks), npad = n rounded up to 8 tokens (nt8 = npad / 8 tiles):
//   qx  [block][nt8][256 B]: lane L's 8 bytes = x[8 tile + g][32 block + 4c .. +3], x[..][32 block + 16 + 4c .. +3]
//   dx  [block][npad] float  (BlockQ8::d)
//   dsx [block][npad] float  (d * float(s[0] + s[1]), the Q4_K min term, gemm_avx512.cpp:145)
//   sh  [block][npad] uint32 (int16 s[0] | int16 s[1] << 16, the BlockQ8 half sums)
//
// Tensor-core layout of Q8_0 weights (the A operand of tcgen05.mma kind::i8, K-major, no swizzle). A tile is 128
// rows; per tile and 32-value block one 4352-byte record, records ordered [tile][block]:
//   [0,4096)     int8 values in core matrices of 8 rows x 16 bytes: (row r, value k) at
//                (r / 8) * 256 + (k / 16) * 128 + (r % 8) * 16 + k % 16
//   [4096,4352)  fp16 d of rows 0..127
// Its activations (the B operand) use the same core-matrix order with tokens as rows:
//   qc  [block][npad / 8][2][8][16 B]: (token t, value k) at block * npad * 32 + (t / 8) * 256 + (k / 16) * 128
//       + (t % 8) * 16 + k % 16, npad a multiple of 16.
//   xh  [block][npad / 8][4][8][8 halves]: fp16 of q * d (the dequantized Q8 value), (token t, value k) at half
//       block * npad * 32 + (t / 8) * 256 + (k / 8) * 64 + (t % 8) * 8 + k % 8 (the fp16 GEMM's B operand).
#pragma once
#include <cstddef>
#include <cstdint>

namespace mkb {

constexpr int kPanelRows = 16;
constexpr int kTcRows = 128;
constexpr size_t kTcRecord = 4352;
constexpr size_t kChunkQ8_0 = 544, kChunkQ4_K = 2304, kChunkQ6_K = 3360;

// F32 / F16 / BF16 weights stream as GGUF rows; their k-unit is a 32-value block like Q8_0's.
inline constexpr bool float_type(uint32_t type) { return type == 0 || type == 1 || type == 30; }
inline constexpr int kunit_values(uint32_t type) { return type == 8 || float_type(type) ? 32 : 256; }
inline constexpr size_t chunk_bytes(uint32_t type) {
  return type == 8 ? kChunkQ8_0 : type == 12 ? kChunkQ4_K : type == 14 ? kChunkQ6_K : 0;
}

}  // namespace mkb
