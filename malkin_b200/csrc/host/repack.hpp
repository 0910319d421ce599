#pragma once
#include <cstddef>
#include <cstdint>

namespace mkb {

bool repack_supported(uint32_t type);
// Device bytes of rows x units k-units of `type` in the panel layout (rows padded to 16).
size_t repack_bytes(uint32_t type, int64_t rows, int64_t units);
// Repacks k-units [unit0, unit0 + units) of `rows` GGUF rows (row r at src + r * src_stride) into dst.
void repack(uint32_t type, const uint8_t* src, size_t src_stride, int64_t rows, int64_t unit0, int64_t units,
            uint8_t* dst, int n_threads);
// Q8_0 in the tensor-core tile layout (layout.hpp): bytes of rows x blocks (rows padded to 128), and the repack of
// blocks [block0, block0 + blocks) of `rows` GGUF rows. Rows beyond the source are zero (d = 0, q = 0).
size_t repack_tc_bytes(int64_t rows, int64_t blocks);
void repack_tc(const uint8_t* src, size_t src_stride, int64_t rows, int64_t block0, int64_t blocks, uint8_t* dst,
               int n_threads);
// The layout the GEMMs stream a rows x cols weight of `type` in (kLayoutTc / kLayoutPanels of kernels.hpp): for
// Q8_0 the tensor-core tile layout or the mma.sync panels by shape (MALKIN_B200_Q8_LAYOUT=tc|panels forces one);
// panels for the K-quants.
int weight_layout(uint32_t type, int64_t rows, int64_t cols);
// Rows a piece must hold for the next piece to continue the same weight (fused q|k|v, gate|up) in `layout`.
int layout_row_quantum(int layout);
size_t repack_layout_bytes(uint32_t type, int layout, int64_t rows, int64_t units);
void repack_layout(uint32_t type, int layout, const uint8_t* src, size_t src_stride, int64_t rows, int64_t unit0,
                   int64_t units, uint8_t* dst, int n_threads);

}  // namespace mkb
