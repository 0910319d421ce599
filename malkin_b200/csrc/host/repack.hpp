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

}  // namespace mkb
