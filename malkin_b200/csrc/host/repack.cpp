// Host repack of GGUF rows into the device panel layout (layout.hpp); the B200 counterpart of malkin's
// pack_weight_into / kern::pack_panel (quant.cpp:218-229, gemm_avx512.cpp:376-544). Rows beyond the source are
// zero-filled (they contribute exactly 0: zero scales), so matrices of any row count pad to whole panels.
#include "repack.hpp"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

#include <cstdlib>
#include <string>

#include "../kernels/kernels.hpp"
#include "gguf.hpp"
#include "layout.hpp"

namespace mkb {

namespace {

// 6-bit value k (0..255) of a Q6_K super-block, stored +32 (quant.cpp:108-128 layout).
inline int q6_at(const uint8_t* s, int k) {
  const int n = k / 128, rem = k % 128, c = rem / 32, l = rem % 32;
  const uint8_t lo = s[64 * n + l + (c & 1) * 32];
  const int nib = c >= 2 ? lo >> 4 : lo & 0xF;
  const int hb = (s[128 + 32 * n + l] >> (2 * c)) & 3;
  return nib | (hb << 4);
}

// Q4_K nibble k (0..255) of a super-block.
inline int q4_at(const uint8_t* s, int k) {
  const int j = k / 32, l = k % 32;
  const uint8_t b = s[16 + 32 * (j / 2) + l];
  return (j & 1) ? b >> 4 : b & 0xF;
}

void pack_chunk(uint32_t type, const uint8_t* const rows[16], size_t unit_off, uint8_t* dst) {
  switch (type) {
    case kQ8_0: {
      std::memset(dst, 0, kChunkQ8_0);
      for (int L = 0; L < 32; ++L) {
        const int g = L / 4, c = L % 4;
        uint8_t* o = dst + 16 * L;
        const int rr[4] = {g, g + 8, g, g + 8};
        const int kk[4] = {4 * c, 4 * c, 16 + 4 * c, 16 + 4 * c};
        for (int w = 0; w < 4; ++w) {
          const uint8_t* s = rows[rr[w]];
          if (!s) continue;
          std::memcpy(o + 4 * w, s + unit_off + 2 + kk[w], 4);
        }
      }
      for (int g = 0; g < 8; ++g) {
        if (rows[g]) std::memcpy(dst + 512 + 4 * g, rows[g] + unit_off, 2);
        if (rows[g + 8]) std::memcpy(dst + 512 + 4 * g + 2, rows[g + 8] + unit_off, 2);
      }
      return;
    }
    case kQ4_K:
    case kQ6_K: {
      const bool q6 = type == kQ6_K;
      std::memset(dst, 0, q6 ? kChunkQ6_K : kChunkQ4_K);
      auto val = [&](int r, int k) -> int {
        const uint8_t* s = rows[r];
        if (!s) return 0;
        return q6 ? q6_at(s + unit_off, k) : q4_at(s + unit_off, k);
      };
      for (int j = 0; j < 8; ++j) {
        for (int L = 0; L < 32; ++L) {
          const int g = L / 4, c = L % 4;
          uint8_t* nib = dst + 256 * j + 8 * L;
          for (int i = 0; i < 4; ++i) {
            const int a0 = val(g, 32 * j + 4 * c + i), a1 = val(g + 8, 32 * j + 4 * c + i);
            const int a2 = val(g, 32 * j + 16 + 4 * c + i), a3 = val(g + 8, 32 * j + 16 + 4 * c + i);
            nib[i] = static_cast<uint8_t>((a0 & 0xF) | ((a2 & 0xF) << 4));
            nib[4 + i] = static_cast<uint8_t>((a1 & 0xF) | ((a3 & 0xF) << 4));
            if (q6) {
              dst[2048 + 128 * j + 4 * L + i] =
                  static_cast<uint8_t>((a0 >> 4) | ((a1 >> 4) << 2) | ((a2 >> 4) << 4) | ((a3 >> 4) << 6));
            }
          }
        }
      }
      for (int g = 0; g < 8; ++g) {
        for (int h = 0; h < 2; ++h) {
          const uint8_t* s = rows[g + 8 * h];
          if (!s) continue;
          if (q6) {
            std::memcpy(dst + 3072 + 32 * g + 16 * h, s + unit_off + 192, 16);
            std::memcpy(dst + 3328 + 4 * g + 2 * h, s + unit_off + 208, 2);
          } else {
            std::memcpy(dst + 2048 + 32 * g + 16 * h, s + unit_off, 16);
          }
        }
      }
      return;
    }
    default:
      throw std::runtime_error("repack: unsupported weight type");
  }
}

}  // namespace

bool repack_supported(uint32_t type) {
  return type == kQ8_0 || type == kQ4_K || type == kQ6_K || float_type(type);
}

size_t repack_bytes(uint32_t type, int64_t rows, int64_t units) {
  const int64_t panels = (rows + kPanelRows - 1) / kPanelRows;
  return static_cast<size_t>(panels) * static_cast<size_t>(units) * chunk_bytes(type);
}

namespace {

// Runs body(i) for i in [0, count) on n_threads threads (0 = all hardware threads).
template <class F>
void parallel_for(int64_t count, int n_threads, F body) {
  std::atomic<int64_t> next{0};
  auto worker = [&] {
    for (int64_t i; (i = next.fetch_add(1)) < count;) body(i);
  };
  int nt = n_threads > 0 ? n_threads : static_cast<int>(std::thread::hardware_concurrency());
  nt = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(nt, count)));
  std::vector<std::thread> pool;
  for (int i = 1; i < nt; ++i) pool.emplace_back(worker);
  worker();
  for (auto& t : pool) t.join();
}

}  // namespace

void repack(uint32_t type, const uint8_t* src, size_t src_stride, int64_t rows, int64_t unit0, int64_t units,
            uint8_t* dst, int n_threads) {
  if (!repack_supported(type)) throw std::runtime_error(std::string("repack: unsupported type ") + type_name(type));
  const size_t cb = chunk_bytes(type);
  const size_t unit_src = type_size(type).bytes;  // GGUF bytes of one k-unit of one row
  const int64_t panels = (rows + kPanelRows - 1) / kPanelRows;
  parallel_for(panels, n_threads, [&](int64_t p) {
    const uint8_t* rp[16];
    for (int r = 0; r < 16; ++r) {
      const int64_t row = p * kPanelRows + r;
      rp[r] = row < rows ? src + static_cast<size_t>(row) * src_stride : nullptr;
    }
    for (int64_t u = 0; u < units; ++u)
      pack_chunk(type, rp, static_cast<size_t>(unit0 + u) * unit_src, dst + (static_cast<size_t>(p) * units + u) * cb);
  });
}

size_t repack_tc_bytes(int64_t rows, int64_t blocks) {
  const int64_t tiles = (rows + kTcRows - 1) / kTcRows;
  return static_cast<size_t>(tiles) * static_cast<size_t>(blocks) * kTcRecord;
}

void repack_tc(const uint8_t* src, size_t src_stride, int64_t rows, int64_t block0, int64_t blocks, uint8_t* dst,
               int n_threads) {
  const size_t bsrc = type_size(kQ8_0).bytes;  // 34: fp16 d, 32 int8
  const int64_t tiles = (rows + kTcRows - 1) / kTcRows;
  parallel_for(tiles, n_threads, [&](int64_t tile) {
    for (int64_t u = 0; u < blocks; ++u) {
      uint8_t* rec = dst + (static_cast<size_t>(tile) * blocks + u) * kTcRecord;
      std::memset(rec, 0, kTcRecord);
      for (int r = 0; r < kTcRows; ++r) {
        const int64_t row = tile * kTcRows + r;
        if (row >= rows) break;
        const uint8_t* s = src + static_cast<size_t>(row) * src_stride + static_cast<size_t>(block0 + u) * bsrc;
        std::memcpy(rec + 4096 + 2 * r, s, 2);
        for (int h = 0; h < 2; ++h) std::memcpy(rec + (r / 8) * 256 + h * 128 + (r % 8) * 16, s + 2 + 16 * h, 16);
      }
    }
  });
}

int weight_layout(uint32_t type, int64_t rows, int64_t cols) {
  if (float_type(type)) return kLayoutRows;
  if (type != kQ8_0) return kLayoutPanels;
  const char* e = std::getenv("MALKIN_B200_Q8_LAYOUT");
  if (e && std::string(e) == "panels") return kLayoutPanels;
  if (e && std::string(e) == "tc") return kLayoutTc;
  // Measured on B200 at 136 tokens (8B shapes), each with its tuned kernel shape: the panel kernels beat the
  // tcgen05 kernel on every matrix (q|k|v 56.7 vs 66.9 us per layer, attention output 48 vs 66, ffn gate+up 108 vs
  // 186, ffn down 101 vs 148): both are bound by the per-block fp32 epilogue, not by the integer dots. Both give
  // identical results; MALKIN_B200_Q8_LAYOUT=tc selects the tcgen05 layout.
  (void)rows;
  (void)cols;
  return kLayoutPanels;
}

int layout_row_quantum(int layout) { return layout == kLayoutTc ? kTcRows : (layout == kLayoutRows ? 1 : kPanelRows); }

size_t repack_layout_bytes(uint32_t type, int layout, int64_t rows, int64_t units) {
  if (layout == kLayoutRows) return static_cast<size_t>(rows) * units * 32 * (type == kF32 ? 4 : 2);
  return layout == kLayoutTc ? repack_tc_bytes(rows, units) : repack_bytes(type, rows, units);
}

void repack_layout(uint32_t type, int layout, const uint8_t* src, size_t src_stride, int64_t rows, int64_t unit0,
                   int64_t units, uint8_t* dst, int n_threads) {
  if (layout == kLayoutRows) {  // the rows' values [32 unit0, 32 (unit0 + units)) as they are
    const size_t elt = type == kF32 ? 4 : 2, nb = static_cast<size_t>(units) * 32 * elt;
    parallel_for(rows, n_threads, [&](int64_t r) {
      std::memcpy(dst + static_cast<size_t>(r) * nb, src + static_cast<size_t>(r) * src_stride + unit0 * 32 * elt, nb);
    });
    return;
  }
  if (layout == kLayoutTc) {
    if (type != kQ8_0) throw std::runtime_error("repack: the tensor-core layout holds Q8_0 only");
    repack_tc(src, src_stride, rows, unit0, units, dst, n_threads);
  } else {
    repack(type, src, src_stride, rows, unit0, units, dst, n_threads);
  }
}

}  // namespace mkb
