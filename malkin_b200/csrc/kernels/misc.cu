// Token embedding gather + dequantize (Model::run, model.cpp:331-334 -> dequantize_row, quant.cpp:70-169) and
// KV row moves (Model::move_kv, model.cpp:432-440).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

namespace {

__device__ __forceinline__ float ld_h(const uint8_t* p) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// Value i of one GGUF row, as dequantize_row computes it (same float operation order).
__device__ float dequant_at(uint32_t type, const uint8_t* row, int i) {
  switch (type) {
    case 0:
      return reinterpret_cast<const float*>(row)[i];
    case 1:
      return ld_h(row + 2 * i);
    case 30:  // BF16
      return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(row)[i]) << 16);
    case 8: {
      const uint8_t* b = row + (i / 32) * 34;
      return __fmul_rn(ld_h(b), static_cast<float>(static_cast<int8_t>(b[2 + i % 32])));
    }
    case 12: {  // Q4_K
      const uint8_t* b = row + (i / 256) * 144;
      const int k = i % 256, j = k / 32, l = k % 32;
      const uint8_t* s = b + 4;
      int sc, m;
      if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
      } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
      }
      const uint8_t q8 = b[16 + 32 * (j / 2) + l];
      const int q = (j & 1) ? q8 >> 4 : q8 & 0xF;
      // d * sc * q - dmin * m as g++ contracts dequant_q4_k (quant.cpp:77-90): fma(q, d * sc, -(dmin * m))
      return __fmaf_rn(static_cast<float>(q), __fmul_rn(ld_h(b), static_cast<float>(sc)),
                       -__fmul_rn(ld_h(b + 2), static_cast<float>(m)));
    }
    case 14: {  // Q6_K: d * sc * (q - 32)
      const uint8_t* b = row + (i / 256) * 210;
      const int k = i % 256, n = k / 128, r = k % 128, c = r / 32, l = r % 32;
      const uint8_t lo = b[64 * n + l + (c & 1) * 32];
      const int nib = c >= 2 ? lo >> 4 : lo & 0xF;
      const int q = (nib | (((b[128 + 32 * n + l] >> (2 * c)) & 3) << 4)) - 32;
      const int sc = static_cast<int8_t>(b[192 + k / 16]);
      return __fmul_rn(__fmul_rn(ld_h(b + 208), static_cast<float>(sc)), static_cast<float>(q));
    }
    default:
      return 0.0f;
  }
}

__global__ void k_embed(const uint8_t* __restrict__ tab, uint32_t type, size_t row_bytes, int E,
                        const int32_t* __restrict__ ids, float* __restrict__ x) {
  const int t = blockIdx.x;
  const uint8_t* row = tab + static_cast<size_t>(ids[t]) * row_bytes;
  for (int i = threadIdx.x; i < E; i += blockDim.x) x[static_cast<size_t>(t) * E + i] = dequant_at(type, row, i);
}

// One thread per (layer, head, K|V, 16-byte chunk of D); it applies every list's moves in order, so a move that
// reads a row an earlier move of the same list wrote sees the new value, as in malkin's sequential move_kv calls.
__global__ void k_move_kv(KvCacheRef c, const int32_t* __restrict__ from, const int32_t* __restrict__ to,
                          const int32_t* __restrict__ count, int n_lists, int stride) {
  const int chunks = c.D / 16;
  const int64_t total = static_cast<int64_t>(c.n_layer) * c.kvh * 2 * chunks;
  const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (id >= total) return;
  const int ch = static_cast<int>(id % chunks);
  const int64_t plane = id / chunks;  // (layer * kvh + head) * 2 + kv
  const int kv = static_cast<int>(plane & 1);
  const int64_t lh = plane >> 1;
  int8_t* base = (kv ? c.v : c.k) + lh * c.n_rows * c.D;
  float* sc = (kv ? c.vs : c.ks) + lh * c.n_rows;
  for (int l = 0; l < n_lists; ++l) {
    const int cnt = count[l];
    for (int m = 0; m < cnt; ++m) {
      const int64_t f = from[l * stride + m], t = to[l * stride + m];
      if (f == t) continue;
      *reinterpret_cast<uint4*>(base + t * c.D + 16 * ch) = *reinterpret_cast<const uint4*>(base + f * c.D + 16 * ch);
      if (ch == 0) sc[t] = sc[f];
    }
  }
}

}  // namespace

void launch_embed(const uint8_t* tab, uint32_t type, size_t row_bytes, int E, const int32_t* ids, int n, float* x,
                  cudaStream_t s) {
  if (n > 0) k_embed<<<n, 256, 0, s>>>(tab, type, row_bytes, E, ids, x);
}

void launch_move_kv(const KvCacheRef& c, const int32_t* from, const int32_t* to, const int32_t* count, int n_lists,
                    int stride, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(c.n_layer) * c.kvh * 2 * (c.D / 16);
  if (total == 0 || n_lists == 0) return;
  k_move_kv<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(c, from, to, count, n_lists, stride);
}

}  // namespace mkb
