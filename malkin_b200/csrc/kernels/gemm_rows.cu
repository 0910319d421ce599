// F32 / F16 / BF16 weights: malkin's row path (quant.cpp:171-191, 330-351) - y[t][r] = vec_dot(w_r, x_t) on the
// float activations, with dot_f32 / dot_f16 / dot_bf16's arithmetic (kernels_avx512.cpp:82-107): 16 lanes, lane l
// accumulates fma(w[16 i + l], x[16 i + l], acc) over i in order from zero (the F16 / BF16 weights converted to f32
// exactly), then _mm512_reduce_add_ps's pairing (lanes l + 8 and l, then l + 4 and l, then (0 + 2, 1 + 3), then
// 0 + 1). The same operations in the same order, so the result is bit-identical to malkin's.
//
// grid (ceil(rows / 32), ceil(n / 8)), block 256: thread (r, t) owns one output; the CTA stages 32 weight rows and 8
// activation rows 128 values at a time in shared memory (rows padded by 4 floats against bank conflicts).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

namespace {

constexpr int kRowsPerCta = 32, kTokPerCta = 8, kChunk = 128;

template <uint32_t T>
__device__ __forceinline__ float weight_at(const uint8_t* w, size_t i) {
  if constexpr (T == 0) {
    return reinterpret_cast<const float*>(w)[i];
  } else if constexpr (T == 1) {
    return __half2float(reinterpret_cast<const __half*>(w)[i]);
  } else {
    return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(w)[i]) << 16);
  }
}

template <uint32_t T>
__global__ void __launch_bounds__(256) k_gemm_rows(const uint8_t* __restrict__ w, int64_t rows, int64_t K,
                                                   const float* __restrict__ x, int64_t ldx, int n,
                                                   float* __restrict__ y, int64_t ldy) {
  __shared__ float ws[kRowsPerCta][kChunk + 4];
  __shared__ float xs[kTokPerCta][kChunk + 4];
  const int tid = threadIdx.x, rr = tid >> 3, tt = tid & 7;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kRowsPerCta;
  const int t0 = blockIdx.y * kTokPerCta;
  float acc[16];
#pragma unroll
  for (int l = 0; l < 16; ++l) acc[l] = 0.0f;
  for (int64_t k0 = 0; k0 < K; k0 += kChunk) {
    const int kc = static_cast<int>(K - k0 < kChunk ? K - k0 : kChunk);  // a multiple of 32
    for (int i = tid; i < kRowsPerCta * kc; i += 256) {
      const int r = i / kc, c = i % kc;
      const int64_t row = r0 + r;
      ws[r][c] = row < rows ? weight_at<T>(w, static_cast<size_t>(row) * K + k0 + c) : 0.0f;
    }
    for (int i = tid; i < kTokPerCta * kc; i += 256) {
      const int t = i / kc, c = i % kc;
      xs[t][c] = t0 + t < n ? x[static_cast<size_t>(t0 + t) * ldx + k0 + c] : 0.0f;
    }
    __syncthreads();
    for (int i = 0; i < kc / 16; ++i) {
#pragma unroll
      for (int l = 0; l < 16; ++l) acc[l] = __fmaf_rn(ws[rr][16 * i + l], xs[tt][16 * i + l], acc[l]);
    }
    __syncthreads();
  }
  float b8[8], c4[4];
#pragma unroll
  for (int l = 0; l < 8; ++l) b8[l] = __fadd_rn(acc[l + 8], acc[l]);
#pragma unroll
  for (int l = 0; l < 4; ++l) c4[l] = __fadd_rn(b8[l + 4], b8[l]);
  const float s = __fadd_rn(__fadd_rn(c4[0], c4[2]), __fadd_rn(c4[1], c4[3]));
  const int64_t row = r0 + rr;
  if (row < rows && t0 + tt < n) y[static_cast<size_t>(t0 + tt) * ldy + row] = s;
}

}  // namespace

void launch_gemm_rows(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, cudaStream_t s) {
  if (n <= 0 || w.rows <= 0) return;
  const dim3 grid(static_cast<unsigned>((w.rows + kRowsPerCta - 1) / kRowsPerCta),
                  static_cast<unsigned>((n + kTokPerCta - 1) / kTokPerCta));
  switch (w.type) {
    case 0:
      k_gemm_rows<0><<<grid, 256, 0, s>>>(w.data, w.rows, w.cols, act.xf, act.ldxf, n, y, ldy);
      break;
    case 1:
      k_gemm_rows<1><<<grid, 256, 0, s>>>(w.data, w.rows, w.cols, act.xf, act.ldxf, n, y, ldy);
      break;
    default:
      k_gemm_rows<30><<<grid, 256, 0, s>>>(w.data, w.rows, w.cols, act.xf, act.ldxf, n, y, ldy);
      break;
  }
}

}  // namespace mkb
