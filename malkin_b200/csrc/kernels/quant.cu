// Activation quantization to Q8 blocks (kern::quantize_row_q8, kernels_avx512.cpp:66-80), fused with the ops that
// produce the activations: RMSNorm (model.cpp:46-49) and SiLU(gate) * up (kernels_avx512.cpp:271-280).
// One warp quantizes one 32-value block: lane i holds value i.
//
// Bit-exactness with malkin's BlockQ8 given the same float input: d = amax / 127 (IEEE division), id = 1 / d
// (0 when d == 0), q = round-half-even(x * id) saturated to int8, s[0] / s[1] = integer sums of the two 16-value
// halves of the unsaturated ints.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <utility>

#include "common.cuh"
#include "kernels.hpp"
#include "quant.cuh"

namespace mkb {

namespace {

__device__ __forceinline__ void store_zero(const ActQ& a, int b, int t, int lane) {
  QBlock z{0, 0.0f, 0, 0};
  store_act(a, b, t, z, lane, 0.0f);
}

// grid (ceil(nb / 8), npad), block 256: warp w quantizes block blockIdx.x * 8 + w of token blockIdx.y.
__global__ void k_quant_rows(const float* __restrict__ x, int64_t ldx, int n, int nb, ActQ a) {
  const int lane = threadIdx.x & 31, b = blockIdx.x * 8 + (threadIdx.x >> 5), t = blockIdx.y;
  if (b >= nb) return;
  if (t >= n) {
    store_zero(a, b, t, lane);
    return;
  }
  const float v = x[static_cast<size_t>(t) * ldx + b * 32 + lane];
  store_act(a, b, t, quant_block32(v, lane), lane, v);
}

// grid (npad), block 256: one token row. y = x * s * w, s = 1 / sqrt(dot(x, x) / K + eps), the dot in malkin's
// 16-lane order (dot16_self over the row in global memory, written back by this block before the barrier).
__global__ void k_rmsnorm_quant(float* __restrict__ x, int64_t ldx, Slices add, const int32_t* __restrict__ rows,
                                const float* __restrict__ w, float eps, int n, int K, ActQ a) {
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = K / 32;
  if (t >= n) {
    for (int b = warp; b < nb; b += 8) store_zero(a, b, t, lane);
    return;
  }
  const int r = rows ? rows[t] : t;
  float* xr = x + static_cast<size_t>(r) * ldx;
  __shared__ float s_sh;
  if (add.n > 0) {
    for (int i = threadIdx.x; i < K; i += blockDim.x)
      xr[i] = __fadd_rn(xr[i], sum_strided16(add.p + static_cast<size_t>(r) * ldx + i, add.n, add.stride));
    __syncthreads();
  }
  if (warp == 0) {
    const float ss = dot16_self(xr, K, lane);
    if (lane == 0) s_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
  }
  __syncthreads();
  const float s = s_sh;
  for (int b = warp; b < nb; b += 8) {
    const int i = b * 32 + lane;
    const float v = __fmul_rn(__fmul_rn(xr[i], s), w[i]);
    store_act(a, b, t, quant_block32(v, lane), lane, v);
  }
}

// The same with one 1024-thread block per token row and the row held in registers (K <= 8192): thread i holds
// values i, i + 1024, ..., so warp w's lanes already hold block w + 32 j for the quantization pass, and every load
// of the row (and of its residual slices) is in flight at once. The row also goes to shared memory, where warp 0
// forms malkin's 16-lane dot (dot16_self): the scale is bit-identical to rmsnorm's (model.cpp:46-49).
constexpr int kNormThreads = 1024, kNormMaxJ = 8;
template <int NS>  // residual slices added first (add.n == NS)
__global__ void __launch_bounds__(kNormThreads) k_rmsnorm_quant_wide(float* __restrict__ x, int64_t ldx, Slices add,
                                                                     const int32_t* __restrict__ rows,
                                                                     const float* __restrict__ w, float eps, int n,
                                                                     int K, ActQ a) {
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nb = K / 32;
  if (t >= n) {
    for (int b = warp; b < nb; b += 32) store_zero(a, b, t, lane);
    return;
  }
  const int r = rows ? rows[t] : t;
  float* xr = x + static_cast<size_t>(r) * ldx;
  float v[kNormMaxJ], wv[kNormMaxJ];
#pragma unroll
  for (int j = 0; j < kNormMaxJ; ++j) {
    const int i = threadIdx.x + kNormThreads * j;
    v[j] = i < K ? xr[i] : 0.0f;
    wv[j] = i < K ? w[i] : 0.0f;
  }
  if constexpr (NS > 0) {
#pragma unroll
    for (int j = 0; j < kNormMaxJ; ++j) {
      const int i = threadIdx.x + kNormThreads * j;
      if (i < K) v[j] = __fadd_rn(v[j], sum_strided<NS>(add.p + static_cast<size_t>(r) * ldx + i, add.stride));
    }
#pragma unroll
    for (int j = 0; j < kNormMaxJ; ++j) {
      const int i = threadIdx.x + kNormThreads * j;
      if (i < K) xr[i] = v[j];
    }
  }
  __shared__ float row[kNormThreads * kNormMaxJ];
  __shared__ float s_sh;
#pragma unroll
  for (int j = 0; j < kNormMaxJ; ++j) {
    const int i = threadIdx.x + kNormThreads * j;
    if (i < K) row[i] = v[j];
  }
  __syncthreads();
  if (warp == 0) {
    const float ss = dot16_self(row, K, lane);
    if (lane == 0) s_sh = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps)));
  }
  __syncthreads();
  const float sc = s_sh;
#pragma unroll
  for (int j = 0; j < kNormMaxJ; ++j) {
    const int b = warp + 32 * j;
    if (b < nb) {
      const float y = __fmul_rn(__fmul_rn(v[j], sc), wv[j]);
      store_act(a, b, t, quant_block32(y, lane), lane, y);
    }
  }
}

__device__ __forceinline__ float sum_slices(const Slices& s, size_t off) { return sum_strided16(s.p + off, s.n, s.stride); }

// grid (ceil(nb / 8), npad), block 256; NS = gu.n slices.
template <int NS>
__global__ void k_silu_quant(Slices gu, int64_t ld, int F, int n, ActQ a) {
  const int lane = threadIdx.x & 31, b = blockIdx.x * 8 + (threadIdx.x >> 5), t = blockIdx.y;
  const int nb = F / 32;
  if (b >= nb) return;
  if (t >= n) {
    store_zero(a, b, t, lane);
    return;
  }
  const size_t row = static_cast<size_t>(t) * ld;
  const float g = sum_strided<NS>(gu.p + row + b * 32 + lane, gu.stride);
  const float u = sum_strided<NS>(gu.p + row + F + b * 32 + lane, gu.stride);
  const float e = exp_malkin(__fsub_rn(0.0f, g));
  const float h = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, e)), u);
  store_act(a, b, t, quant_block32(h, lane), lane, h);
}

// malkin BlockQ8 {float d; int16 s[2]; int8 qs[32]} output. grid (ceil(nb / 8), n), block 256.
__global__ void k_quant_blockq8(const float* __restrict__ x, int64_t K, uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t nb = K / 32, b = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int t = blockIdx.y;
  if (b >= nb) return;
  const QBlock q = quant_block32(x[static_cast<size_t>(t) * K + b * 32 + lane], lane);
  uint8_t* o = out + (static_cast<size_t>(t) * nb + b) * 40;
  o[8 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q.q));
  if (lane == 0) {
    *reinterpret_cast<float*>(o) = q.d;
    reinterpret_cast<int16_t*>(o + 4)[0] = static_cast<int16_t>(q.s0);
    reinterpret_cast<int16_t*>(o + 4)[1] = static_cast<int16_t>(q.s1);
  }
}

// quantize_i8 (quant.cpp:134-140) of one row per warp: d = amax / 127, q = lrintf(x * (1 / d)).
__global__ void k_quant_i8(const float* __restrict__ x, int n, int len, int8_t* __restrict__ q, float* __restrict__ sc) {
  const int lane = threadIdx.x & 31, r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= n) return;
  const float* xr = x + static_cast<size_t>(r) * len;
  float amax = 0.0f;
  for (int i = lane; i < len; i += 32) amax = fmaxf(amax, fabsf(xr[i]));
  amax = warp_max(amax);
  const float d = __fdiv_rn(amax, 127.0f), id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  for (int i = lane; i < len; i += 32) q[static_cast<size_t>(r) * len + i] = static_cast<int8_t>(__float2int_rn(__fmul_rn(xr[i], id)));
  if (lane == 0) sc[r] = d;
}

__global__ void k_sum_slices(Slices src, int64_t ld, int n, int cols, float* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(n) * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const size_t off = static_cast<size_t>(i / cols) * ld + i % cols;
    dst[off] = sum_slices(src, off);
  }
}

__global__ void k_silu_mul(float* __restrict__ g, const float* __restrict__ u, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = g[i];
    const float e = exp_malkin(__fsub_rn(0.0f, x));
    g[i] = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, e)), u[i]);
  }
}

template <int... I>
constexpr auto norm_table(std::integer_sequence<int, I...>) {
  return std::array<void (*)(float*, int64_t, Slices, const int32_t*, const float*, float, int, int, ActQ),
                    sizeof...(I)>{&k_rmsnorm_quant_wide<I>...};
}
template <int... I>
constexpr auto silu_table(std::integer_sequence<int, I...>) {
  return std::array<void (*)(Slices, int64_t, int, int, ActQ), sizeof...(I)>{&k_silu_quant<I + 1>...};
}

}  // namespace

void launch_quant_rows(const float* x, int64_t ldx, int n, int K, const ActQ& act, cudaStream_t s) {
  const int nb = K / 32;
  dim3 grid((nb + 7) / 8, act.nt8 * 8);
  k_quant_rows<<<grid, 256, 0, s>>>(x, ldx, n, nb, act);
}

void launch_rmsnorm_quant(float* x, int64_t ldx, Slices add, const int32_t* rows, const float* w, float eps, int n,
                          int K, const ActQ& act, cudaStream_t s) {
  static constexpr auto fns = norm_table(std::make_integer_sequence<int, 17>{});
  if (K <= kNormThreads * kNormMaxJ && add.n >= 0 && add.n <= 16)
    fns[add.n]<<<act.nt8 * 8, kNormThreads, 0, s>>>(x, ldx, add, rows, w, eps, n, K, act);
  else
    k_rmsnorm_quant<<<act.nt8 * 8, 256, 0, s>>>(x, ldx, add, rows, w, eps, n, K, act);
}

void launch_sum_slices(Slices src, int64_t ld, int n, int cols, float* dst, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(n) * cols;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 2048));
  if (total > 0) k_sum_slices<<<blocks, 256, 0, s>>>(src, ld, n, cols, dst);
}

void launch_silu_quant(Slices gu, int64_t ld, int F, int n, const ActQ& act, cudaStream_t s) {
  const int nb = F / 32;
  dim3 grid((nb + 7) / 8, act.nt8 * 8);
  static constexpr auto fns = silu_table(std::make_integer_sequence<int, 16>{});
  if (gu.n >= 1 && gu.n <= 16) fns[gu.n - 1]<<<grid, 256, 0, s>>>(gu, ld, F, n, act);
}

void launch_quant_blockq8(const float* x, int n, int64_t K, void* blocks, cudaStream_t s) {
  const int64_t nb = K / 32;
  dim3 grid(static_cast<unsigned>((nb + 7) / 8), n);
  k_quant_blockq8<<<grid, 256, 0, s>>>(x, K, static_cast<uint8_t*>(blocks));
}

void launch_quant_i8(const float* x, int n, int len, int8_t* q, float* scale, cudaStream_t s) {
  k_quant_i8<<<(n + 7) / 8, 256, 0, s>>>(x, n, len, q, scale);
}

void launch_silu_mul(float* g, const float* u, int64_t n, cudaStream_t s) {
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4096));
  k_silu_mul<<<blocks > 0 ? blocks : 1, 256, 0, s>>>(g, u, n);
}

}  // namespace mkb
