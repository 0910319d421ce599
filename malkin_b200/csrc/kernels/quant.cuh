// Warp-level Q8 block quantization (kern::quantize_row_q8, kernels_avx512.cpp:66-80) and the store of a quantized
// block into the GEMM activation layouts (layout.hpp). Lane i of the warp holds value i of the 32-value block.
//
// Bit-exactness with malkin's BlockQ8 given the same float input: d = amax / 127 (IEEE division), id = 1 / d
// (0 when d == 0), q = round-half-even(x * id) saturated to int8, s[0] / s[1] = integer sums of the two 16-value
// halves of the unsaturated ints.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

struct QBlock {
  int q;     // saturated int8 value of this lane
  float d;
  int s0, s1;
};

__device__ __forceinline__ QBlock quant_block32(float v, int lane) {
  QBlock r;
  const float amax = warp_max(fabsf(v));
  r.d = __fdiv_rn(amax, 127.0f);
  const float id = r.d != 0.0f ? __fdiv_rn(1.0f, r.d) : 0.0f;
  const int qi = __float2int_rn(__fmul_rn(v, id));
  r.q = max(-128, min(127, qi));
  int h = qi;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) h += __shfl_xor_sync(0xffffffffu, h, o);  // sums within 16-lane halves
  r.s0 = __shfl_sync(0xffffffffu, h, 0);
  r.s1 = __shfl_sync(0xffffffffu, h, 16);
  (void)lane;
  return r;
}

// Writes block b of token t (this warp's lane values already quantized; v: the lane's float value) into the GEMM
// layout, and the float value into a.xf when float weights read it.
__device__ __forceinline__ void store_act(const ActQ& a, int b, int t, const QBlock& qb, int lane, float v) {
  const int npad = a.nt8 * 8;
  if (a.xf) a.xf[static_cast<size_t>(t) * a.ldxf + b * 32 + lane] = v;
  // Gather 4 consecutive lanes' bytes into one word at lane 4m.
  const uint32_t byte = static_cast<uint32_t>(qb.q) & 0xFFu;
  const uint32_t b1 = __shfl_down_sync(0xffffffffu, byte, 1);
  const uint32_t b2 = __shfl_down_sync(0xffffffffu, byte, 2);
  const uint32_t b3 = __shfl_down_sync(0xffffffffu, byte, 3);
  if ((lane & 3) == 0) {
    const uint32_t word = byte | (b1 << 8) | (b2 << 16) | (b3 << 24);
    const int m = lane >> 2;  // k = 4m .. 4m+3
    const int c = m & 3, hi = m >> 2;
    const int j = t >> 3, g = t & 7;
    uint8_t* dst = a.qx + (static_cast<size_t>(b) * a.nt8 + j) * 256 + (g * 4 + c) * 8 + hi * 4;
    *reinterpret_cast<uint32_t*>(dst) = word;
    if (a.qc) {
      // tensor-core order: values 16 h .. 16 h + 15 of token t at (t / 8) * 256 + h * 128 + (t % 8) * 16
      uint8_t* dq = a.qc + static_cast<size_t>(b) * npad * 32 + j * 256 + (m >> 2) * 128 + g * 16 + (m & 3) * 4;
      *reinterpret_cast<uint32_t*>(dq) = word;
    }
  }
  if (lane == 0) {
    const size_t o = static_cast<size_t>(b) * npad + t;
    a.dx[o] = qb.d;
    if (a.dsx) a.dsx[o] = __fmul_rn(qb.d, static_cast<float>(qb.s0 + qb.s1));
    if (a.sh) a.sh[o] = (static_cast<uint32_t>(qb.s0) & 0xFFFFu) | (static_cast<uint32_t>(qb.s1) << 16);
  }
}

}  // namespace mkb
