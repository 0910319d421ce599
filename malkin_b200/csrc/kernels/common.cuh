// Device helpers shared by the kernels: packed f32x2 arithmetic (sm_100), int8 warp MMA, streaming loads,
// warp reductions, and the device panel layouts the host repack writes (layout.hpp).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "../host/layout.hpp"

namespace mkb {

// ---- packed f32x2 (two fp32 lanes in one 64-bit register; one instruction, round to nearest even) ----
typedef unsigned long long f2;

__device__ __forceinline__ f2 f2_make(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ f2 f2_bits(uint32_t lo, uint32_t hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(f2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo;
}
__device__ __forceinline__ float f2_hi(f2 v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return hi;
}
__device__ __forceinline__ f2 f2_sub(f2 a, f2 b) {
  f2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
  f2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
  f2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// a * b + c, one rounding per lane.
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
  f2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// ---- int8 warp MMA (legacy mma.sync; accumulator init C carries the float-conversion bias, see kMagic) ----
// The int32 result d = C + sum(a * b). With C = kMagicBits (the bits of 1.5 * 2^23), d's bits are the float
// 12582912 + dot exactly for |dot| < 2^22, so one float subtract of kMagicF yields float(dot) with no I2F.
constexpr int32_t kMagicBits = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ void mma_s8_k32(int32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                           int32_t c0, int32_t c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
}
// Unsigned A (0..255) x signed B, K = 16.
__device__ __forceinline__ void mma_u8s8_k16(int32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0, int32_t c0,
                                             int32_t c1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
               : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1), "r"(c0), "r"(c1));
}

// ---- loads ----
// Weights are streamed once per forward: bypass L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ float h2f_lo(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFF))); }
__device__ __forceinline__ float h2f_hi(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))); }

// ---- warp reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_isum(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// The horizontal sum of malkin's 16-lane AVX-512 accumulators (_mm512_reduce_add_ps), over the 16 consecutive lanes
// that hold them (lane l of each half-warp holds accumulator l): lanes l and l ^ 8 first, then l ^ 4, l ^ 2, l ^ 1 -
// the same additions in the same pairing (IEEE addition is commutative), so every lane of the half-warp ends with the
// bit-identical sum.
__device__ __forceinline__ float reduce16(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return v;
}

// kern::dot_f32(n, x, x) (kernels_avx512.cpp:82-89) of a row in shared memory, the way malkin's RMSNorm computes it
// (model.cpp:46-49): 16 accumulators, accumulator l summing x[l + 16 k]^2 by fma in k order from zero, then reduce16.
// Called by one whole warp (lanes 0..15 run the chains); every lane returns the sum. n % 16 == 0.
__device__ __forceinline__ float dot16_self(const float* x, int n, int lane) {
  float acc = 0.0f;
  if (lane < 16) {
#pragma unroll 8
    for (int i = lane; i < n; i += 16) acc = __fmaf_rn(x[i], x[i], acc);
  }
  acc = reduce16(acc);
  return __shfl_sync(0xffffffffu, acc, 0);
}

// Sum of n <= 16 values p[0], p[stride], ... in index order. All loads are issued before the first add, so the
// latency of the n loads overlaps (a plain runtime-bounded loop would wait for each in turn).
__device__ __forceinline__ float sum_strided16(const float* p, int n, int64_t stride) {
  float v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = i < n ? p[i * stride] : 0.0f;
  float r = v[0];
#pragma unroll
  for (int i = 1; i < 16; ++i)
    if (i < n) r = __fadd_rn(r, v[i]);
  return r;
}

// The same for a slice count fixed at compile time (no predicates): loads first, then the sum in index order.
template <int NS>
__device__ __forceinline__ float sum_strided(const float* p, int64_t stride) {
  float v[NS > 0 ? NS : 1];
#pragma unroll
  for (int i = 0; i < NS; ++i) v[i] = p[i * stride];
  float r = NS > 0 ? v[0] : 0.0f;
#pragma unroll
  for (int i = 1; i < NS; ++i) r = __fadd_rn(r, v[i]);
  return r;
}

// e^x as malkin computes it for softmax and SiLU (kernels_avx512.cpp:186-203): clamp below at -87, Cody-Waite
// reduction with ln 2 split in two, degree-6 Taylor polynomial in Horner form with fused multiply-adds, then
// scaling by 2^n. (malkin's own algorithm, restated, so both sides exponentiate identically.)
// cp.async (16-byte global -> shared copies, 4-byte for unaligned scalars), commit groups and bounded waits
__device__ __forceinline__ void cp_async16(void* sm, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(sm))),
               "l"(g)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* sm, const void* g) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(sm))),
               "l"(g)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ float exp_malkin(float x) {
  x = fmaxf(x, -87.0f);
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860682030941723e-6f, r);
  float p = 1.0f / 720.0f;
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  // p * 2^n: n >= -126 after the clamp; n >= 128 gives +inf, as scaling by 2^n does.
  const int e = static_cast<int>(fminf(n, 128.0f));
  return __fmul_rn(p, __int_as_float((e + 127) << 23));
}

}  // namespace mkb
