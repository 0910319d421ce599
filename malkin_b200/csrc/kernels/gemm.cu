// Quantized weight-streaming GEMM: y[t][r] = sum over blocks of float(int8 block dot) * (weight scale * act scale),
// the arithmetic of malkin's panel kernels k_q8_0 / k_q45_k / k_q6_k (gemm_avx512.cpp:67-205), on B200.
//
// Work split: a warp owns one 16-row panel and all tokens of the batch (NT tiles of 8); a CTA is 4 warps
// (4 panels) and a k-unit range (split-K: grid.y). Weights are read once, straight from HBM into registers in the
// mma.sync A-fragment layout of the panel repack (one 16-byte coalesced load per lane per 32-value block,
// prefetched PF blocks ahead); activations (the n x K Q8 blocks, small and shared by all warps) come through L1.
//
// Per 32-value block (16-value half for Q6_K) and 16 x 8 tile, one int8 mma.sync produces the exact integer dots;
// the accumulator init carries the float-conversion bias (kMagicBits) so the dot becomes a float with one packed
// subtract, then the per-block scale product and the accumulate are packed f32x2 multiply / fma - the same
// roundings, in the same order over blocks, as malkin: acc = fma(float(dot), d_w * d_x, acc) (Q4_K: then
// acc = fma(-d_min * m, d_x * float(s0 + s1), acc)). With split = 1 each (row, token) sums its blocks in order, so
// y is bit-identical to malkin's compact panel kernels.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

namespace {

constexpr int kWarps = 4;
constexpr int kMaxNT = 18;  // 144 tokens per pass

struct GemmArgs {
  const uint8_t* w;
  int64_t panels;
  int kunits, per_split;
  const uint8_t* qx;
  const float* dx;
  const float* dsx;
  const uint32_t* sh;
  int nt8;  // layout stride (token tiles of the activation buffer)
  int t0;   // first token of this pass
  float* y;
  int64_t ldy, rows;
  int n;  // total tokens
  int atomic;
};

template <int NT>
__device__ __forceinline__ void store_tile(const GemmArgs& a, f2 (&acc)[NT][2], int64_t p, int lane) {
  const int g = lane >> 2, c = lane & 3;
  const int64_t r0 = p * 16 + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int t = a.t0 + 8 * j + 2 * c;
    const float v[4] = {f2_lo(acc[j][0]), f2_hi(acc[j][0]), f2_lo(acc[j][1]), f2_hi(acc[j][1])};
    const int tt[4] = {t, t + 1, t, t + 1};
    const int64_t rr[4] = {r0, r0, r1, r1};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (tt[e] < a.n && rr[e] < a.rows) {
        float* dst = a.y + static_cast<int64_t>(tt[e]) * a.ldy + rr[e];
        if (a.atomic)
          atomicAdd(dst, v[e]);
        else
          *dst = v[e];
      }
    }
  }
}

// ---------------- Q8_0 ----------------
template <int NT>
__global__ void __launch_bounds__(kWarps * 32) k_gemm_q8_0(GemmArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, c = lane & 3;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (p >= a.panels) return;
  const int u0 = blockIdx.y * a.per_split, u1 = min(a.kunits, u0 + a.per_split);
  const int npad = a.nt8 * 8;
  const uint8_t* wp = a.w + static_cast<size_t>(p) * a.kunits * kChunkQ8_0;
  const f2 magic2 = f2_make(kMagicF, kMagicF);
  f2 acc[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = f2_make(0.0f, 0.0f);

  constexpr int PF = 4;
  uint4 abuf[PF];
  uint32_t sbuf[PF];
#pragma unroll
  for (int i = 0; i < PF; ++i) {
    if (u0 + i < u1) {
      abuf[i] = ld_stream16(wp + static_cast<size_t>(u0 + i) * kChunkQ8_0 + lane * 16);
      sbuf[i] = ld_stream4(wp + static_cast<size_t>(u0 + i) * kChunkQ8_0 + 512 + (lane >> 2) * 4);
    }
  }
  const uint8_t* qxl = a.qx + lane * 8 + static_cast<size_t>(a.t0 / 8) * 256;
  const float* dxl = a.dx + 2 * c + a.t0;
  for (int u = u0; u < u1; u += PF) {
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int uu = u + i;
      if (uu < u1) {
        const uint32_t av[4] = {abuf[i].x, abuf[i].y, abuf[i].z, abuf[i].w};
        const uint32_t sw = sbuf[i];
        if (uu + PF < u1) {
          abuf[i] = ld_stream16(wp + static_cast<size_t>(uu + PF) * kChunkQ8_0 + lane * 16);
          sbuf[i] = ld_stream4(wp + static_cast<size_t>(uu + PF) * kChunkQ8_0 + 512 + (lane >> 2) * 4);
        }
        const float dwg = h2f_lo(sw), dwg8 = h2f_hi(sw);
        const f2 DWG = f2_make(dwg, dwg), DWG8 = f2_make(dwg8, dwg8);
        const uint8_t* qxb = qxl + static_cast<size_t>(uu) * a.nt8 * 256;
        const float* dxb = dxl + static_cast<size_t>(uu) * npad;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          const uint2 b = __ldg(reinterpret_cast<const uint2*>(qxb + j * 256));
          const float2 dx = __ldg(reinterpret_cast<const float2*>(dxb + 8 * j));
          int32_t d[4];
          mma_s8_k32(d, av, b.x, b.y, kMagicBits, kMagicBits);
          const f2 DX = f2_make(dx.x, dx.y);
          const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
          acc[j][0] = f2_fma(f01, f2_mul(DWG, DX), acc[j][0]);
          acc[j][1] = f2_fma(f23, f2_mul(DWG8, DX), acc[j][1]);
        }
      }
    }
  }
  store_tile<NT>(a, acc, p, lane);
}

// ---------------- Q4_K ----------------
// scale_min_k4 (kernels.h:18-26) on the 12 packed bytes held in words w1 (bytes 4-7), w2 (8-11), w3 (12-15).
__device__ __forceinline__ void q4k_scale_min(int j, uint32_t w1, uint32_t w2, uint32_t w3, int& sc, int& m) {
  if (j < 4) {
    sc = (w1 >> (8 * j)) & 63;
    m = (w2 >> (8 * j)) & 63;
  } else {
    const int jj = j - 4;
    sc = ((w3 >> (8 * jj)) & 0xF) | (((w1 >> (8 * jj + 6)) & 3) << 4);
    m = ((w3 >> (8 * jj + 4)) & 0xF) | (((w2 >> (8 * jj + 6)) & 3) << 4);
  }
}

template <int NT>
__global__ void __launch_bounds__(kWarps * 32) k_gemm_q4_k(GemmArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (p >= a.panels) return;
  const int u0 = blockIdx.y * a.per_split, u1 = min(a.kunits, u0 + a.per_split);
  const int npad = a.nt8 * 8;
  const uint8_t* wp = a.w + static_cast<size_t>(p) * a.kunits * kChunkQ4_K;
  const f2 magic2 = f2_make(kMagicF, kMagicF);
  f2 acc[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = f2_make(0.0f, 0.0f);
  const uint8_t* qxl = a.qx + lane * 8 + static_cast<size_t>(a.t0 / 8) * 256;
  const float* dxl = a.dx + 2 * c + a.t0;
  const float* dsxl = a.dsx + 2 * c + a.t0;

  uint2 nb[2][8];
  uint4 hg[2], hg8[2];
  auto load = [&](int slot, int u) {
    const uint8_t* cp = wp + static_cast<size_t>(u) * kChunkQ4_K;
#pragma unroll
    for (int j = 0; j < 8; ++j) nb[slot][j] = ld_stream8(cp + 256 * j + 8 * lane);
    hg[slot] = ld_stream16(cp + 2048 + 32 * g);
    hg8[slot] = ld_stream16(cp + 2048 + 32 * g + 16);
  };
  if (u0 < u1) load(0, u0);
  int slot = 0;
  for (int u = u0; u < u1; ++u, slot ^= 1) {
    if (u + 1 < u1) load(slot ^ 1, u + 1);
    const uint4 H = hg[slot], H8 = hg8[slot];
    const float dg = h2f_lo(H.x), dming = h2f_hi(H.x), dg8 = h2f_lo(H8.x), dming8 = h2f_hi(H8.x);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int sc0, m0, sc1, m1;
      q4k_scale_min(j, H.y, H.z, H.w, sc0, m0);
      q4k_scale_min(j, H8.y, H8.z, H8.w, sc1, m1);
      const float scg = __fmul_rn(dg, static_cast<float>(sc0)), scg8 = __fmul_rn(dg8, static_cast<float>(sc1));
      const float mng = __fmul_rn(dming, static_cast<float>(m0)), mng8 = __fmul_rn(dming8, static_cast<float>(m1));
      const f2 SC = f2_make(scg, scg), SC8 = f2_make(scg8, scg8);
      const f2 MN = f2_make(-mng, -mng), MN8 = f2_make(-mng8, -mng8);
      const uint2 w = nb[slot][j];
      const uint32_t av[4] = {w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, (w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu};
      const int blk = u * 8 + j;
      const uint8_t* qxb = qxl + static_cast<size_t>(blk) * a.nt8 * 256;
      const float* dxb = dxl + static_cast<size_t>(blk) * npad;
      const float* dsxb = dsxl + static_cast<size_t>(blk) * npad;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint2 b = __ldg(reinterpret_cast<const uint2*>(qxb + t * 256));
        const float2 dx = __ldg(reinterpret_cast<const float2*>(dxb + 8 * t));
        const float2 dsx = __ldg(reinterpret_cast<const float2*>(dsxb + 8 * t));
        int32_t d[4];
        mma_s8_k32(d, av, b.x, b.y, kMagicBits, kMagicBits);
        const f2 DX = f2_make(dx.x, dx.y), DSX = f2_make(dsx.x, dsx.y);
        const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
        acc[t][0] = f2_fma(MN, DSX, f2_fma(f01, f2_mul(SC, DX), acc[t][0]));
        acc[t][1] = f2_fma(MN8, DSX, f2_fma(f23, f2_mul(SC8, DX), acc[t][1]));
      }
    }
  }
  store_tile<NT>(a, acc, p, lane);
}

// ---------------- Q6_K ----------------
template <int NT>
__global__ void __launch_bounds__(kWarps * 32) k_gemm_q6_k(GemmArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t p = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  if (p >= a.panels) return;
  const int u0 = blockIdx.y * a.per_split, u1 = min(a.kunits, u0 + a.per_split);
  const int npad = a.nt8 * 8;
  const uint8_t* wp = a.w + static_cast<size_t>(p) * a.kunits * kChunkQ6_K;
  const f2 magic2 = f2_make(kMagicF, kMagicF);
  f2 acc[NT][2];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = f2_make(0.0f, 0.0f);
  const uint8_t* qxl = a.qx + lane * 8 + static_cast<size_t>(a.t0 / 8) * 256;
  const float* dxl = a.dx + 2 * c + a.t0;
  const uint32_t* shl = a.sh + 2 * c + a.t0;

  uint2 nb[2][8];
  uint32_t hb[2][8];
  uint4 scg[2], scg8[2];
  uint32_t dw[2];
  auto load = [&](int slot, int u) {
    const uint8_t* cp = wp + static_cast<size_t>(u) * kChunkQ6_K;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      nb[slot][j] = ld_stream8(cp + 256 * j + 8 * lane);
      hb[slot][j] = ld_stream4(cp + 2048 + 128 * j + 4 * lane);
    }
    scg[slot] = ld_stream16(cp + 3072 + 32 * g);
    scg8[slot] = ld_stream16(cp + 3072 + 32 * g + 16);
    dw[slot] = ld_stream4(cp + 3328 + 4 * g);
  };
  if (u0 < u1) load(0, u0);
  int slot = 0;
  for (int u = u0; u < u1; ++u, slot ^= 1) {
    if (u + 1 < u1) load(slot ^ 1, u + 1);
    const float dg = h2f_lo(dw[slot]), dg8 = h2f_hi(dw[slot]);
    const uint32_t sgw[4] = {scg[slot].x, scg[slot].y, scg[slot].z, scg[slot].w};
    const uint32_t sgw8[4] = {scg8[slot].x, scg8[slot].y, scg8[slot].z, scg8[slot].w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint2 w = nb[slot][j];
      const uint32_t h = hb[slot][j];
      const uint32_t a0 = (w.x & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
      const uint32_t a1 = (w.y & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
      const uint32_t a2 = ((w.x >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);
      const uint32_t a3 = ((w.y >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
      // int8 scales of sub-blocks 2j, 2j+1 (bytes of the 16-byte scale vectors)
      const int i0 = 2 * j, i1 = 2 * j + 1;
      const int s0g = static_cast<int8_t>((sgw[i0 >> 2] >> (8 * (i0 & 3))) & 0xFF);
      const int s1g = static_cast<int8_t>((sgw[i1 >> 2] >> (8 * (i1 & 3))) & 0xFF);
      const int s0g8 = static_cast<int8_t>((sgw8[i0 >> 2] >> (8 * (i0 & 3))) & 0xFF);
      const int s1g8 = static_cast<int8_t>((sgw8[i1 >> 2] >> (8 * (i1 & 3))) & 0xFF);
      const float d0g = __fmul_rn(dg, static_cast<float>(s0g)), d1g = __fmul_rn(dg, static_cast<float>(s1g));
      const float d0g8 = __fmul_rn(dg8, static_cast<float>(s0g8)), d1g8 = __fmul_rn(dg8, static_cast<float>(s1g8));
      const f2 D0 = f2_make(d0g, d0g), D1 = f2_make(d1g, d1g), D08 = f2_make(d0g8, d0g8), D18 = f2_make(d1g8, d1g8);
      const int blk = u * 8 + j;
      const uint8_t* qxb = qxl + static_cast<size_t>(blk) * a.nt8 * 256;
      const float* dxb = dxl + static_cast<size_t>(blk) * npad;
      const uint32_t* shb = shl + static_cast<size_t>(blk) * npad;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint2 b = __ldg(reinterpret_cast<const uint2*>(qxb + t * 256));
        const float2 dx = __ldg(reinterpret_cast<const float2*>(dxb + 8 * t));
        const uint2 s = __ldg(reinterpret_cast<const uint2*>(shb + 8 * t));
        const f2 DX = f2_make(dx.x, dx.y);
        // half 0: C = magic - 32 * s[0] per token; half 1: s[1]
        const int c0a = kMagicBits - 32 * static_cast<int16_t>(s.x & 0xFFFF);
        const int c0b = kMagicBits - 32 * static_cast<int16_t>(s.y & 0xFFFF);
        const int c1a = kMagicBits - 32 * static_cast<int16_t>(s.x >> 16);
        const int c1b = kMagicBits - 32 * static_cast<int16_t>(s.y >> 16);
        int32_t d[4], e[4];
        mma_u8s8_k16(d, a0, a1, b.x, c0a, c0b);
        mma_u8s8_k16(e, a2, a3, b.y, c1a, c1b);
        const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
        const f2 h01 = f2_sub(f2_bits(e[0], e[1]), magic2), h23 = f2_sub(f2_bits(e[2], e[3]), magic2);
        acc[t][0] = f2_fma(h01, f2_mul(D1, DX), f2_fma(f01, f2_mul(D0, DX), acc[t][0]));
        acc[t][1] = f2_fma(h23, f2_mul(D18, DX), f2_fma(f23, f2_mul(D08, DX), acc[t][1]));
      }
    }
  }
  store_tile<NT>(a, acc, p, lane);
}

// ---------------- exact block dots (parity tests) ----------------
// grid (panels), block 32: one warp per panel, all tokens in tiles of 8, every block.
__global__ void k_block_dots(uint32_t type, const uint8_t* __restrict__ w, int64_t panels, int kunits, int64_t rows,
                             ActQ act, int n, int32_t* __restrict__ out) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t p = blockIdx.x;
  const int npad = act.nt8 * 8;
  const bool q6 = type == 14;
  const int nblk = q6 ? kunits * 16 : (type == 8 ? kunits : kunits * 8);  // output blocks per (row, token)
  const int blocks = type == 8 ? kunits : kunits * 8;                        // 32-value blocks
  for (int bl = 0; bl < blocks; ++bl) {
    uint32_t av[4];
    if (type == 8) {
      const uint4 A = *reinterpret_cast<const uint4*>(w + (static_cast<size_t>(p) * kunits + bl) * kChunkQ8_0 + lane * 16);
      av[0] = A.x, av[1] = A.y, av[2] = A.z, av[3] = A.w;
    } else {
      const size_t cb = q6 ? kChunkQ6_K : kChunkQ4_K;
      const uint8_t* cp = w + (static_cast<size_t>(p) * kunits + bl / 8) * cb;
      const int j = bl % 8;
      const uint2 wv = *reinterpret_cast<const uint2*>(cp + 256 * j + 8 * lane);
      av[0] = wv.x & 0x0F0F0F0Fu, av[1] = wv.y & 0x0F0F0F0Fu;
      av[2] = (wv.x >> 4) & 0x0F0F0F0Fu, av[3] = (wv.y >> 4) & 0x0F0F0F0Fu;
      if (q6) {
        const uint32_t h = *reinterpret_cast<const uint32_t*>(cp + 2048 + 128 * j + 4 * lane);
        av[0] |= (h << 4) & 0x30303030u;
        av[1] |= (h << 2) & 0x30303030u;
        av[2] |= h & 0x30303030u;
        av[3] |= (h >> 2) & 0x30303030u;
      }
    }
    for (int tt = 0; tt < act.nt8; ++tt) {
      const uint2 b = *reinterpret_cast<const uint2*>(act.qx + (static_cast<size_t>(bl) * act.nt8 + tt) * 256 + lane * 8);
      const int t0 = 8 * tt + 2 * c;
      int32_t d[4], e[4];
      if (q6) {
        const uint32_t s0 = act.sh[static_cast<size_t>(bl) * npad + t0], s1 = act.sh[static_cast<size_t>(bl) * npad + t0 + 1];
        mma_u8s8_k16(d, av[0], av[1], b.x, kMagicBits - 32 * static_cast<int16_t>(s0 & 0xFFFF),
                     kMagicBits - 32 * static_cast<int16_t>(s1 & 0xFFFF));
        mma_u8s8_k16(e, av[2], av[3], b.y, kMagicBits - 32 * static_cast<int16_t>(s0 >> 16),
                     kMagicBits - 32 * static_cast<int16_t>(s1 >> 16));
      } else {
        mma_s8_k32(d, av, b.x, b.y, kMagicBits, kMagicBits);
      }
      const int64_t rr[4] = {p * 16 + g, p * 16 + g, p * 16 + g + 8, p * 16 + g + 8};
      const int ts[4] = {t0, t0 + 1, t0, t0 + 1};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (rr[q] >= rows || ts[q] >= n) continue;
        int32_t* o = out + (rr[q] * n + ts[q]) * static_cast<int64_t>(nblk);
        if (q6) {
          o[2 * bl] = d[q] - kMagicBits;
          o[2 * bl + 1] = e[q] - kMagicBits;
        } else {
          o[bl] = d[q] - kMagicBits;
        }
      }
    }
  }
}

template <template <int> class K>
struct Table;

#define MK_TABLE(KERNEL)                                                                                        \
  using Fn_##KERNEL = void (*)(GemmArgs);                                                                       \
  constexpr Fn_##KERNEL tab_##KERNEL[kMaxNT] = {                                                                \
      KERNEL<1>,  KERNEL<2>,  KERNEL<3>,  KERNEL<4>,  KERNEL<5>,  KERNEL<6>,  KERNEL<7>,  KERNEL<8>,  KERNEL<9>, \
      KERNEL<10>, KERNEL<11>, KERNEL<12>, KERNEL<13>, KERNEL<14>, KERNEL<15>, KERNEL<16>, KERNEL<17>, KERNEL<18>};
MK_TABLE(k_gemm_q8_0)
MK_TABLE(k_gemm_q4_k)
MK_TABLE(k_gemm_q6_k)
#undef MK_TABLE

}  // namespace

int gemm_auto_split(const DevWeight& w, int n, int num_sms) {
  (void)n;
  const int64_t ctas = (w.panels + kWarps - 1) / kWarps;
  const int64_t target = 2LL * num_sms;
  if (ctas >= target) return 1;
  int split = static_cast<int>((target + ctas - 1) / ctas);
  split = std::min(split, std::max(1, w.kunits / 2));
  return std::max(1, split);
}

void launch_gemm(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int split, bool atomic,
                 cudaStream_t s) {
  if (n <= 0) return;
  split = std::max(1, std::min(split, w.kunits));
  const int per = (w.kunits + split - 1) / split;
  const int gy = (w.kunits + per - 1) / per;
  GemmArgs a{};
  a.w = w.data;
  a.panels = w.panels;
  a.kunits = w.kunits;
  a.per_split = per;
  a.qx = act.qx;
  a.dx = act.dx;
  a.dsx = act.dsx;
  a.sh = act.sh;
  a.nt8 = act.nt8;
  a.y = y;
  a.ldy = ldy;
  a.rows = w.rows;
  a.n = n;
  a.atomic = (atomic || gy > 1) ? 1 : 0;
  const dim3 grid(static_cast<unsigned>((w.panels + kWarps - 1) / kWarps), static_cast<unsigned>(gy));
  // Token passes of up to kMaxNT tiles (larger batches stream the weights once per pass).
  const int tiles = (n + 7) / 8;
  for (int t0 = 0; t0 < tiles; t0 += kMaxNT) {
    const int nt = std::min(kMaxNT, tiles - t0);
    a.t0 = t0 * 8;
    switch (w.type) {
      case 8:
        tab_k_gemm_q8_0[nt - 1]<<<grid, kWarps * 32, 0, s>>>(a);
        break;
      case 12:
        tab_k_gemm_q4_k[nt - 1]<<<grid, kWarps * 32, 0, s>>>(a);
        break;
      case 14:
        tab_k_gemm_q6_k[nt - 1]<<<grid, kWarps * 32, 0, s>>>(a);
        break;
      default:
        break;
    }
  }
}

void launch_block_dots(const DevWeight& w, const ActQ& act, int n, int32_t* out, cudaStream_t s) {
  k_block_dots<<<static_cast<unsigned>(w.panels), 32, 0, s>>>(w.type, w.data, w.panels, w.kunits, w.rows, act, n, out);
}

}  // namespace mkb
