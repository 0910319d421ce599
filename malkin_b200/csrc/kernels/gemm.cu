// Quantized weight-streaming GEMM: y[t][r] = sum over blocks of float(int8 block dot) * (weight scale * act scale),
// the arithmetic of malkin's panel kernels k_q8_0 / k_q45_k / k_q6_k (gemm_avx512.cpp:67-205), on B200.
//
// Pipeline: a CTA owns a tile of 2 WP panels (32 WP weight rows), one token pass of WT x NTW tiles of 8 tokens
// (WT = 8 / WP) and one k-range (split-K slice). Warp 0 streams the tile's weight chunks and the matching activation
// blocks (Q8 fragments, scales) from HBM / L2 into a 2-3 stage shared-memory ring with TMA bulk copies
// (cp.async.bulk, completion counted on mbarriers) and refills a stage as soon as all eight warps have released it;
// warp w takes panels 2 (w % WP), +1 x token tiles (w / WP) NTW .. + NTW - 1. Token passes (grid.z) and narrow
// tiles (WP < 8) give the SMs work without splitting K, so every (row, token) sums its blocks in malkin's order;
// the passes of one tile read its weights from L2 after the first.
//
// Arithmetic per 32-value block (16-value half for Q6_K) and 16 x 8 tile: one int8 mma.sync gives the exact
// integer dots; its accumulator init carries the float-conversion bias (kMagicBits) so the dot becomes a float with
// one packed subtract; then the per-block scale product and the accumulate are packed f32x2 mul / fma - the same
// roundings in the same block order as malkin: acc = fma(float(dot), d_w * d_x, acc) (Q4_K then
// acc = fma(-(d_min * m), d_x * float(s0 + s1), acc); Q6_K per half with d * sc). A slice of split-K writes its
// partial sums with plain stores to its own output slice; the consuming kernel adds the slices in slice order, so
// results are deterministic, and with one slice each (row, token) sums its blocks in malkin's order: y is then
// bit-identical to malkin's compact panel kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <array>
#include <utility>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "kernels.hpp"
#include "pipeline.cuh"

namespace mkb {

namespace {

constexpr int kTilePanels = 16;                      // panels of the widest tile (WP = 8)
constexpr int kConsumers = 8;                        // warps, 2 panels each; warp 0 also issues the TMA copies
constexpr int kThreadsG = kConsumers * 32;           // 2 warps per SM sub-partition: up to 255 registers
constexpr int kMaxNT = 18;                           // 144 tokens per pass

template <uint32_t T>
struct TypeCfg;
template <>
struct TypeCfg<8> {  // Q8_0: unit = one 32-value block
  static constexpr int KS = 4, NS = 3, BPU = 1;
  static constexpr uint32_t UNIT = kChunkQ8_0;
  static constexpr bool kDsx = false, kSh = false;
};
template <>
struct TypeCfg<12> {  // Q4_K: unit = 256-value super-block
  static constexpr int KS = 1, NS = 2, BPU = 8;
  static constexpr uint32_t UNIT = kChunkQ4_K;
  static constexpr bool kDsx = true, kSh = false;
};
template <>
struct TypeCfg<14> {  // Q6_K
  static constexpr int KS = 1, NS = 2, BPU = 8;
  static constexpr uint32_t UNIT = kChunkQ6_K;
  static constexpr bool kDsx = false, kSh = true;
};

struct GemmArgs {
  const uint8_t* w;
  int64_t panels;
  int kunits, per_split;
  const uint8_t* qx;
  const float* dx;
  const float* dsx;
  const uint32_t* sh;
  int nt8;  // token tiles of the activation buffer (its layout stride)
  float* y;
  int64_t ldy, rows, slice;  // slice: floats between split-K output slices
  int n;                     // tokens
  int* status;
};

// Shared-memory layout of one stage (NT token tiles, TP panels, KSX k-units per stage; 0 = the type's default) and
// the ring depth: the type's default, fewer stages when a stage is large (at most ~200 KB in all, at least 2).
template <uint32_t T, int NT, int TP = kTilePanels, int KSX = 0>
struct Stage {
  using C = TypeCfg<T>;
  static constexpr int KS = KSX ? KSX : C::KS;
  static constexpr uint32_t A = TP * KS * C::UNIT;
  static constexpr uint32_t B = KS * C::BPU * NT * 256;
  static constexpr uint32_t DX = KS * C::BPU * NT * 8 * 4;
  static constexpr uint32_t EX = (C::kDsx || C::kSh) ? DX : 0;
  static constexpr uint32_t BYTES = A + B + DX + EX;
  // the type's ring depth when it fits 2 CTAs per SM or only 1 CTA fits anyway; else 2 stages, so 2 CTAs share an SM
  static constexpr int NS = C::NS * BYTES <= 110u * 1024 ? C::NS
                            : (2 * BYTES <= 110u * 1024 ? 2 : (C::NS * BYTES <= 200u * 1024 ? C::NS : 2));
  static constexpr uint32_t SMEM = NS * BYTES + 2 * NS * 8;
};

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

// NTW token tiles per warp, WP panel pairs per CTA (WT = 8 / WP warps along the tokens), KSX k-units per stage
// (0: the type's default; narrow tiles take more per stage, so a stage's work outweighs its barrier).
template <uint32_t T, int NTW, int WP, int KSX>
__global__ void __launch_bounds__(kThreadsG, NTW <= 7 ? 2 : 1) k_gemm(GemmArgs a) {
  using C = TypeCfg<T>;
  constexpr int WT = kConsumers / WP, NT = WT * NTW, TP = 2 * WP;
  using S = Stage<T, NT, TP, KSX>;
  static_assert(S::NS >= 2, "stage ring too small");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::NS * S::BYTES);
  uint64_t* empty = full + S::NS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  // grid (passes, slices, row tiles): the passes of one tile are launched together, so after the first one reads
  // the tile's weights from HBM the others find them in L2
  const int64_t p0 = static_cast<int64_t>(blockIdx.z) * TP;
  const int tile_panels = static_cast<int>(a.panels - p0 < TP ? a.panels - p0 : TP);
  const int u0 = blockIdx.y * a.per_split, u1 = min(a.kunits, u0 + a.per_split);
  const int t0 = blockIdx.x * (NT * 8);  // first token of this pass
  const int jt0 = (warp / WP) * NTW;     // this warp's first token tile within the pass
  const int npad = a.nt8 * 8;
  const int n_it = (u1 - u0 + S::KS - 1) / S::KS;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    mbar_fence_init();
  }
  __syncthreads();

  // Stage refill, issued by warp 0: lane 0 arms the full barrier with the byte count, lanes 0-15 copy the tile's
  // weight chunks (one per panel), lanes 16-23 the activation blocks, dx (and dsx / sh) of each 32-value block.
  auto issue = [&](int it) {
    const int s = it % S::NS;
    const int ua = u0 + it * S::KS, uk = min(S::KS, u1 - ua);  // units in this stage
    const int nb = uk * C::BPU;                                // 32-value blocks in this stage
    // token tiles this pass reads: a last pass past the padded activation rows reads only those that exist (the
    // columns of the missing tiles hold stale shared memory; their outputs are tokens >= n and are never stored)
    const int ntp = min(NT, a.nt8 - t0 / 8);
    const uint32_t bytes = static_cast<uint32_t>(tile_panels) * uk * C::UNIT +
                           static_cast<uint32_t>(nb) * ntp * (256 + 32 + ((C::kDsx || C::kSh) ? 32 : 0));
    uint8_t* st = smem + static_cast<size_t>(s) * S::BYTES;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
    __syncwarp();
    if (lane < tile_panels)
      bulk_g2s(st + lane * (S::KS * C::UNIT), a.w + (static_cast<size_t>(p0 + lane) * a.kunits + ua) * C::UNIT,
               uk * C::UNIT, &full[s]);
    const int blk0 = ua * C::BPU;
    if (lane >= 16 && lane - 16 < nb) {
      const int b = lane - 16;
      bulk_g2s(st + S::A + b * NT * 256, a.qx + (static_cast<size_t>(blk0 + b) * a.nt8 + t0 / 8) * 256, ntp * 256,
               &full[s]);
      bulk_g2s(st + S::A + S::B + b * NT * 32, a.dx + static_cast<size_t>(blk0 + b) * npad + t0, ntp * 32, &full[s]);
      if (C::kDsx)
        bulk_g2s(st + S::A + S::B + S::DX + b * NT * 32, a.dsx + static_cast<size_t>(blk0 + b) * npad + t0, ntp * 32,
                 &full[s]);
      if (C::kSh)
        bulk_g2s(st + S::A + S::B + S::DX + b * NT * 32, a.sh + static_cast<size_t>(blk0 + b) * npad + t0, ntp * 32,
                 &full[s]);
    }
  };
  if (warp == 0)
    for (int it = 0; it < S::NS && it < n_it; ++it) issue(it);

  // ---------------- consumers: warp owns panels pw, pw + 1 of the tile x token tiles jt0 .. jt0 + NTW - 1 ----------------
  const int pw = 2 * (warp % WP);
  const bool has0 = pw < tile_panels, has1 = pw + 1 < tile_panels;
  const f2 magic2 = f2_make(kMagicF, kMagicF);
  f2 acc[2][NTW][2];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int j = 0; j < NTW; ++j) acc[q][j][0] = acc[q][j][1] = f2_make(0.0f, 0.0f);

  for (int it = 0; it < n_it; ++it) {
    const int s = it % S::NS, r = it / S::NS;
    if (!mbar_wait(&full[s], r & 1, a.status, kErrWaitFull)) break;
    const uint8_t* st = smem + static_cast<size_t>(s) * S::BYTES;
    const int uk = min(S::KS, u1 - (u0 + it * S::KS));
    if (has0) {
      const uint8_t* sa0 = st + pw * (S::KS * C::UNIT);
      const uint8_t* sa1 = sa0 + S::KS * C::UNIT;
      const uint8_t* sb = st + S::A + jt0 * 256 + lane * 8;
      const float* sdx = reinterpret_cast<const float*>(st + S::A + S::B) + 8 * jt0 + 2 * c;
      const float* sex = reinterpret_cast<const float*>(st + S::A + S::B + S::DX) + 8 * jt0 + 2 * c;
      for (int u = 0; u < uk; ++u) {
        const uint8_t* ca[2] = {sa0 + u * C::UNIT, sa1 + u * C::UNIT};
        if constexpr (T == 8) {
          uint32_t av[2][4];
          f2 DW[2][2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const uint4 A = *reinterpret_cast<const uint4*>(ca[q] + lane * 16);
            av[q][0] = A.x, av[q][1] = A.y, av[q][2] = A.z, av[q][3] = A.w;
            const uint32_t sw = *reinterpret_cast<const uint32_t*>(ca[q] + 512 + g * 4);
            DW[q][0] = f2_make(h2f_lo(sw), h2f_lo(sw));
            DW[q][1] = f2_make(h2f_hi(sw), h2f_hi(sw));
          }
          const uint8_t* sbb = sb + u * NT * 256;
          const float* dxb = sdx + u * NT * 8;
#pragma unroll
          for (int j = 0; j < NTW; ++j) {
            const uint2 b = *reinterpret_cast<const uint2*>(sbb + j * 256);
            const float2 dx = *reinterpret_cast<const float2*>(dxb + 8 * j);
            const f2 DX = f2_make(dx.x, dx.y);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              int32_t d[4];
              mma_s8_k32(d, av[q], b.x, b.y, kMagicBits, kMagicBits);
              const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
              acc[q][j][0] = f2_fma(f01, f2_mul(DW[q][0], DX), acc[q][j][0]);
              acc[q][j][1] = f2_fma(f23, f2_mul(DW[q][1], DX), acc[q][j][1]);
            }
          }
        } else if constexpr (T == 12) {
          uint4 H[2], H8[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            H[q] = *reinterpret_cast<const uint4*>(ca[q] + 2048 + 32 * g);
            H8[q] = *reinterpret_cast<const uint4*>(ca[q] + 2048 + 32 * g + 16);
          }
#pragma unroll 1
          for (int jb = 0; jb < 8; ++jb) {
            uint32_t av[2][4];
            f2 SC[2][2], MN[2][2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint2 w = *reinterpret_cast<const uint2*>(ca[q] + 256 * jb + 8 * lane);
              av[q][0] = w.x & 0x0F0F0F0Fu, av[q][1] = w.y & 0x0F0F0F0Fu;
              av[q][2] = (w.x >> 4) & 0x0F0F0F0Fu, av[q][3] = (w.y >> 4) & 0x0F0F0F0Fu;
              int sc0, m0, sc1, m1;
              q4k_scale_min(jb, H[q].y, H[q].z, H[q].w, sc0, m0);
              q4k_scale_min(jb, H8[q].y, H8[q].z, H8[q].w, sc1, m1);
              const float scg = __fmul_rn(h2f_lo(H[q].x), static_cast<float>(sc0));
              const float scg8 = __fmul_rn(h2f_lo(H8[q].x), static_cast<float>(sc1));
              const float mng = __fmul_rn(h2f_hi(H[q].x), static_cast<float>(m0));
              const float mng8 = __fmul_rn(h2f_hi(H8[q].x), static_cast<float>(m1));
              SC[q][0] = f2_make(scg, scg), SC[q][1] = f2_make(scg8, scg8);
              MN[q][0] = f2_make(-mng, -mng), MN[q][1] = f2_make(-mng8, -mng8);
            }
            const int bl = u * 8 + jb;
            const uint8_t* sbb = sb + bl * NT * 256;
            const float* dxb = sdx + bl * NT * 8;
            const float* dsb = sex + bl * NT * 8;
#pragma unroll
            for (int j = 0; j < NTW; ++j) {
              const uint2 b = *reinterpret_cast<const uint2*>(sbb + j * 256);
              const float2 dx = *reinterpret_cast<const float2*>(dxb + 8 * j);
              const float2 ds = *reinterpret_cast<const float2*>(dsb + 8 * j);
              const f2 DX = f2_make(dx.x, dx.y), DSX = f2_make(ds.x, ds.y);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                int32_t d[4];
                mma_s8_k32(d, av[q], b.x, b.y, kMagicBits, kMagicBits);
                const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
                acc[q][j][0] = f2_fma(MN[q][0], DSX, f2_fma(f01, f2_mul(SC[q][0], DX), acc[q][j][0]));
                acc[q][j][1] = f2_fma(MN[q][1], DSX, f2_fma(f23, f2_mul(SC[q][1], DX), acc[q][j][1]));
              }
            }
          }
        } else {  // Q6_K
          uint4 SG[2], SG8[2];
          uint32_t DWD[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            SG[q] = *reinterpret_cast<const uint4*>(ca[q] + 3072 + 32 * g);
            SG8[q] = *reinterpret_cast<const uint4*>(ca[q] + 3072 + 32 * g + 16);
            DWD[q] = *reinterpret_cast<const uint32_t*>(ca[q] + 3328 + 4 * g);
          }
#pragma unroll 1
          for (int jb = 0; jb < 8; ++jb) {
            uint32_t av[2][4];
            f2 D0[2][2], D1[2][2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const uint2 w = *reinterpret_cast<const uint2*>(ca[q] + 256 * jb + 8 * lane);
              const uint32_t h = *reinterpret_cast<const uint32_t*>(ca[q] + 2048 + 128 * jb + 4 * lane);
              av[q][0] = (w.x & 0x0F0F0F0Fu) | ((h << 4) & 0x30303030u);
              av[q][1] = (w.y & 0x0F0F0F0Fu) | ((h << 2) & 0x30303030u);
              av[q][2] = ((w.x >> 4) & 0x0F0F0F0Fu) | (h & 0x30303030u);
              av[q][3] = ((w.y >> 4) & 0x0F0F0F0Fu) | ((h >> 2) & 0x30303030u);
              const uint32_t sgw[4] = {SG[q].x, SG[q].y, SG[q].z, SG[q].w};
              const uint32_t sgw8[4] = {SG8[q].x, SG8[q].y, SG8[q].z, SG8[q].w};
              const int i0 = 2 * jb, i1 = 2 * jb + 1;
              const float s0g = static_cast<float>(static_cast<int8_t>((sgw[i0 >> 2] >> (8 * (i0 & 3))) & 0xFF));
              const float s1g = static_cast<float>(static_cast<int8_t>((sgw[i1 >> 2] >> (8 * (i1 & 3))) & 0xFF));
              const float s0g8 = static_cast<float>(static_cast<int8_t>((sgw8[i0 >> 2] >> (8 * (i0 & 3))) & 0xFF));
              const float s1g8 = static_cast<float>(static_cast<int8_t>((sgw8[i1 >> 2] >> (8 * (i1 & 3))) & 0xFF));
              const float dg = h2f_lo(DWD[q]), dg8 = h2f_hi(DWD[q]);
              const float d0g = __fmul_rn(dg, s0g), d1g = __fmul_rn(dg, s1g);
              const float d0g8 = __fmul_rn(dg8, s0g8), d1g8 = __fmul_rn(dg8, s1g8);
              D0[q][0] = f2_make(d0g, d0g), D0[q][1] = f2_make(d0g8, d0g8);
              D1[q][0] = f2_make(d1g, d1g), D1[q][1] = f2_make(d1g8, d1g8);
            }
            const int bl = u * 8 + jb;
            const uint8_t* sbb = sb + bl * NT * 256;
            const float* dxb = sdx + bl * NT * 8;
            const uint32_t* shb = reinterpret_cast<const uint32_t*>(sex) + bl * NT * 8;
#pragma unroll
            for (int j = 0; j < NTW; ++j) {
              const uint2 b = *reinterpret_cast<const uint2*>(sbb + j * 256);
              const float2 dx = *reinterpret_cast<const float2*>(dxb + 8 * j);
              const uint2 sv = *reinterpret_cast<const uint2*>(shb + 8 * j);
              const f2 DX = f2_make(dx.x, dx.y);
              // half 0: C = magic - 32 * s[0] per token; half 1: s[1]
              const int c0a = kMagicBits - 32 * static_cast<int16_t>(sv.x & 0xFFFF);
              const int c0b = kMagicBits - 32 * static_cast<int16_t>(sv.y & 0xFFFF);
              const int c1a = kMagicBits - 32 * static_cast<int16_t>(sv.x >> 16);
              const int c1b = kMagicBits - 32 * static_cast<int16_t>(sv.y >> 16);
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                int32_t d[4], e[4];
                mma_u8s8_k16(d, av[q][0], av[q][1], b.x, c0a, c0b);
                mma_u8s8_k16(e, av[q][2], av[q][3], b.y, c1a, c1b);
                const f2 f01 = f2_sub(f2_bits(d[0], d[1]), magic2), f23 = f2_sub(f2_bits(d[2], d[3]), magic2);
                const f2 h01 = f2_sub(f2_bits(e[0], e[1]), magic2), h23 = f2_sub(f2_bits(e[2], e[3]), magic2);
                acc[q][j][0] = f2_fma(h01, f2_mul(D1[q][0], DX), f2_fma(f01, f2_mul(D0[q][0], DX), acc[q][j][0]));
                acc[q][j][1] = f2_fma(h23, f2_mul(D1[q][1], DX), f2_fma(f23, f2_mul(D0[q][1], DX), acc[q][j][1]));
              }
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // warp 0 refills this stage for iteration it + NS once all warps have released it
    if (warp == 0 && it + S::NS < n_it) {
      if (!mbar_wait(&empty[s], r & 1, a.status, kErrWaitEmpty)) break;
      issue(it + S::NS);
    }
  }
  // ---------------- epilogue: this slice's partial sums ----------------
  float* ys = a.y + static_cast<int64_t>(blockIdx.y) * a.slice;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if (pw + q >= tile_panels) break;
    const int64_t r0 = (p0 + pw + q) * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < NTW; ++j) {
      const int t = t0 + 8 * (jt0 + j) + 2 * c;
      const float v[4] = {f2_lo(acc[q][j][0]), f2_hi(acc[q][j][0]), f2_lo(acc[q][j][1]), f2_hi(acc[q][j][1])};
      const int tt[4] = {t, t + 1, t, t + 1};
      const int64_t rr[4] = {r0, r0, r1, r1};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (tt[e] < a.n && rr[e] < a.rows) ys[static_cast<int64_t>(tt[e]) * a.ldy + rr[e]] = v[e];
    }
  }
}


// ---------------- small-row regime: dp4a ----------------
// A few tokens against a deep or narrow weight give the mma tiles few CTAs (rows / 32 at most) and leave most of
// their warps without token tiles. Here a warp covers one whole panel (16 rows) x 2 tokens, one (row, token) chain
// per lane, from a shared-memory copy of the panel chunk and the token tile. Each 32-value block's integer dot comes
// from dp4a: for Q8_0 and Q6_K lane 4 g + c reads fragment slot 4 g + c (rows g, g + 8, value quarter c), takes the
// quarter's partial dots of (row g, g + 8) x (token t0, t0 + 1) and a two-step shuffle butterfly over the quad
// leaves lane c with entry c's whole dot; for Q4_K a lane reads its own row's four quarters and its token's 32
// values and needs no shuffle (the form measured faster per type). Integer sums are exact in any order, so each dot
// equals the mma's; the lane then runs malkin's float chain for its (row, token) over the blocks in order with the
// same roundings as k_gemm: bit-identical.
constexpr int kDpWarps = 4;  // warps per CTA: one panel x one 8-token tile

__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
  return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

// lanes c of a quad hold partial dots p0..p3 of entries 0..3; returns the quad's total of entry c
__device__ __forceinline__ int quad_take(int p0, int p1, int p2, int p3, int c) {
  const bool b0 = c & 1, b1 = (c >> 1) & 1;
  const int k0 = b0 ? p1 : p0, s0 = b0 ? p0 : p1;  // keep entry b0, send the partner's
  const int k1 = b0 ? p3 : p2, s1 = b0 ? p2 : p3;  // keep entry 2 + b0
  const int r0 = k0 + __shfl_xor_sync(0xffffffffu, s0, 1);
  const int r1 = k1 + __shfl_xor_sync(0xffffffffu, s1, 1);
  const int k = b1 ? r1 : r0, sd = b1 ? r0 : r1;  // keep entry b0 + 2 b1
  return k + __shfl_xor_sync(0xffffffffu, sd, 2);
}

// entries (row g, t0), (row g, t1), (row g + 8, t0), (row g + 8, t1) of one 16-value half: weight words wg, wg8,
// activation words x0, x1 (4 values each)
__device__ __forceinline__ int quad_dot(uint32_t wg, uint32_t wg8, uint32_t x0, uint32_t x1, int c) {
  return quad_take(__dp4a(static_cast<int>(wg), static_cast<int>(x0), 0), __dp4a(static_cast<int>(wg), static_cast<int>(x1), 0),
                   __dp4a(static_cast<int>(wg8), static_cast<int>(x0), 0), __dp4a(static_cast<int>(wg8), static_cast<int>(x1), 0), c);
}

// One stage of the dp4a ring: KU k-units of the panel's weight chunks, the token tile's activation blocks (int8
// fragments), their d (and the Q4_K min term or the Q6_K half sums); every part a multiple of 16 bytes.
template <uint32_t T>
struct DpCfg {
  using C = TypeCfg<T>;
  static constexpr int KU = T == 8 ? 8 : 2;       // k-units per stage (8 or 16 blocks of 32 values)
  static constexpr int BLK = KU * C::BPU;
  static constexpr int WB = KU * C::UNIT, XB = BLK * 256, SB = BLK * 32;
  static constexpr int EX = (C::kDsx || C::kSh) ? SB : 0;
  static constexpr int BYTES = WB + XB + SB + EX;
};
constexpr int kDpStages = 4;

template <uint32_t T>
__device__ __forceinline__ void dp_issue(const GemmArgs& a, int64_t p, int tt, int u0, uint8_t* sm) {
  using D = DpCfg<T>;
  using C = TypeCfg<T>;
  const int uk = min(D::KU, a.kunits - u0), nb = uk * C::BPU;
  const uint8_t* wsrc = a.w + (static_cast<size_t>(p) * a.kunits + u0) * C::UNIT;
  for (int i = threadIdx.x; i < uk * static_cast<int>(C::UNIT) / 16; i += blockDim.x) cp_async16(sm + 16 * i, wsrc + 16 * i);
  const int64_t b0 = static_cast<int64_t>(u0) * C::BPU, npad = static_cast<int64_t>(a.nt8) * 8;
  for (int i = threadIdx.x; i < nb * 16; i += blockDim.x) {
    const int bb = i >> 4, q = i & 15;
    cp_async16(sm + D::WB + bb * 256 + 16 * q, a.qx + ((b0 + bb) * a.nt8 + tt) * 256 + 16 * q);
  }
  for (int i = threadIdx.x; i < nb * 2; i += blockDim.x) {
    const int bb = i >> 1, q = i & 1;
    const int64_t off = (b0 + bb) * npad + tt * 8 + 4 * q;
    cp_async16(sm + D::WB + D::XB + bb * 32 + 16 * q, a.dx + off);
    if constexpr (C::kDsx) cp_async16(sm + D::WB + D::XB + D::SB + bb * 32 + 16 * q, a.dsx + off);
    if constexpr (C::kSh) cp_async16(sm + D::WB + D::XB + D::SB + bb * 32 + 16 * q, a.sh + off);
  }
  cp_async_commit();
}

// grid (panels, token tiles), block 32 kDpWarps: warp w takes tokens 8 blockIdx.y + 2 w, + 1 of the panel; the CTA
// streams the panel's chunks and the tile's activations through a kDpStages-deep cp.async ring.
template <uint32_t T>
__global__ void __launch_bounds__(32 * kDpWarps) k_gemm_dp4a(GemmArgs a) {
  using C = TypeCfg<T>;
  using D = DpCfg<T>;
  __shared__ __align__(16) uint8_t sm[kDpStages][D::BYTES];
  constexpr bool kQuad = T != 12;  // quad butterfly (Q8_0, Q6_K) or a lane's own row (Q4_K)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = kQuad ? lane >> 2 : lane & 7, c = lane & 3;
  const int h = kQuad ? c >> 1 : (lane >> 3) & 1;
  const int64_t p = blockIdx.x;
  const int tt = blockIdx.y, t0 = tt * 8 + 2 * warp;
  const bool active = t0 < a.n;    // warps past the last token still copy and wait
  const int tl = 2 * warp + (kQuad ? (c & 1) : (lane >> 4)), t = tt * 8 + tl;  // this lane's token (tile, overall)
  const int64_t row = p * 16 + g + 8 * h;
  const int nst = (a.kunits + D::KU - 1) / D::KU;
  for (int s = 0; s < kDpStages - 1; ++s) {
    if (s < nst)
      dp_issue<T>(a, p, tt, s * D::KU, sm[s]);
    else
      cp_async_commit();
  }
  float acc = 0.0f;
  for (int it = 0; it < nst; ++it) {
    cp_async_wait<kDpStages - 2>();
    __syncthreads();  // stage `it` landed for every thread; the stage of it - 1 is free
    const int nx = it + kDpStages - 1;
    if (nx < nst)
      dp_issue<T>(a, p, tt, nx * D::KU, sm[nx % kDpStages]);
    else
      cp_async_commit();
    if (!active) continue;
    const uint8_t* st = sm[it % kDpStages];
    // quad: token t0's quarter c (t0 + 1 at + 32); lane: the token's 32 bytes, (low 4, high 4) per quarter
    const uint8_t* xs = st + D::WB + (kQuad ? 8 * (4 * (2 * warp) + c) : 32 * tl);
    const float* dxs = reinterpret_cast<const float*>(st + D::WB + D::XB) + tl;
    if constexpr (T == 8) {
      const int uk = min(D::KU, a.kunits - it * D::KU);
#pragma unroll 4
      for (int uu = 0; uu < uk; ++uu) {
        const uint8_t* ch = st + uu * C::UNIT;
        const uint4 A = *reinterpret_cast<const uint4*>(ch + 16 * lane);  // (g lo, g+8 lo, g hi, g+8 hi)
        const uint2 x0 = *reinterpret_cast<const uint2*>(xs + uu * 256), x1 = *reinterpret_cast<const uint2*>(xs + uu * 256 + 32);
        const int lo = quad_dot(A.x, A.y, x0.x, x1.x, c), hi = quad_dot(A.z, A.w, x0.y, x1.y, c);
        const float dw = __half2float(*reinterpret_cast<const __half*>(ch + 512 + 4 * g + 2 * h));
        acc = __fmaf_rn(__int2float_rn(lo + hi), __fmul_rn(dw, dxs[uu * 8]), acc);
      }
    } else if constexpr (T == 12) {
      const int uk = min(D::KU, a.kunits - it * D::KU);
      for (int uu = 0; uu < uk; ++uu) {
      const uint8_t* cu = st + uu * C::UNIT;
      const uint4 H = *reinterpret_cast<const uint4*>(cu + 2048 + 32 * g + 16 * h);  // this lane's row's head
      const float d = h2f_lo(H.x), dmin = h2f_hi(H.x);
      const float* dss = reinterpret_cast<const float*>(st + D::WB + D::XB + D::SB) + tl + 64 * uu;
#pragma unroll 2
      for (int j = 0; j < 8; ++j) {
        const int bj = 8 * uu + j;  // block in the stage
        const uint4 W0 = *reinterpret_cast<const uint4*>(cu + 256 * j + 32 * g);  // slots 4g, 4g+1: (row g, row g+8)
        const uint4 W1 = *reinterpret_cast<const uint4*>(cu + 256 * j + 32 * g + 16);
        const uint32_t wv[4] = {h ? W0.y : W0.x, h ? W0.w : W0.z, h ? W1.y : W1.x, h ? W1.w : W1.z};
        const uint4 X0 = *reinterpret_cast<const uint4*>(xs + bj * 256), X1 = *reinterpret_cast<const uint4*>(xs + bj * 256 + 16);
        const uint32_t xv[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
        int dot = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dot = dp4((wv[q] >> 4) & 0x0F0F0F0Fu, xv[2 * q + 1], dp4(wv[q] & 0x0F0F0F0Fu, xv[2 * q], dot));
        int sc, m;
        q4k_scale_min(j, H.y, H.z, H.w, sc, m);
        const float scg = __fmul_rn(d, static_cast<float>(sc)), mng = __fmul_rn(dmin, static_cast<float>(m));
        acc = __fmaf_rn(-mng, dss[j * 8], __fmaf_rn(__int2float_rn(dot), __fmul_rn(scg, dxs[bj * 8]), acc));
      }
      }
    } else {  // Q6_K: two 16-value halves per block, q stored +32 (the half sums s remove the offset)
      const int uk = min(D::KU, a.kunits - it * D::KU);
      for (int uu = 0; uu < uk; ++uu) {
      const uint8_t* cu = st + uu * C::UNIT;
      const uint4 SG = *reinterpret_cast<const uint4*>(cu + 3072 + 32 * g + 16 * h);  // this row's 16 scales
      const float dd = __half2float(*reinterpret_cast<const __half*>(cu + 3328 + 4 * g + 2 * h));
      const uint32_t* shs = reinterpret_cast<const uint32_t*>(st + D::WB + D::XB + D::SB) + tl + 64 * uu;
#pragma unroll 2
      for (int j = 0; j < 8; ++j) {
        const int bj = 8 * uu + j;  // block in the stage
        const uint2 w = *reinterpret_cast<const uint2*>(cu + 256 * j + 8 * lane);
        const uint32_t hb = *reinterpret_cast<const uint32_t*>(cu + 2048 + 128 * j + 4 * lane);
        const uint2 x0 = *reinterpret_cast<const uint2*>(xs + bj * 256), x1 = *reinterpret_cast<const uint2*>(xs + bj * 256 + 32);
        const int lo = quad_dot((w.x & 0x0F0F0F0Fu) | ((hb << 4) & 0x30303030u),
                                (w.y & 0x0F0F0F0Fu) | ((hb << 2) & 0x30303030u), x0.x, x1.x, c);
        const int hi = quad_dot(((w.x >> 4) & 0x0F0F0F0Fu) | (hb & 0x30303030u),
                                ((w.y >> 4) & 0x0F0F0F0Fu) | ((hb >> 2) & 0x30303030u), x0.y, x1.y, c);
        const uint32_t sv = shs[j * 8];
        const int dot0 = lo - 32 * static_cast<int16_t>(sv & 0xFFFF), dot1 = hi - 32 * static_cast<int16_t>(sv >> 16);
        const uint32_t sw = j < 2 ? SG.x : (j < 4 ? SG.y : (j < 6 ? SG.z : SG.w));  // scales 2 j, 2 j + 1
        const float s0 = static_cast<float>(static_cast<int8_t>((sw >> (16 * (j & 1))) & 0xFF));
        const float s1 = static_cast<float>(static_cast<int8_t>((sw >> (16 * (j & 1) + 8)) & 0xFF));
        const float dx = dxs[bj * 8];
        acc = __fmaf_rn(__int2float_rn(dot1), __fmul_rn(__fmul_rn(dd, s1), dx),
                        __fmaf_rn(__int2float_rn(dot0), __fmul_rn(__fmul_rn(dd, s0), dx), acc));
      }
      }
    }
  }
  cp_async_wait<0>();
  if (active && t < a.n && row < a.rows) a.y[static_cast<int64_t>(t) * a.ldy + row] = acc;
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


using GemmFn = void (*)(GemmArgs);

// Kernel variants: WP = 8 (16-panel tiles) with NTW = 1..18 token tiles per warp; WP = 2 (4 panels, 4 warps along the
// tokens) with NTW = 1..4; WP = 1 (2 panels, 8 warps along the tokens) with NTW = 1..3.
struct Variant {
  GemmFn fn;
  uint32_t smem;
  int wp, ntw;
};
// WP = 8 (16-panel tiles): NTW 1..18, default stage depth. WP = 4 (8 panels): NTW 4..9; WP = 2 (4 panels): NTW 2..5;
// WP = 1 (2 panels): NTW 1..3; the narrow Q8_0 tiles with 8 blocks per stage.
constexpr int kVariants = kMaxNT + 6 + 4 + 3;

template <uint32_t T>
constexpr int narrow_ks() {
  return T == 8 ? 8 : 0;  // K-quant stages already hold 8 blocks (one super-block)
}

template <uint32_t T, int WP, int N0, int KSX, int... N>
constexpr void fill(Variant* v, std::integer_sequence<int, N...>) {
  ((v[N] = Variant{&k_gemm<T, N + N0, WP, KSX>, Stage<T, (kConsumers / WP) * (N + N0), 2 * WP, KSX>::SMEM, WP,
                   N + N0}),
   ...);
}

template <uint32_t T>
constexpr std::array<Variant, kVariants> variants() {
  std::array<Variant, kVariants> v{};
  fill<T, 8, 1, 0>(v.data(), std::make_integer_sequence<int, kMaxNT>{});
  fill<T, 4, 4, narrow_ks<T>()>(v.data() + kMaxNT, std::make_integer_sequence<int, 6>{});
  fill<T, 2, 2, narrow_ks<T>()>(v.data() + kMaxNT + 6, std::make_integer_sequence<int, 4>{});
  fill<T, 1, 1, narrow_ks<T>()>(v.data() + kMaxNT + 10, std::make_integer_sequence<int, 3>{});
  return v;
}

template <uint32_t T>
const std::array<Variant, kVariants>& variant_table() {
  static constexpr auto v = variants<T>();
  return v;
}

const std::array<Variant, kVariants>& table_of(uint32_t type) {
  return type == 12 ? variant_table<12>() : (type == 14 ? variant_table<14>() : variant_table<8>());
}

struct DevInfo {
  int sms = 148;
  int occ[3][kVariants] = {};  // resident CTAs per SM of each variant (0 = not yet queried)
  bool attr[3][kVariants] = {};
};

DevInfo& dev_info(int dev) {
  static DevInfo info[kMaxDevices];
  static bool init[kMaxDevices] = {};
  DevInfo& d = info[dev < kMaxDevices ? dev : 0];
  if (!init[dev < kMaxDevices ? dev : 0]) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    init[dev < kMaxDevices ? dev : 0] = true;
  }
  return d;
}

int type_index(uint32_t type) { return type == 12 ? 1 : (type == 14 ? 2 : 0); }

// Prepares variant i on the current device (shared-memory opt-in) and returns its residency.
int prepare(uint32_t type, int i) {
  int dev = 0;
  cudaGetDevice(&dev);
  DevInfo& d = dev_info(dev);
  const int ti = type_index(type);
  const Variant& v = table_of(type)[i];
  if (!d.attr[ti][i]) {
    cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(v.smem));
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, v.fn, kThreadsG, v.smem) != cudaSuccess) {
      cudaGetLastError();
      occ = 1;
    }
    d.occ[ti][i] = occ > 0 ? occ : 1;
    d.attr[ti][i] = true;
  }
  return d.occ[ti][i];
}

struct Plan {
  int variant = 0, passes = 1;
};
constexpr int kDp4a = kVariants;       // plan value of the dp4a kernel (k_gemm_dp4a)
constexpr int kDp4aMaxTiles = 4;       // token tiles (of 8) up to which the tuner times it

// The kernel shape for a weight, n tokens (tiles of 8, at most nt8 readable) and split-K slices. With one slice the
// SMs are filled by token passes and narrow tiles instead: the estimate is the busiest SM's share of the per-block
// float work (the bound of these kernels) plus the L2 re-reads the passes and narrow tiles cost.
Plan plan_for(const DevWeight& w, int n, int nt8, int split) {
  const int tiles = (n + 7) / 8;
  const auto& tab = table_of(w.type);
  Plan best;
  if (split > 1) {  // K slices fill the SMs: the widest tile, every token in as few passes as possible
    const int passes = (tiles + kMaxNT - 1) / kMaxNT;
    best.variant = (passes == 1 ? tiles : kMaxNT) - 1;
    best.passes = passes;
    return best;
  }
  // MALKIN_B200_GEMM_PLAN=<wp>:<ntw> (or dp4a) forces one kernel shape (tests and measurements), when it is valid here
  if (const char* e = std::getenv("MALKIN_B200_GEMM_PLAN")) {
    if (std::string(e) == "dp4a") return Plan{kDp4a, 1};
    int wp = 0, ntw = 0;
    if (std::sscanf(e, "%d:%d", &wp, &ntw) == 2)
      for (int i = 0; i < kVariants; ++i)
        if (tab[i].wp == wp && tab[i].ntw == ntw) {
          const int nt = (kConsumers / wp) * ntw;
          return Plan{i, (tiles + nt - 1) / nt};
        }
  }
  // the measured shape (gemm_tune)
  if (const int ch = gemm_choice(w, n); ch == kDp4a) return Plan{kDp4a, 1};
  if (const int ch = gemm_choice(w, n); ch >= 0 && ch < kVariants) {
    const int nt = (kConsumers / tab[ch].wp) * tab[ch].ntw;
    return Plan{ch, (tiles + nt - 1) / nt};
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = dev_info(dev).sms;
  const double blocks = static_cast<double>(w.kunits) * (w.type == 8 ? 1 : 8);  // 32-value blocks per row
  const double wbytes = static_cast<double>(w.panels) * 16 * w.kunits * (w.type == 8 ? 34 : (w.type == 12 ? 144 : 210));
  const double abytes_tile = blocks * 8 * 36;  // one token tile's activations (int8 + scale), all blocks
  double best_t = 1e30;
  for (int i = 0; i < kVariants; ++i) {
    const Variant& v = tab[i];
    const int nt = (kConsumers / v.wp) * v.ntw;  // token tiles per CTA
    if (nt > 2 * tiles + 1 && i != 0) continue;  // far more token columns than tokens
    const int passes = (tiles + nt - 1) / nt;
    const int64_t rtiles = (w.panels + 2 * v.wp - 1) / (2 * v.wp);
    const int64_t ctas = rtiles * passes;
    const int occ = prepare(w.type, i);
    // per-SM float work: CTAs round-robin over SMs, `occ` of them share an SM at a time
    const double per_sm_ctas = std::ceil(static_cast<double>(ctas) / sms);
    const double work = per_sm_ctas * (2.0 * v.wp * 16) * (nt * 8.0) * blocks;  // element-blocks on the busiest SM
    const double t_fp = work * 3.0 / (128.0 * 1.9e9);                          // 3 FP32 ops per element-block
    const double l2 = wbytes * passes + abytes_tile * tiles * rtiles;          // bytes through L2
    const double t_l2 = l2 / 18e12;
    const double t = std::max(t_fp, t_l2) + (occ > 1 ? 0.0 : 0.2e-6 * per_sm_ctas);
    if (t < best_t * 0.98) best_t = t, best.variant = i, best.passes = passes;
  }
  return best;
}

// ---- kernel-shape tuning ----
using TuneKey = std::tuple<int, uint32_t, int, int64_t, int, int>;  // device, type, layout, rows, k units, tiles
std::mutex g_tune_mu;
std::map<TuneKey, int> g_tuned;
thread_local int g_force = -1;
constexpr size_t kFlushBytes = size_t{256} << 20;  // > L2 (126 MB)

TuneKey tune_key(const DevWeight& w, int n) {
  int dev = 0;
  cudaGetDevice(&dev);
  return TuneKey{dev, w.type, w.layout, w.rows, w.kunits, (n + 7) / 8};
}

void* flush_buffer(int dev) {
  static void* buf[kMaxDevices] = {};
  static bool tried[kMaxDevices] = {};
  if (dev >= kMaxDevices) return nullptr;
  if (!tried[dev]) {
    tried[dev] = true;
    if (cudaMalloc(&buf[dev], kFlushBytes) != cudaSuccess) {
      cudaGetLastError();
      buf[dev] = nullptr;
    }
  }
  return buf[dev];
}

}  // namespace

int gemm_choice(const DevWeight& w, int n) {
  if (g_force >= 0) return g_force;
  std::lock_guard<std::mutex> lk(g_tune_mu);
  const auto it = g_tuned.find(tune_key(w, n));
  return it == g_tuned.end() ? -1 : it->second;
}

void gemm_tune(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int* status, cudaStream_t s) {
  static const bool off = [] {
    const char* e = std::getenv("MALKIN_B200_GEMM_TUNE");
    return e && std::string(e) == "0";
  }();
  if (off || n <= 0 || w.rows <= 0 || w.kunits <= 0) return;
  if (w.layout != kLayoutTc && w.type != 8 && w.type != 12 && w.type != 14) return;
  if (gemm_choice(w, n) >= 0) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  const int tiles = (n + 7) / 8;
  std::vector<int> cand;
  if (w.layout == kLayoutTc) {  // pass sizes: multiples of 16 up to the one that covers n at once
    const int npad = act.nt8 * 8;
    for (int N = 16; N <= gemm_tc_max_tokens() && N < n + 16; N += 16)
      if (static_cast<int64_t>((n + N - 1) / N) * N <= npad) cand.push_back(N);
  } else {  // panel variants with at most about twice the token columns needed
    const auto& tab = table_of(w.type);
    for (int i = 0; i < kVariants; ++i)
      if ((kConsumers / tab[i].wp) * tab[i].ntw <= std::max(8, 2 * tiles + 1)) cand.push_back(i);
    if (tiles <= kDp4aMaxTiles) cand.push_back(kDp4a);
  }
  if (cand.empty()) return;
  const TuneKey key = tune_key(w, n);
  if (cand.size() == 1) {
    std::lock_guard<std::mutex> lk(g_tune_mu);
    g_tuned[key] = cand[0];
    return;
  }
  void* flush = flush_buffer(std::get<0>(key));
  constexpr int kReps = 2;
  const size_t C = cand.size();
  std::vector<cudaEvent_t> ev(2 * C * kReps, nullptr);
  bool ok = true;
  for (auto& e : ev) ok = ok && cudaEventCreate(&e) == cudaSuccess;
  for (int r = 0; r < kReps && ok; ++r)
    for (size_t c = 0; c < C && ok; ++c) {
      if (flush) ok = cudaMemsetAsync(flush, r + 1, kFlushBytes, s) == cudaSuccess;
      g_force = cand[c];
      ok = ok && cudaEventRecord(ev[2 * (r * C + c)], s) == cudaSuccess;
      launch_gemm(w, act, n, y, ldy, 0, 1, status, s);
      ok = ok && cudaGetLastError() == cudaSuccess;
      ok = ok && cudaEventRecord(ev[2 * (r * C + c) + 1], s) == cudaSuccess;
      g_force = -1;
    }
  ok = ok && cudaStreamSynchronize(s) == cudaSuccess;
  int best = -1;
  float best_ms = 0.0f;
  for (size_t c = 0; c < C && ok; ++c) {
    float t = 0.0f;
    for (int r = 0; r < kReps; ++r) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, ev[2 * (r * C + c)], ev[2 * (r * C + c) + 1]) != cudaSuccess) ok = false;
      t = r == 0 ? ms : std::min(t, ms);
    }
    if (best < 0 || t < best_ms) best = cand[c], best_ms = t;
  }
  for (auto& e : ev)
    if (e) cudaEventDestroy(e);
  if (!ok) {
    cudaGetLastError();
    return;
  }
  std::lock_guard<std::mutex> lk(g_tune_mu);
  g_tuned[key] = best;
}

// Split-K is never chosen automatically: token passes and narrow tiles fill the SMs (plan_for) and keep every
// (row, token) sum in malkin's block order, so results are bit-identical to its compact panel kernels. An explicit
// split (mk_matmul's split_k > 1) still runs, with per-slice sums added in slice order.
int gemm_split_for(const DevWeight& w, int num_sms) {
  (void)w;
  (void)num_sms;
  return 1;
}

int gemm_slices(const DevWeight& w, int split) {
  if (w.layout == kLayoutTc) return gemm_tc_slices(w, split);
  split = std::max(1, std::min(split, w.kunits));
  const int per = (w.kunits + split - 1) / split;
  return (w.kunits + per - 1) / per;
}

void launch_gemm(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                 int* status, cudaStream_t s) {
  if (n <= 0) return;
  if (w.layout == kLayoutRows) {
    if (!act.xf) throw std::runtime_error("gemm: F32 / F16 / BF16 weights need the float activations");
    launch_gemm_rows(w, act, n, y, ldy, s);  // one slice: the row path has no split
    return;
  }
  if (w.layout == kLayoutTc) {
    launch_gemm_tc(w, act, n, y, ldy, slice, split, nullptr, status, s);
    return;
  }
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
  a.slice = slice;
  a.n = n;
  a.status = status;
  if (w.type != 8 && w.type != 12 && w.type != 14) return;
  const Plan pl = plan_for(w, n, act.nt8, gy);
  if (pl.variant == kDp4a && gy == 1) {
    const dim3 grid(static_cast<unsigned>(w.panels), static_cast<unsigned>((n + 7) / 8));
    switch (w.type) {
      case 8: k_gemm_dp4a<8><<<grid, 32 * kDpWarps, 0, s>>>(a); break;
      case 12: k_gemm_dp4a<12><<<grid, 32 * kDpWarps, 0, s>>>(a); break;
      default: k_gemm_dp4a<14><<<grid, 32 * kDpWarps, 0, s>>>(a); break;
    }
    return;
  }
  const Variant& v = table_of(w.type)[pl.variant];
  prepare(w.type, pl.variant);
  const dim3 grid(static_cast<unsigned>(pl.passes), static_cast<unsigned>(gy),
                  static_cast<unsigned>((w.panels + 2 * v.wp - 1) / (2 * v.wp)));
  v.fn<<<grid, kThreadsG, v.smem, s>>>(a);
}

void launch_block_dots(const DevWeight& w, const ActQ& act, int n, int32_t* out, int* status, cudaStream_t s) {
  if (w.layout == kLayoutTc) {
    launch_gemm_tc(w, act, n, nullptr, 0, 0, 1, out, status, s);
    return;
  }
  k_block_dots<<<static_cast<unsigned>(w.panels), 32, 0, s>>>(w.type, w.data, w.panels, w.kunits, w.rows, act, n, out);
}

}  // namespace mkb
