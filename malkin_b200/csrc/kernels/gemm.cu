// Quantized weight-streaming GEMM: y[t][r] = sum over blocks of float(int8 block dot) * (weight scale * act scale),
// the arithmetic of malkin's panel kernels k_q8_0 / k_q45_k / k_q6_k (gemm_avx512.cpp:67-205), on B200.
//
// Pipeline: a CTA owns a tile of 16 panels (256 weight rows) and one k-range (split-K slice). Warp 0 streams the
// tile's weight chunks and the matching activation blocks (Q8 fragments, scales) from HBM / L2 into a 2-3 stage
// shared-memory ring with TMA bulk copies (cp.async.bulk, completion counted on mbarriers) and refills a stage as
// soon as all eight warps have released it; every warp takes 2 panels x all tokens of the pass. Every weight byte
// is read from HBM once and every activation byte once per CTA.
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
#include <cstdlib>
#include <string>
#include <array>
#include <utility>

#include "common.cuh"
#include "kernels.hpp"
#include "pipeline.cuh"

namespace mkb {

namespace {

constexpr int kTilePanels = 16;
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

// Shared-memory layout of one stage.
template <uint32_t T, int NT>
struct Stage {
  using C = TypeCfg<T>;
  static constexpr uint32_t A = kTilePanels * C::KS * C::UNIT;
  static constexpr uint32_t B = C::KS * C::BPU * NT * 256;
  static constexpr uint32_t DX = C::KS * C::BPU * NT * 8 * 4;
  static constexpr uint32_t EX = (C::kDsx || C::kSh) ? DX : 0;
  static constexpr uint32_t BYTES = A + B + DX + EX;
  static constexpr uint32_t SMEM = C::NS * BYTES + 2 * C::NS * 8;
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

template <uint32_t T, int NT>
__global__ void __launch_bounds__(kThreadsG, 1) k_gemm(GemmArgs a) {
  using C = TypeCfg<T>;
  using S = Stage<T, NT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::NS * S::BYTES);
  uint64_t* empty = full + C::NS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kTilePanels;
  const int tile_panels = static_cast<int>(a.panels - p0 < kTilePanels ? a.panels - p0 : kTilePanels);
  const int u0 = blockIdx.y * a.per_split, u1 = min(a.kunits, u0 + a.per_split);
  const int t0 = blockIdx.z * (kMaxNT * 8);  // first token of this pass
  const int npad = a.nt8 * 8;
  const int n_it = (u1 - u0 + C::KS - 1) / C::KS;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    mbar_fence_init();
  }
  __syncthreads();

  // Stage refill, issued by warp 0: lane 0 arms the full barrier with the byte count, lanes 0-15 copy the tile's
  // weight chunks (one per panel), lanes 16-23 the activation blocks, dx (and dsx / sh) of each 32-value block.
  auto issue = [&](int it) {
    const int s = it % C::NS;
    const int ua = u0 + it * C::KS, uk = min(C::KS, u1 - ua);  // units in this stage
    const int nb = uk * C::BPU;                                // 32-value blocks in this stage
    const uint32_t bytes = static_cast<uint32_t>(tile_panels) * uk * C::UNIT +
                           static_cast<uint32_t>(nb) * NT * (256 + 32 + ((C::kDsx || C::kSh) ? 32 : 0));
    uint8_t* st = smem + static_cast<size_t>(s) * S::BYTES;
    if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
    __syncwarp();
    if (lane < tile_panels)
      bulk_g2s(st + lane * (C::KS * C::UNIT), a.w + (static_cast<size_t>(p0 + lane) * a.kunits + ua) * C::UNIT,
               uk * C::UNIT, &full[s]);
    const int blk0 = ua * C::BPU;
    if (lane >= 16 && lane - 16 < nb) {
      const int b = lane - 16;
      bulk_g2s(st + S::A + b * NT * 256, a.qx + (static_cast<size_t>(blk0 + b) * a.nt8 + t0 / 8) * 256, NT * 256,
               &full[s]);
      bulk_g2s(st + S::A + S::B + b * NT * 32, a.dx + static_cast<size_t>(blk0 + b) * npad + t0, NT * 32, &full[s]);
      if (C::kDsx)
        bulk_g2s(st + S::A + S::B + S::DX + b * NT * 32, a.dsx + static_cast<size_t>(blk0 + b) * npad + t0, NT * 32,
                 &full[s]);
      if (C::kSh)
        bulk_g2s(st + S::A + S::B + S::DX + b * NT * 32, a.sh + static_cast<size_t>(blk0 + b) * npad + t0, NT * 32,
                 &full[s]);
    }
  };
  if (warp == 0)
    for (int it = 0; it < C::NS && it < n_it; ++it) issue(it);

  // ---------------- consumers: warp owns panels 2w, 2w+1 of the tile ----------------
  const int pw = 2 * warp;
  const bool has0 = pw < tile_panels, has1 = pw + 1 < tile_panels;
  const f2 magic2 = f2_make(kMagicF, kMagicF);
  f2 acc[2][NT][2];
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[q][j][0] = acc[q][j][1] = f2_make(0.0f, 0.0f);

  for (int it = 0; it < n_it; ++it) {
    const int s = it % C::NS, r = it / C::NS;
    if (!mbar_wait(&full[s], r & 1, a.status, kErrWaitFull)) break;
    const uint8_t* st = smem + static_cast<size_t>(s) * S::BYTES;
    const int uk = min(C::KS, u1 - (u0 + it * C::KS));
    if (has0) {
      const uint8_t* sa0 = st + pw * (C::KS * C::UNIT);
      const uint8_t* sa1 = sa0 + C::KS * C::UNIT;
      const uint8_t* sb = st + S::A + lane * 8;
      const float* sdx = reinterpret_cast<const float*>(st + S::A + S::B) + 2 * c;
      const float* sex = reinterpret_cast<const float*>(st + S::A + S::B + S::DX) + 2 * c;
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
          for (int j = 0; j < NT; ++j) {
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
            for (int j = 0; j < NT; ++j) {
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
            for (int j = 0; j < NT; ++j) {
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
    if (warp == 0 && it + C::NS < n_it) {
      if (!mbar_wait(&empty[s], r & 1, a.status, kErrWaitEmpty)) break;
      issue(it + C::NS);
    }
  }
  // ---------------- epilogue: this slice's partial sums ----------------
  float* ys = a.y + static_cast<int64_t>(blockIdx.y) * a.slice;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    if (pw + q >= tile_panels) break;
    const int64_t r0 = (p0 + pw + q) * 16 + g, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int t = t0 + 8 * j + 2 * c;
      const float v[4] = {f2_lo(acc[q][j][0]), f2_hi(acc[q][j][0]), f2_lo(acc[q][j][1]), f2_hi(acc[q][j][1])};
      const int tt[4] = {t, t + 1, t, t + 1};
      const int64_t rr[4] = {r0, r0, r1, r1};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (tt[e] < a.n && rr[e] < a.rows) ys[static_cast<int64_t>(tt[e]) * a.ldy + rr[e]] = v[e];
    }
  }
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

template <uint32_t T, int... N>
constexpr std::array<GemmFn, sizeof...(N)> table(std::integer_sequence<int, N...>) {
  return {&k_gemm<T, N + 1>...};
}

template <uint32_t T, int... N>
constexpr std::array<uint32_t, sizeof...(N)> smem_table(std::integer_sequence<int, N...>) {
  return {Stage<T, N + 1>::SMEM...};
}

template <uint32_t T>
void launch_t(const GemmArgs& a, dim3 grid, int nt, cudaStream_t s) {
  static constexpr auto fns = table<T>(std::make_integer_sequence<int, kMaxNT>{});
  static constexpr auto sm = smem_table<T>(std::make_integer_sequence<int, kMaxNT>{});
  // per device: the attribute is a property of the device context
  static bool attr[64][kMaxNT] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev][nt - 1]) {
    cudaFuncSetAttribute(fns[nt - 1], cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm[nt - 1]));
    attr[dev][nt - 1] = true;
  }
  fns[nt - 1]<<<grid, kThreadsG, sm[nt - 1], s>>>(a);
}

}  // namespace

int q8_mode() {
  const char* e = std::getenv("MALKIN_B200_Q8_GEMM");
  if (e && std::string(e) == "fp16") return kQ8Fp16;
  if (e && std::string(e) == "split") return kQ8Split;
  return kQ8Exact;
}

int gemm_split_for(const DevWeight& w, int num_sms) {
  if (w.layout == kLayoutTc) return q8_mode() == kQ8Split ? gemm_x3_split_for(w, num_sms) : gemm_tc_split_for(w, num_sms);
  const int64_t tiles = (w.panels + kTilePanels - 1) / kTilePanels;
  const int max_split = std::max(1, w.kunits / (w.type == 8 ? 8 : 1));
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= std::min(16, max_split); ++s) {
    const int per = (w.kunits + s - 1) / s;
    const int real = (w.kunits + per - 1) / per;
    const int64_t ctas = tiles * real;
    const double eff = static_cast<double>(ctas) / (static_cast<double>((ctas + num_sms - 1) / num_sms) * num_sms);
    if (eff >= 0.85) return real;
    if (eff > best_eff + 1e-9) best_eff = eff, best = real;
  }
  return best;
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
  if (w.layout == kLayoutTc) {
    if (act.q8 == kQ8Split)
      launch_gemm_x3(w, act, n, y, ldy, slice, split, status, s);
    else if (act.q8 == kQ8Fp16)
      launch_gemm_f16(w, act, n, y, ldy, slice, split, status, s);
    else
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
  const int tiles = (n + 7) / 8;
  const int passes = (tiles + kMaxNT - 1) / kMaxNT;
  const int nt = passes == 1 ? tiles : kMaxNT;  // full passes; the last pass reads zero-padded tiles
  const dim3 grid(static_cast<unsigned>((w.panels + kTilePanels - 1) / kTilePanels), static_cast<unsigned>(gy),
                  static_cast<unsigned>(passes));
  switch (w.type) {
    case 8:
      launch_t<8>(a, grid, nt, s);
      break;
    case 12:
      launch_t<12>(a, grid, nt, s);
      break;
    case 14:
      launch_t<14>(a, grid, nt, s);
      break;
    default:
      break;
  }
}

void launch_block_dots(const DevWeight& w, const ActQ& act, int n, int32_t* out, int* status, cudaStream_t s) {
  if (w.layout == kLayoutTc) {
    launch_gemm_tc(w, act, n, nullptr, 0, 0, 1, out, status, s);
    return;
  }
  k_block_dots<<<static_cast<unsigned>(w.panels), 32, 0, s>>>(w.type, w.data, w.panels, w.kunits, w.rows, act, n, out);
}

}  // namespace mkb
