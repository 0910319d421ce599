// Q8_0 weight-streaming GEMM on tcgen05 with fp16 operands (kind::f16, A operand in TMEM, fp32 accumulator in TMEM).
//
// y[t][r] = sum_k fp16(q_w[r][k] * d_w[r][blk]) * fp16(q_x[t][k] * d_x[t][blk]): the dequantized form of malkin's
// Q8_0 x Q8 product (gemm_avx512.cpp:67-102 computes sum_blk d_w d_x dot_blk). The tensor core accumulates every
// block of the CTA's K range in fp32, so the per-block scales cost one fp16 rounding of each operand (relative error
// <= 2^-11 per product) instead of a (row, token, block) epilogue; the block dots themselves stay exact in the int8
// kernel (gemm_tc.cu), which the exact mode and the block-dot entry point use.
//
// Warps (320 threads, one CTA per SM; a CTA = 128 weight rows x N <= 256 tokens x a K range):
//   0     producer: TMA bulk copies of the fp16 activation blocks (the B operand, layout.hpp `xh`) into a ring
//   1     TMEM owner; lane 0 issues two MMAs (K = 16 each) per 32-value block and the commits
//   2..9  dequant: warp w serves TMEM lane quarter w % 4 (its 32 weight rows) and every other block (parity
//         (w - 2) / 4). Each thread streams its row's 34-byte blocks from HBM into registers kDqAhead blocks ahead,
//         converts them to fp16(q * d_w) and stores them into an A slot in TMEM; at the end the same warps read the
//         accumulator and write y.
// Weights never pass through shared memory; every wait is bounded and TMEM is released on every path.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <utility>

#include "common.cuh"
#include "kernels.hpp"
#include "pipeline.cuh"
#include "tcgen05.cuh"

namespace mkb {

namespace {

constexpr int kF16KB = 4;  // 32-value blocks per stage
constexpr int kF16Threads = 320;
constexpr int kF16MaxN = 256;
constexpr int kF16MaxStages = 8;
constexpr uint32_t kF16SmemBudget = 200 * 1024;
constexpr uint32_t kF16Cols = 512;
constexpr uint32_t kAccCols = 256;  // accumulator columns [0, 256); A slots after it
constexpr int kSlots = 16;          // A slots of 16 columns (128 rows x 32 fp16)
constexpr int kDqAhead = 8;         // blocks each dequant thread keeps in flight
constexpr int kErrF16AFull = 5, kErrF16AEmpty = 6, kErrF16Acc = 7;

struct F16Args {
  const uint8_t* w;  // [tile][block][kTcRecord]
  int kblocks, per_split;
  const uint16_t* xh;  // [block][npad / 8][4][8][8] fp16 (this pass's first token at offset 0)
  int npad;
  float* y;
  int64_t ldy, rows, slice;
  int n;
  int* status;
};

__host__ __device__ constexpr uint32_t f16_stage_bytes(int N) { return (kF16KB * N * 64 + 127) / 128 * 128; }
__host__ __device__ constexpr int f16_stages(int N) {
  return kF16SmemBudget / f16_stage_bytes(N) < kF16MaxStages ? static_cast<int>(kF16SmemBudget / f16_stage_bytes(N))
                                                              : kF16MaxStages;
}
__host__ __device__ constexpr uint32_t f16_smem(int N) { return f16_stages(N) * f16_stage_bytes(N) + 512; }

// Four int8 values (one word) -> two fp16x2 of q * d: the bytes become fp16 1152 + q exactly (0x6400 | (q + 128)),
// one subtraction recovers q, one multiplication rounds q * d once.
__device__ __forceinline__ void q8x4_to_h2(uint32_t w, __half2 d2, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const __half2 bias = __float2half2_rn(1152.0f);
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140), b = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 pa = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&a), bias), d2);
  const __half2 pb = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&b), bias), d2);
  lo = *reinterpret_cast<const uint32_t*>(&pa);
  hi = *reinterpret_cast<const uint32_t*>(&pb);
}

// NCH: 8-column chunks of the accumulator per epilogue thread (its half of N): N = 16 * NCH.
template <int NCH>
__global__ void __launch_bounds__(kF16Threads, 1) k_gemm_f16(F16Args a) {
  constexpr int N = 16 * NCH;
  constexpr uint32_t SB = f16_stage_bytes(N);
  constexpr int NS = f16_stages(N);
  static_assert(NS >= 2, "stage ring too small");

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + kF16MaxStages;
  uint64_t* a_full = empty + kF16MaxStages;
  uint64_t* a_empty = a_full + kSlots;
  uint64_t* acc_full = a_empty + kSlots;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int b0 = blockIdx.y * a.per_split, b1 = min(a.kblocks, b0 + a.per_split);
  const int nblk = b1 - b0;
  const int n_it = (nblk + kF16KB - 1) / kF16KB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);  // the MMA commit (only the MMAs read the B stage)
    }
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&a_full[i], 4);  // the four lane-quarter warps of the slot's parity
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, kF16Cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------- TMA producer (B operand) ----------------
    int issued = 0;
    for (int it = 0; it < n_it; ++it, ++issued) {
      const int s = it % NS;
      if (it >= NS && !mbar_wait_warp(&empty[s], ((it / NS) - 1) & 1, a.status, kErrWaitEmpty)) break;
      const int bb = b0 + it * kF16KB, kb = min(kF16KB, b1 - bb);
      uint8_t* st = smem + static_cast<size_t>(s) * SB;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(kb * N * 64));
      __syncwarp();
      if (lane < kb)
        bulk_g2s(st + lane * N * 64, a.xh + static_cast<size_t>(bb + lane) * a.npad * 32, N * 64, &full[s]);
      __syncwarp();
    }
    for (int it = issued > NS ? issued - NS : 0; it < issued; ++it)
      if (!mbar_wait_warp(&full[it % NS], (it / NS) & 1, a.status, kErrWaitFull)) break;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = umma_idesc_f16_f32(128, N);
    int i = 0;
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int s = it % NS;
      if (!mbar_wait_warp(&full[s], (it / NS) & 1, a.status, kErrWaitFull)) break;
      tc_fence_after();
      const int kb = min(kF16KB, b1 - (b0 + it * kF16KB));
      const uint32_t st = smem_addr(smem + static_cast<size_t>(s) * SB);
      for (int k = 0; k < kb; ++k, ++i) {
        const int slot = i % kSlots;
        if (!mbar_wait_warp(&a_full[slot], (i / kSlots) & 1, a.status, kErrF16AFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t at = tmem + kAccCols + slot * 16;
          const uint32_t bs = st + k * N * 64;
          // K halves of the block: A columns 0-7 / 8-15, B chunks 0-1 / 2-3 (LBO 128 B, SBO 512 B)
          tc_mma_f16_ts(tmem, at, umma_desc_kmajor(bs, 128, 512), idesc, i > 0 ? 1u : 0u);
          tc_mma_f16_ts(tmem, at + 8, umma_desc_kmajor(bs + 256, 128, 512), idesc, 1u);
          tc_commit(&a_empty[slot]);
          if (k == kb - 1) tc_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
    // the accumulator is final once every MMA issued has completed (also the drain before TMEM is released)
    if (lane == 0) tc_commit(acc_full);
    __syncwarp();
    mbar_wait_warp(acc_full, 0, a.status, kErrF16Acc);
  } else {
    // ---------------- dequant, then epilogue ----------------
    const int quarter = warp & 3, par = (warp - 2) >> 2;
    const int row = 32 * quarter + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const uint8_t* wt = a.w + static_cast<size_t>(tile) * a.kblocks * kTcRecord;
    const int off = (row >> 3) * 256 + (row & 7) * 16;
    uint4 ra[kDqAhead], rb[kDqAhead];
    uint32_t rd[kDqAhead];
    auto load = [&](int u, int i) {
      if (i < nblk) {
        const uint8_t* rec = wt + static_cast<size_t>(b0 + i) * kTcRecord;
        ra[u] = ld_stream16(rec + off);
        rb[u] = ld_stream16(rec + off + 128);
        rd[u] = static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(rec + 4096)[row]);
      }
    };
#pragma unroll
    for (int u = 0; u < kDqAhead; ++u) load(u, par + 2 * u);
    bool ok = true;
    for (int i0 = par; i0 < nblk && ok; i0 += 2 * kDqAhead) {
#pragma unroll
      for (int u = 0; u < kDqAhead; ++u) {
        const int i = i0 + 2 * u;
        if (i >= nblk) break;
        const int slot = i % kSlots, use = i / kSlots;
        const __half2 d2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(rd[u])));
        uint32_t h[16];
        q8x4_to_h2(ra[u].x, d2, h[0], h[1]);
        q8x4_to_h2(ra[u].y, d2, h[2], h[3]);
        q8x4_to_h2(ra[u].z, d2, h[4], h[5]);
        q8x4_to_h2(ra[u].w, d2, h[6], h[7]);
        q8x4_to_h2(rb[u].x, d2, h[8], h[9]);
        q8x4_to_h2(rb[u].y, d2, h[10], h[11]);
        q8x4_to_h2(rb[u].z, d2, h[12], h[13]);
        q8x4_to_h2(rb[u].w, d2, h[14], h[15]);
        load(u, i + 2 * kDqAhead);
        if (use > 0 && !mbar_wait_warp(&a_empty[slot], (use - 1) & 1, a.status, kErrF16AEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st16(tmem + lane_base + kAccCols + slot * 16, h);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[slot]);
      }
    }
    // epilogue: this thread's row x its half of the columns
    const bool acc_ok = mbar_wait_warp(acc_full, 0, a.status, kErrF16Acc);
    tc_fence_after();
    const int64_t grow = tile * kTcRows + row;
    const int c0 = par * (N / 2);
    if (acc_ok && a.y) {
      float* ys = a.y + static_cast<int64_t>(blockIdx.y) * a.slice;
      constexpr int GRP = NCH < 4 ? NCH : 4;
#pragma unroll
      for (int g0 = 0; g0 < NCH; g0 += GRP) {
        uint32_t v[GRP][8];
#pragma unroll
        for (int q = 0; q < GRP; ++q)
          if (g0 + q < NCH) tmem_ld8(tmem + lane_base + c0 + 8 * (g0 + q), v[q]);
        tmem_wait_ld();
        if (grow < a.rows) {
#pragma unroll
          for (int q = 0; q < GRP; ++q)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int t = c0 + 8 * (g0 + q) + j;
              if (g0 + q < NCH && t < a.n) ys[static_cast<int64_t>(t) * a.ldy + grow] = __uint_as_float(v[q][j]);
            }
        }
      }
    }
  }
  // every warp reaches this point on every path, so TMEM is released exactly once
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kF16Cols);
  }
}

using F16Fn = void (*)(F16Args);
template <int... I>
constexpr std::array<F16Fn, sizeof...(I)> f16_table(std::integer_sequence<int, I...>) {
  return {&k_gemm_f16<I + 1>...};
}
constexpr int kF16Variants = kF16MaxN / 16;

}  // namespace

void launch_gemm_f16(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                     int* status, cudaStream_t s) {
  if (n <= 0 || w.rows <= 0 || w.kunits <= 0) return;
  static constexpr auto fns = f16_table(std::make_integer_sequence<int, kF16Variants>{});
  static bool attr_set[kMaxDevices][kF16Variants] = {};
  const int kb = w.kunits;
  split = std::max(1, std::min(split, kb));
  const int per = (kb + split - 1) / split;
  const int gy = (kb + per - 1) / per;
  const int npad = act.nt8 * 8;
  int dev = 0;
  cudaGetDevice(&dev);
  F16Args a{};
  a.w = w.data;
  a.kblocks = kb;
  a.per_split = per;
  a.npad = npad;
  a.ldy = ldy;
  a.rows = w.rows;
  a.slice = slice;
  a.status = status;
  const dim3 grid(static_cast<unsigned>((w.rows + kTcRows - 1) / kTcRows), static_cast<unsigned>(gy));
  for (int t0 = 0; t0 < n; t0 += kF16MaxN) {
    const int N = (std::min(npad - t0, kF16MaxN) + 15) / 16 * 16;
    const int v = N / 16 - 1;
    if (dev < kMaxDevices && !attr_set[dev][v]) {
      cudaFuncSetAttribute(fns[v], cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(f16_smem(N)));
      attr_set[dev][v] = true;
    }
    F16Args ap = a;
    ap.xh = act.xh + static_cast<size_t>(t0) * 32;
    ap.y = y + static_cast<int64_t>(t0) * ldy;
    ap.n = std::min(kF16MaxN, n - t0);
    fns[v]<<<grid, kF16Threads, f16_smem(N), s>>>(ap);
  }
}

}  // namespace mkb
