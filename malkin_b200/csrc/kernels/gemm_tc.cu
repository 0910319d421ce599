// Q8_0 weight-streaming GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8, accumulators in TMEM).
//
// y[t][r] = sum over 32-value blocks of float(int8 block dot) * (d_w * d_x): malkin's Q8_0 panel arithmetic
// (gemm_avx512.cpp:67-102), acc = fma(float(dot), d_w * d_x, acc) per block in block order. One tcgen05.mma
// (M = 128 weight rows, N = tokens <= 256, K = 32) computes the exact integer dots of one block for a whole tile into
// a TMEM accumulator buffer. The buffers are pre-loaded with the bits of 1.5 * 2^23 (kMagicBits) and every MMA
// accumulates onto them, so each TMEM word read back is the float 12582912 + dot exactly; the epilogue subtracts
// the bias (packed f32x2), multiplies by d_w * d_x, accumulates in registers in block order (split 1 is
// bit-identical to malkin), and writes the bias back to re-arm the buffer.
//
// Warp roles (448 threads, one CTA per SM): warp 0 issues TMA bulk copies of the weight records (tile-major,
// values already in the UMMA core-matrix order, layout.hpp), activation blocks (same order) and activation scales
// into a ring of stages; warp 1 owns TMEM (alloc / dealloc) and its lane 0 issues the MMAs and tcgen05.commit;
// warps 2-13 are the epilogue, three per TMEM lane quarter, each covering a third of the N columns of its 32 rows.
// Every wait is bounded (a status word records the first timeout); TMEM is released on every path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <array>
#include <utility>

#include "common.cuh"
#include "kernels.hpp"
#include "pipeline.cuh"
#include "tcgen05.cuh"

namespace mkb {

namespace {

constexpr int kTcKB = 4;  // 32-value blocks per stage
constexpr int kTcColGroups = 3;                 // epilogue warps per TMEM lane quarter
constexpr int kTcEpiWarps = 4 * kTcColGroups;
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;
constexpr uint32_t kTcCols = 512;  // TMEM columns allocated (the whole SM: one CTA per SM)
constexpr int kTcMaxN = 256;
constexpr int kTcMaxStages = 8;
constexpr uint32_t kTcSmemBudget = 200 * 1024;
constexpr int kErrTcAccFull = 3, kErrTcAccEmpty = 4;

struct TcArgs {
  const uint8_t* w;  // [tile][block][kTcRecord]
  int kblocks, per_split;
  const uint8_t* qc;  // [block][npad / 8][2][8][16] int8 activations (this pass's first token at offset 0)
  const float* dx;    // [block][npad]
  int npad;
  float* y;  // y[slice][t][ldy] (nullptr in dots mode)
  int64_t ldy, rows, slice;
  int n;          // valid tokens of this pass
  int32_t* dots;  // dots mode: dots[(r * dots_n + t) * kblocks + b] = exact int dot
  int dots_n;
  int* status;
};

// Stage: W kTcKB records | B kTcKB x (N x 32) | DX kTcKB x N floats.
__host__ __device__ constexpr uint32_t tc_stage_bytes(int N) {
  return (kTcKB * static_cast<uint32_t>(kTcRecord) + kTcKB * N * 32 + kTcKB * N * 4 + 127) / 128 * 128;
}
__host__ __device__ constexpr int tc_stages(int N) {
  return kTcSmemBudget / tc_stage_bytes(N) < kTcMaxStages ? static_cast<int>(kTcSmemBudget / tc_stage_bytes(N))
                                                          : kTcMaxStages;
}
__host__ __device__ constexpr uint32_t tc_smem(int N) { return tc_stages(N) * tc_stage_bytes(N) + 256; }

// N = 16 * NCH tokens per launch.
template <int NCH>
__global__ void __launch_bounds__(kTcThreads, 1) k_gemm_tc(TcArgs args) {
  constexpr int N = 16 * NCH;
  // blockIdx.z: token pass of N tokens (passes instead of split-K slices keep every (row, token) sum in malkin's
  // block order while filling the SMs); the pass sees its tokens from offset 0
  TcArgs a = args;
  {
    const int t0 = static_cast<int>(blockIdx.z) * N;
    a.qc += static_cast<size_t>(t0) * 32;
    a.dx += t0;
    if (a.y) a.y += static_cast<int64_t>(t0) * a.ldy;
    if (a.dots) a.dots += static_cast<int64_t>(t0) * a.kblocks;
    a.n = min(N, args.n - t0);
  }
  constexpr uint32_t SB = tc_stage_bytes(N);
  constexpr int NS = tc_stages(N);
  constexpr uint32_t OFF_B = kTcKB * static_cast<uint32_t>(kTcRecord), OFF_DX = OFF_B + kTcKB * N * 32;
  constexpr uint32_t BUF_STRIDE = (N + 31) / 32 * 32;
  constexpr int NBUF = kTcCols / BUF_STRIDE > 3 ? 3 : static_cast<int>(kTcCols / BUF_STRIDE);
  static_assert(NS >= 2, "stage ring too small");

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * SB);
  uint64_t* empty = full + kTcMaxStages;
  uint64_t* acc_full = empty + kTcMaxStages;
  uint64_t* acc_empty = acc_full + 4;
  uint64_t* mma_done = acc_empty + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int b0 = blockIdx.y * a.per_split, b1 = min(a.kblocks, b0 + a.per_split);
  const int n_it = (b1 - b0 + kTcKB - 1) / kTcKB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + kTcEpiWarps);  // the MMA commit + every epilogue warp
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kTcEpiWarps);
    }
    mbar_init(mma_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(tmem_holder, kTcCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    int issued = 0;
    for (int it = 0; it < n_it; ++it, ++issued) {
      const int s = it % NS;
      if (it >= NS && !mbar_wait_warp(&empty[s], ((it / NS) - 1) & 1, a.status, kErrWaitEmpty)) break;
      const int bb = b0 + it * kTcKB, kb = min(kTcKB, b1 - bb);
      uint8_t* st = smem + static_cast<size_t>(s) * SB;
      if (lane == 0)
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(kb) * (static_cast<uint32_t>(kTcRecord) + N * 36));
      __syncwarp();
      if (lane == 0)
        bulk_g2s(st, a.w + (static_cast<size_t>(tile) * a.kblocks + bb) * kTcRecord,
                 static_cast<uint32_t>(kb * kTcRecord), &full[s]);
      if (lane >= 1 && lane <= kb) {
        const int k = lane - 1;
        bulk_g2s(st + OFF_B + k * N * 32, a.qc + static_cast<size_t>(bb + k) * a.npad * 32, N * 32, &full[s]);
        bulk_g2s(st + OFF_DX + k * N * 4, a.dx + static_cast<size_t>(bb + k) * a.npad, N * 4, &full[s]);
      }
      __syncwarp();
    }
    // copies still in flight land before the CTA can exit (already complete unless a consumer gave up)
    for (int it = issued > NS ? issued - NS : 0; it < issued; ++it)
      if (!mbar_wait_warp(&full[it % NS], (it / NS) & 1, a.status, kErrWaitFull)) break;
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = umma_idesc_i8(128, N);
    int b = 0;
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int s = it % NS;
      if (!mbar_wait_warp(&full[s], (it / NS) & 1, a.status, kErrWaitFull)) break;
      tc_fence_after();
      const int kb = min(kTcKB, b1 - (b0 + it * kTcKB));
      const uint32_t st = smem_addr(smem + static_cast<size_t>(s) * SB);
      for (int k = 0; k < kb; ++k, ++b) {
        const int buf = b % NBUF;
        if (!mbar_wait_warp(&acc_empty[buf], (b / NBUF) & 1, a.status, kErrTcAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          // K-major core matrices: the two 16-byte K halves of a block 128 B apart, 8-row groups 256 B apart
          tc_mma_i8(tmem + buf * BUF_STRIDE, umma_desc_kmajor(st + k * static_cast<uint32_t>(kTcRecord), 128, 256),
                    umma_desc_kmajor(st + OFF_B + k * N * 32, 128, 256), idesc, 1u);
          tc_commit(&acc_full[buf]);
          if (k == kb - 1) tc_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
    // every MMA issued has completed before TMEM can be released
    if (lane == 0) tc_commit(mma_done);
    __syncwarp();
    mbar_wait_warp(mma_done, 0, a.status, kErrTcAccFull);
  } else {
    // ---------------- epilogue ----------------
    // 12 warps: three per TMEM lane quarter (a warp may only access the lanes of quarter warp % 4), each with a
    // third of the N columns in 8-column chunks.
    constexpr int C8 = N / 8, CPW = (C8 + kTcColGroups - 1) / kTcColGroups;
    const int quarter = warp & 3;         // TMEM lanes 32 * quarter .. + 31
    const int grp = (warp - 2) >> 2;      // column group
    const int row = 32 * quarter + lane;  // row within the tile
    const int ch0 = grp * CPW, nch = min(CPW, C8 - ch0);  // this warp's chunks (nch may be <= 0 for small N)
    const int c0 = ch0 * 8;
    const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + c0;
    // arm every accumulator buffer with the bias, then hand them to the MMA issuer
    for (int buf = 0; buf < NBUF; ++buf)
#pragma unroll
      for (int q = 0; q < CPW; ++q)
        if (q < nch) tmem_fill8(tbase + buf * BUF_STRIDE + 8 * q, kMagicBits);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int buf = 0; buf < NBUF; ++buf) mbar_arrive(&acc_empty[buf]);
    const f2 magic2 = f2_make(kMagicF, kMagicF);
    const int64_t grow = tile * kTcRows + row;
    const int nblk = b1 - b0;
    f2 acc[CPW * 4];
#pragma unroll
    for (int i = 0; i < CPW * 4; ++i) acc[i] = f2_make(0.0f, 0.0f);
    if (a.dots) {
      // exact block dots: the bits minus the bias, as integers (a test path: not pipelined, not unrolled)
      for (int b = 0; b < nblk; ++b) {
        const int buf = b % NBUF;
        if (!mbar_wait_warp(&acc_full[buf], (b / NBUF) & 1, a.status, kErrTcAccFull)) break;
        tc_fence_after();
        const uint32_t tb = tbase + buf * BUF_STRIDE;
#pragma unroll 1
        for (int q = 0; q < nch; ++q) {
          uint32_t v[8];
          tmem_ld8(tb + 8 * q, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int t = c0 + 8 * q + j;
            if (t < a.n && grow < a.rows)
              a.dots[(grow * a.dots_n + t) * a.kblocks + b0 + b] = static_cast<int32_t>(v[j]) - kMagicBits;
          }
          tmem_fill8(tb + 8 * q, kMagicBits);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&acc_empty[buf]);
          if (b % kTcKB == kTcKB - 1 || b == nblk - 1) mbar_arrive(&empty[(b / kTcKB) % NS]);
        }
      }
    } else if constexpr (CPW > 6) {
      // wide tiles (N > 144): not pipelined, TMEM loads in two groups per block (register budget)
      constexpr int GRP = (CPW + 1) / 2;
      bool ok = true;
      for (int b = 0; b < nblk && ok; ++b) {
        const int buf = b % NBUF, s = (b / kTcKB) % NS, k = b % kTcKB;
        if (!mbar_wait_warp(&acc_full[buf], (b / NBUF) & 1, a.status, kErrTcAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tbase + buf * BUF_STRIDE;
        const uint8_t* st = smem + static_cast<size_t>(s) * SB;
        const float dw =
            __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(st + k * kTcRecord + 4096)[row]));
        const f2 DW = f2_make(dw, dw);
        const float* dxs = reinterpret_cast<const float*>(st + OFF_DX + k * N * 4) + c0;
#pragma unroll
        for (int g0 = 0; g0 < CPW; g0 += GRP) {
          uint32_t v[GRP][8];
#pragma unroll
          for (int q = 0; q < GRP; ++q)
            if (g0 + q < nch) tmem_ld8(tb + 8 * (g0 + q), v[q]);
          tmem_wait_ld();
          if (g0 + GRP >= CPW) {
#pragma unroll
            for (int q = 0; q < CPW; ++q)
              if (q < nch) tmem_fill8(tb + 8 * q, kMagicBits);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
          }
#pragma unroll
          for (int q = 0; q < GRP; ++q) {
            const int ch = g0 + q;
            if (ch < nch) {
              const float4 xa = *reinterpret_cast<const float4*>(dxs + 8 * ch);
              const float4 xb = *reinterpret_cast<const float4*>(dxs + 8 * ch + 4);
              const f2 S[4] = {f2_mul(DW, f2_make(xa.x, xa.y)), f2_mul(DW, f2_make(xa.z, xa.w)),
                               f2_mul(DW, f2_make(xb.x, xb.y)), f2_mul(DW, f2_make(xb.z, xb.w))};
#pragma unroll
              for (int p = 0; p < 4; ++p)
                acc[ch * 4 + p] = f2_fma(f2_sub(f2_bits(v[q][2 * p], v[q][2 * p + 1]), magic2), S[p], acc[ch * 4 + p]);
            }
          }
        }
        __syncwarp();
        if (lane == 0 && (k == kTcKB - 1 || b == nblk - 1)) mbar_arrive(&empty[s]);
      }
    } else {
      // Software pipeline over blocks, in two halves of this warp's chunks: while the math of block b runs, the
      // TMEM loads of block b + 1 are in flight (first half during b's second half of math).
      constexpr int CA = (CPW + 1) / 2, CB = CPW - CA;
      uint32_t ra[CA][8], rb[CB > 0 ? CB : 1][8];
      // block j's TMEM contents into ra / rb (loads issued, not waited)
      auto load_a = [&](int j) {
        const uint32_t tb = tbase + (j % NBUF) * BUF_STRIDE;
#pragma unroll
        for (int q = 0; q < CA; ++q)
          if (q < nch) tmem_ld8(tb + 8 * q, ra[q]);
      };
      auto load_b = [&](int j) {
        const uint32_t tb = tbase + (j % NBUF) * BUF_STRIDE;
#pragma unroll
        for (int q = 0; q < CB; ++q)
          if (CA + q < nch) tmem_ld8(tb + 8 * (CA + q), rb[q]);
      };
      // after block j's loads have landed: re-arm its buffer with the bias and hand it back to the MMA issuer
      auto release = [&](int j) {
        const uint32_t tb = tbase + (j % NBUF) * BUF_STRIDE;
#pragma unroll
        for (int q = 0; q < CPW; ++q)
          if (q < nch) tmem_fill8(tb + 8 * q, kMagicBits);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[j % NBUF]);
      };
      auto wait_full = [&](int j) {
        const bool ok = mbar_wait_warp(&acc_full[j % NBUF], (j / NBUF) & 1, a.status, kErrTcAccFull);
        tc_fence_after();
        return ok;
      };
      // acc[q] += (float(bits) - 12582912) * (d_w * d_x) for chunk q of block j (values in regs)
      auto math = [&](const uint32_t (&v)[8], int q, const f2& DW, const float* dxs) {
        const float4 xa = *reinterpret_cast<const float4*>(dxs + 8 * q);
        const float4 xb = *reinterpret_cast<const float4*>(dxs + 8 * q + 4);
        const f2 S[4] = {f2_mul(DW, f2_make(xa.x, xa.y)), f2_mul(DW, f2_make(xa.z, xa.w)),
                         f2_mul(DW, f2_make(xb.x, xb.y)), f2_mul(DW, f2_make(xb.z, xb.w))};
        f2 f[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) f[p] = f2_sub(f2_bits(v[2 * p], v[2 * p + 1]), magic2);
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[q * 4 + p] = f2_fma(f[p], S[p], acc[q * 4 + p]);
      };
      bool ok = nblk > 0 && wait_full(0);
      if (ok) {
        load_a(0);
        load_b(0);
        tmem_wait_ld();
        release(0);
      }
      for (int b = 0; b < nblk && ok; ++b) {
        const int s = (b / kTcKB) % NS, k = b % kTcKB;
        const uint8_t* st = smem + static_cast<size_t>(s) * SB;
        const float dw =
            __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(st + k * kTcRecord + 4096)[row]));
        const f2 DW = f2_make(dw, dw);
        const float* dxs = reinterpret_cast<const float*>(st + OFF_DX + k * N * 4) + c0;
        const bool next = b + 1 < nblk;
#pragma unroll
        for (int q = 0; q < CA; ++q)
          if (q < nch) math(ra[q], q, DW, dxs);
        if (next) {
          ok = wait_full(b + 1);
          if (ok) load_a(b + 1);
        }
#pragma unroll
        for (int q = 0; q < CB; ++q)
          if (CA + q < nch) math(rb[q], CA + q, DW, dxs);
        if (next && ok) {
          load_b(b + 1);
          tmem_wait_ld();
          release(b + 1);
        }
        // this stage's scales have been read: release it to the producer after its last block
        __syncwarp();
        if (lane == 0 && (k == kTcKB - 1 || b == nblk - 1)) mbar_arrive(&empty[s]);
      }
    }
    // this slice's partial sums: the thread's row x its chunks of columns
    if (a.y && grow < a.rows) {
      float* ys = a.y + static_cast<int64_t>(blockIdx.y) * a.slice;
#pragma unroll
      for (int i = 0; i < CPW * 4; ++i) {
        const int t = c0 + 2 * i;
        if (i < nch * 4 && t < a.n) ys[static_cast<int64_t>(t) * a.ldy + grow] = f2_lo(acc[i]);
        if (i < nch * 4 && t + 1 < a.n) ys[static_cast<int64_t>(t + 1) * a.ldy + grow] = f2_hi(acc[i]);
      }
    }
  }
  // every warp reaches this point on every path, so TMEM is released exactly once
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcCols);
  }
}

using TcFn = void (*)(TcArgs);
template <int... I>
constexpr std::array<TcFn, sizeof...(I)> tc_table(std::integer_sequence<int, I...>) {
  return {&k_gemm_tc<I + 1>...};
}
constexpr int kTcVariants = kTcMaxN / 16;

int sms_of_device(int dev) {
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace

int gemm_tc_split_for(const DevWeight& w, int num_sms) {
  const int64_t tiles = (w.rows + kTcRows - 1) / kTcRows;
  const int kb = w.kunits;
  int best = 1;
  double best_eff = 0.0;
  for (int s = 1; s <= std::min(16, std::max(1, kb / 8)); ++s) {
    const int per = (kb + s - 1) / s;
    const int real = (kb + per - 1) / per;
    const int64_t ctas = tiles * real;
    const double eff = static_cast<double>(ctas) / (static_cast<double>((ctas + num_sms - 1) / num_sms) * num_sms);
    if (eff >= 0.9) return real;
    if (eff > best_eff + 1e-9) best_eff = eff, best = real;
  }
  return best;
}

// Tokens per pass (a multiple of 16, <= 256) for `tiles` 128-row tiles and n tokens at split 1: the fewest passes
// whose CTA count (tiles x passes, one CTA per SM) keeps the waves at least 85 % full, each pass re-reading the
// weight tile (from L2 when the passes of a tile run together). Passes never read past npad activation rows.
int gemm_tc_pass_tokens(int64_t tiles, int n, int npad, int num_sms) {
  const int n16 = (n + 15) / 16;
  int best = (std::min(n, kTcMaxN) + 15) / 16 * 16;
  double best_eff = 0.0;
  for (int passes = (n + kTcMaxN - 1) / kTcMaxN; passes <= n16; ++passes) {
    const int N = (n16 + passes - 1) / passes * 16;
    const int real = (n + N - 1) / N;
    if (static_cast<int64_t>(real) * N > npad) continue;
    const int64_t ctas = tiles * real;
    const double eff = static_cast<double>(ctas) / (static_cast<double>((ctas + num_sms - 1) / num_sms) * num_sms);
    if (eff >= 0.85) return N;
    if (eff > best_eff + 1e-9) best_eff = eff, best = N;
  }
  return best;
}

int gemm_tc_max_tokens() { return kTcMaxN; }

int gemm_tc_slices(const DevWeight& w, int split) {
  const int kb = w.kunits;
  split = std::max(1, std::min(split, kb));
  const int per = (kb + split - 1) / split;
  return (kb + per - 1) / per;
}

void launch_gemm_tc(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                    int32_t* dots, int* status, cudaStream_t s) {
  if (n <= 0 || w.rows <= 0 || w.kunits <= 0) return;
  static constexpr auto fns = tc_table(std::make_integer_sequence<int, kTcVariants>{});
  static bool attr_set[64][kTcVariants] = {};
  const int kb = w.kunits;
  if (dots) split = 1;
  split = std::max(1, std::min(split, kb));
  const int per = (kb + split - 1) / split;
  const int gy = (kb + per - 1) / per;
  const int npad = act.nt8 * 8;
  int dev = 0;
  cudaGetDevice(&dev);
  TcArgs a{};
  a.w = w.data;
  a.kblocks = kb;
  a.per_split = per;
  a.npad = npad;
  a.ldy = ldy;
  a.rows = w.rows;
  a.slice = slice;
  a.dots_n = n;
  a.status = status;
  // Token passes (grid.z) of N tokens: N a multiple of 16 (<= 256) chosen so tiles x slices x passes fill the SMs
  // when the K range is not split (split == 1 keeps malkin's block order for every output).
  const int64_t tiles = (w.rows + kTcRows - 1) / kTcRows;
  int N = (std::min(n, kTcMaxN) + 15) / 16 * 16;
  if (gy == 1) {
    N = gemm_tc_pass_tokens(tiles, n, npad, sms_of_device(dev));
    if (const int ch = gemm_choice(w, n); ch >= 16 && ch <= kTcMaxN && ch % 16 == 0 &&
                                          static_cast<int64_t>((n + ch - 1) / ch) * ch <= npad)
      N = ch;  // the measured pass size (gemm_tune)
    // MALKIN_B200_TC_PASS=<tokens> forces the pass size (tests and measurements), when it fits the padded rows
    if (const char* e = std::getenv("MALKIN_B200_TC_PASS")) {
      const int f = (std::atoi(e) + 15) / 16 * 16;
      if (f >= 16 && f <= kTcMaxN && static_cast<int64_t>((n + f - 1) / f) * f <= npad) N = f;
    }
  }
  const int passes = (n + N - 1) / N;
  if (static_cast<int64_t>(passes) * N > npad)  // a pass may not read past the padded activation rows
    N = (std::min(n, kTcMaxN) + 15) / 16 * 16;
  const int v = N / 16 - 1;
  if (dev < 64 && !attr_set[dev][v]) {
    cudaFuncSetAttribute(fns[v], cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(tc_smem(N)));
    attr_set[dev][v] = true;
  }
  a.qc = act.qc;
  a.dx = act.dx;
  a.y = y;
  a.n = n;
  a.dots = dots;
  const dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(gy), static_cast<unsigned>((n + N - 1) / N));
  fns[v]<<<grid, kTcThreads, tc_smem(N), s>>>(a);
}

}  // namespace mkb
