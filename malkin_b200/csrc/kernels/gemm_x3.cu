// Q8_0 weight-streaming GEMM on tcgen05 with split fp16 operands (kind::f16, A in TMEM, fp32 accumulators in TMEM).
//
// y[t][r] = sum over 32-value blocks of d_w * d_x * dot(q_w, q_x): malkin's Q8_0 x Q8 product
// (gemm_avx512.cpp:67-102), evaluated as sum_k A[r][k] * B[t][k] with A = q_w * d_w and B = q_x * d_x, each
// split into two fp16 terms hi = fp16(v), lo = fp16(v - hi):
//   - weights: q_w * d_w has at most 19 significant bits (int8 times the fp16 d_w); hi keeps 11 and the remainder,
//     a multiple of ulp(d_w) below ulp(hi) / 2, fits the fp16 lo exactly whenever d_w is a normal fp16. A = hi + lo
//     is then exact; the dequantisation runs in registers from the int8 record (two half2 multiply / fma per pair).
//   - activations: the f32 product q_x * d_x (the quantizer's own rounding) split the same way keeps 22 of its
//     bits. The CTA expands them from the int8 tensor-core copy and d_x (layout.hpp `qc`, `dx`): 36 bytes per
//     token and block cross L2 instead of 128.
// Three MMAs per 16 values, A_hi B_hi + A_hi B_lo + A_lo B_hi, accumulate a work item's whole K range into one fp32
// TMEM accumulator: no per-block float epilogue, about 2^-21 relative error per product (the dropped A_lo B_lo
// term and the lo roundings) plus the fp32 accumulation. The exact int8 block dots stay in gemm_tc.cu (block-dot
// entry point, exact mode).
//
// Persistent CTAs (one per SM) walk work items = (128-row tile, K split) with stride gridDim.x, so the weight stream
// runs on across items without a per-CTA ramp, and the accumulator is double-buffered (N <= 192) so an item's
// epilogue overlaps the next item's MMAs. Warps (608 threads):
//   0      weight producer: TMA bulk copies of 4 records (layout.hpp, tile-major) per stage into a deep ring
//   1      activation producer: the int8 block (N x 32) and its N scales per stage, by cp.async (the TMA unit is
//          left to the weight stream; measured no slower than bulk copies)
//   2      TMEM owner; lane 0 issues the six MMAs (K = 16 each) of every block and the commits
//   3..10  dequant: warp w serves TMEM lane quarter w % 4 (its 32 weight rows) and every other block of a stage;
//          each thread forms hi / lo of q * d_w for its row's 32 values and stores them into an A slot in TMEM
//   11..14 epilogue: lane quarter w % 4; read a finished accumulator and write the item's y slice
//   15..18 converters: B_hi / B_lo of each block into shared memory in the UMMA K-major layout (and the fp16
//          range check: an activation beyond 65504 sets kErrFp16Range)
// Every wait is bounded (a status word records the first timeout; a role stops at its first failed wait) and TMEM
// is released on every path.
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

constexpr int kX3WRec = 4;  // weight records (32-value blocks) per weight stage
constexpr int kX3WStages = 6;
constexpr int kX3MaxRStages = 8;   // raw activation stages (int8 block + scales)
constexpr int kX3MaxCStages = 4;   // converted stages (B_hi | B_lo of one block)
constexpr int kX3Threads = 608;
constexpr int kX3WarpW = 0, kX3WarpB = 1, kX3WarpMma = 2, kX3WarpDq = 3, kX3WarpEpi = 11, kX3WarpCv = 15;
constexpr int kX3DqWarps = 8, kX3CvWarps = 4;
constexpr int kX3MaxN = 256;
constexpr uint32_t kX3SmemBudget = 224 * 1024;
constexpr uint32_t kX3Cols = 512;
constexpr int kX3MaxSlots = 8;  // A slots of 32 columns: hi K 0-15 | hi K 16-31 | lo K 0-15 | lo K 16-31
constexpr int kErrX3AFull = 8, kErrX3AEmpty = 9, kErrX3Acc = 10;
constexpr uint32_t kX3WStageBytes = kX3WRec * static_cast<uint32_t>(kTcRecord);
// Sleep between polls of a wait (ns) for warps off the MMA's critical path, so their polling does not compete for
// issue slots with the dequant and converter warps (measured within noise of polling without sleeping). The MMA
// issuer polls without sleeping.
constexpr uint32_t kX3SleepProducer = 128, kX3SleepWorker = 32, kX3SleepEpilogue = 256;

struct X3Args {
  const uint8_t* w;  // [tile][block][kTcRecord]
  int kblocks, per_split, splits, tiles;
  const uint8_t* qc;  // [block][npad / 8][2][8][16] int8 activations (this pass's first token at offset 0)
  const float* dx;    // [block][npad] (this pass's first token at offset 0)
  int npad;
  float* y;  // y[split][t][ldy]
  int64_t ldy, rows, slice;
  int n;  // valid tokens of this pass
  int* status;
};

// Geometry for N tokens: accumulator width (32-column aligned) and count, A slots, activation stages, shared memory.
__host__ __device__ constexpr uint32_t x3_accw(int N) { return (static_cast<uint32_t>(N) + 31) / 32 * 32; }
__host__ __device__ constexpr int x3_nacc(int N) { return kX3Cols - 2 * x3_accw(N) >= 4 * 32 ? 2 : 1; }
__host__ __device__ constexpr int x3_slots(int N) {
  return (kX3Cols - x3_nacc(N) * x3_accw(N)) / 32 < kX3MaxSlots
             ? static_cast<int>((kX3Cols - x3_nacc(N) * x3_accw(N)) / 32)
             : kX3MaxSlots;
}
__host__ __device__ constexpr uint32_t x3_rstage(int N) { return (static_cast<uint32_t>(N) * 36 + 127) / 128 * 128; }
__host__ __device__ constexpr uint32_t x3_cstage(int N) { return static_cast<uint32_t>(N) * 128; }
// Shared memory after the weight ring goes to at least 4 raw stages and up to 4 converted ones, then up to 8 raw.
constexpr uint32_t kX3ActBudget = kX3SmemBudget - kX3WStages * kX3WStageBytes;
__host__ __device__ constexpr int x3_cstages(int N) {
  return (kX3ActBudget - 4 * x3_rstage(N)) / x3_cstage(N) < kX3MaxCStages
             ? static_cast<int>((kX3ActBudget - 4 * x3_rstage(N)) / x3_cstage(N))
             : kX3MaxCStages;
}
__host__ __device__ constexpr int x3_rstages(int N) {
  return (kX3ActBudget - x3_cstages(N) * x3_cstage(N)) / x3_rstage(N) < kX3MaxRStages
             ? static_cast<int>((kX3ActBudget - x3_cstages(N) * x3_cstage(N)) / x3_rstage(N))
             : kX3MaxRStages;
}
__host__ __device__ constexpr uint32_t x3_smem(int N) {
  return kX3WStages * kX3WStageBytes + x3_rstages(N) * x3_rstage(N) + x3_cstages(N) * x3_cstage(N) + 1024;
}

// Sixteen int8 activations (4 words) of one token times its scale -> fp16 hi / lo of the f32 products in the UMMA
// order (hi[0..3] = values 0-7, hi[4..7] = values 8-15; lo alike). The bytes become the f32 8388608 + (q + 128)
// exactly and one subtraction recovers q; v = q * d rounds once (the quantizer's product), hi = fp16(v),
// lo = fp16(v - hi) with v - hi exact in f32. bad |= an exponent field of all ones (|v| >= 65520).
__device__ __forceinline__ void x16_split(uint4 q, float d, uint32_t (&hi)[8], uint32_t (&lo)[8], uint32_t& bad) {
  const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const float v0 = __fmul_rn(__uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7440 + 2 * p)) - 8388736.0f, d);
      const float v1 = __fmul_rn(__uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7441 + 2 * p)) - 8388736.0f, d);
      const __half2 h = __floats2half2_rn(v0, v1);
      const float2 hf = __half22float2(h);
      const __half2 l = __floats2half2_rn(__fsub_rn(v0, hf.x), __fsub_rn(v1, hf.y));
      hi[2 * i + p] = *reinterpret_cast<const uint32_t*>(&h);
      lo[2 * i + p] = *reinterpret_cast<const uint32_t*>(&l);
      bad |= ((hi[2 * i + p] & 0x7C00u) == 0x7C00u) | ((hi[2 * i + p] & 0x7C000000u) == 0x7C000000u);
    }
  }
}

// Four int8 weights (one word) times d -> fp16 hi / lo pairs (values 0,1 -> h0 / l0; values 2,3 -> h1 / l1). The
// bytes become fp16 1152 + q exactly (0x6400 | (q + 128)) and one subtraction recovers q; hi = q * d rounded once,
// lo = fma(q, d, -hi) rounded once (exact: see the header).
__device__ __forceinline__ void q8x4_split(uint32_t w, __half2 d2, uint32_t& h0, uint32_t& h1, uint32_t& l0,
                                           uint32_t& l1) {
  const uint32_t u = w ^ 0x80808080u;
  const __half2 bias = __float2half2_rn(1152.0f);
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140), b = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 qa = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  const __half2 qb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  const __half2 ha = __hmul2(qa, d2), hb = __hmul2(qb, d2);
  const __half2 la = __hfma2(qa, d2, __hneg2(ha)), lb = __hfma2(qb, d2, __hneg2(hb));
  h0 = *reinterpret_cast<const uint32_t*>(&ha);
  h1 = *reinterpret_cast<const uint32_t*>(&hb);
  l0 = *reinterpret_cast<const uint32_t*>(&la);
  l1 = *reinterpret_cast<const uint32_t*>(&lb);
}

// N = 16 * NCH tokens per launch.
template <int NCH>
__global__ void __launch_bounds__(kX3Threads, 1) k_gemm_x3(X3Args a) {
  constexpr int N = 16 * NCH;
  constexpr int NCS = x3_cstages(N), NRS = x3_rstages(N), NACC = x3_nacc(N), NSLOT = x3_slots(N);
  constexpr uint32_t ACCW = x3_accw(N), RSB = x3_rstage(N), CSB = x3_cstage(N);
  constexpr uint32_t OFF_R = kX3WStages * kX3WStageBytes, OFF_C = OFF_R + NRS * RSB,
                     OFF_BAR = OFF_C + NCS * CSB;
  static_assert(NCS >= 2 && NRS >= 4 && NSLOT >= 2, "x3 geometry");

  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* wempty = wfull + kX3WStages;
  uint64_t* rfull = wempty + kX3WStages;
  uint64_t* rempty = rfull + kX3MaxRStages;
  uint64_t* cfull = rempty + kX3MaxRStages;
  uint64_t* cempty = cfull + kX3MaxCStages;
  uint64_t* a_full = cempty + kX3MaxCStages;
  uint64_t* a_empty = a_full + kX3MaxSlots;
  uint64_t* acc_full = a_empty + kX3MaxSlots;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int items = a.tiles * a.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kX3WStages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kX3DqWarps);  // every dequant warp has read its records
    }
    for (int s = 0; s < NRS; ++s) {
      mbar_init(&rfull[s], 32);  // every producer lane's cp.async group
      mbar_init(&rempty[s], kX3CvWarps);
    }
    for (int s = 0; s < NCS; ++s) {
      mbar_init(&cfull[s], kX3CvWarps);
      mbar_init(&cempty[s], 1);  // the MMA commit
    }
    for (int i = 0; i < NSLOT; ++i) {
      mbar_init(&a_full[i], 4);  // one dequant warp per lane quarter
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // the four epilogue warps
    }
    mbar_init(mma_done, 1);
    mbar_fence_init();
  }
  if (warp == kX3WarpMma) tmem_alloc(tmem_holder, kX3Cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // item -> (tile, K range)
  auto range = [&](int item, int& tile, int& b0, int& b1) {
    tile = item / a.splits;
    b0 = (item % a.splits) * a.per_split;
    b1 = min(a.kblocks, b0 + a.per_split);
  };
  // An item's blocks run in groups of kX3WRec (one weight stage each), the groups rotated by the tile index: CTAs
  // that share a K range start at different groups instead of reading the same activation block at the same time
  // (measured neutral on B200; the fp32 accumulation order per item follows the rotation). Group g of [b0, b1)
  // starts at block group_start(g).
  auto groups = [&](int b0, int b1) { return (b1 - b0 + kX3WRec - 1) / kX3WRec; };
  auto group_start = [&](int tile, int b0, int b1, int g) { return b0 + ((g + tile) % groups(b0, b1)) * kX3WRec; };

  if (warp == kX3WarpW) {
    // ---------------- weight producer ----------------
    int n = 0;  // stages issued
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      for (int g = 0; g < groups(b0, b1); ++g, ++n) {
        const int s = n % kX3WStages, bb = group_start(tile, b0, b1, g);
        if (n >= kX3WStages &&
            !mbar_wait_warp_sleep(&wempty[s], ((n / kX3WStages) - 1) & 1, a.status, kErrWaitEmpty, kX3SleepProducer)) {
          ok = false;
          break;
        }
        const uint32_t bytes = static_cast<uint32_t>(min(kX3WRec, b1 - bb)) * static_cast<uint32_t>(kTcRecord);
        if (lane == 0) {
          mbar_arrive_expect_tx(&wfull[s], bytes);
          bulk_g2s(smem + s * kX3WStageBytes, a.w + (static_cast<size_t>(tile) * a.kblocks + bb) * kTcRecord, bytes,
                   &wfull[s]);
        }
        __syncwarp();
      }
    }
    // copies still in flight land before the CTA can exit (already complete unless a consumer gave up)
    for (int i = n > kX3WStages ? n - kX3WStages : 0; i < n; ++i)
      if (!mbar_wait_warp(&wfull[i % kX3WStages], (i / kX3WStages) & 1, a.status, kErrWaitFull)) break;
  } else if (warp == kX3WarpB) {
    // ---------------- activation producer ----------------
    // cp.async (16 bytes per lane and copy, through L1 rather than the TMA unit, which streams the weights). Each
    // lane's copies of a stage arrive on rfull when they land (cp.async.mbarrier.arrive.noinc, 32 arrivals per
    // stage).
    constexpr int CH = N * 36 / 16;  // 16-byte chunks per stage: N * 2 of int8 values, N / 4 of scales
    int n = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      for (int g = 0; g < groups(b0, b1) && ok; ++g) {
        const int bb = group_start(tile, b0, b1, g);
        for (int b = bb; b < min(b1, bb + kX3WRec); ++b, ++n) {
          const int s = n % NRS;
          if (n >= NRS &&
              !mbar_wait_warp_sleep(&rempty[s], ((n / NRS) - 1) & 1, a.status, kErrWaitEmpty, kX3SleepProducer)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_addr(smem + OFF_R + s * RSB);
          const uint8_t* q = a.qc + static_cast<size_t>(b) * a.npad * 32;
          const uint8_t* x = reinterpret_cast<const uint8_t*>(a.dx + static_cast<size_t>(b) * a.npad);
          for (int c = lane; c < CH; c += 32) {
            const uint8_t* src = c < 2 * N ? q + c * 16 : x + (c - 2 * N) * 16;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + c * 16), "l"(src) : "memory");
          }
          asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(&rfull[s])) : "memory");
        }
      }
    }
    // copies still in flight land before the CTA can exit
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kX3WarpMma) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = umma_idesc_f16_f32(128, N);
    int blk = 0, j = 0;  // blocks and items so far
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++j) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      const int buf = j % NACC;
      if (j >= NACC && !mbar_wait_lane0(&acc_empty[buf], ((j / NACC) - 1) & 1, a.status, kErrX3Acc)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * ACCW;
      const int nb = b1 - b0;
      for (int p = 0; p < nb; ++p, ++blk) {
        const int s = blk % NCS, slot = blk % NSLOT;
        if (!mbar_wait_lane0(&cfull[s], (blk / NCS) & 1, a.status, kErrWaitFull) ||
            !mbar_wait_lane0(&a_full[slot], (blk / NSLOT) & 1, a.status, kErrX3AFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t at = tmem + NACC * ACCW + slot * 32;
          // B: 8-token groups 512 B apart, K chunks of 8 values 128 B apart; K 16-31 start 256 B in
          const uint32_t bh = smem_addr(smem + OFF_C + s * CSB), bl = bh + CSB / 2;
          tc_mma_f16_ts(d, at, umma_desc_kmajor(bh, 128, 512), idesc, p > 0 ? 1u : 0u);
          tc_mma_f16_ts(d, at + 8, umma_desc_kmajor(bh + 256, 128, 512), idesc, 1u);
          tc_mma_f16_ts(d, at, umma_desc_kmajor(bl, 128, 512), idesc, 1u);
          tc_mma_f16_ts(d, at + 8, umma_desc_kmajor(bl + 256, 128, 512), idesc, 1u);
          tc_mma_f16_ts(d, at + 16, umma_desc_kmajor(bh, 128, 512), idesc, 1u);
          tc_mma_f16_ts(d, at + 24, umma_desc_kmajor(bh + 256, 128, 512), idesc, 1u);
          tc_commit(&a_empty[slot]);
          tc_commit(&cempty[s]);
          if (p == nb - 1) tc_commit(&acc_full[buf]);
        }
        __syncwarp();
      }
    }
    // every MMA issued has completed before TMEM can be released
    if (lane == 0) tc_commit(mma_done);
    __syncwarp();
    mbar_wait_warp(mma_done, 0, a.status, kErrX3Acc);
  } else if (warp < kX3WarpEpi) {
    // ---------------- dequant ----------------
    const int quarter = warp & 3, par = (warp - kX3WarpDq) >> 2;
    const int row = 32 * quarter + lane;
    const uint32_t slot_base = tmem + (static_cast<uint32_t>(32 * quarter) << 16) + NACC * ACCW;
    const int off = (row >> 3) * 256 + (row & 7) * 16;  // this row's K 0-15 in a record; K 16-31 128 B further
    int n = 0, blk = 0;  // weight stages and blocks so far
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      for (int g = 0; g < groups(b0, b1) && ok; ++g, ++n) {
        const int s = n % kX3WStages, kw = min(kX3WRec, b1 - group_start(tile, b0, b1, g));
        if (!mbar_wait_warp_sleep(&wfull[s], (n / kX3WStages) & 1, a.status, kErrWaitFull, kX3SleepWorker)) {
          ok = false;
          break;
        }
        for (int k = par; k < kw; k += 2) {
          const int i = blk + k;
          const int slot = i % NSLOT, use = i / NSLOT;
          const uint8_t* rec = smem + s * kX3WStageBytes + k * kTcRecord;
          const uint4 ra = *reinterpret_cast<const uint4*>(rec + off);
          const uint4 rb = *reinterpret_cast<const uint4*>(rec + off + 128);
          const __half2 d2 = __half2half2(reinterpret_cast<const __half*>(rec + 4096)[row]);
          uint32_t v[32];  // columns 0-15: hi, 16-31: lo
          q8x4_split(ra.x, d2, v[0], v[1], v[16], v[17]);
          q8x4_split(ra.y, d2, v[2], v[3], v[18], v[19]);
          q8x4_split(ra.z, d2, v[4], v[5], v[20], v[21]);
          q8x4_split(ra.w, d2, v[6], v[7], v[22], v[23]);
          q8x4_split(rb.x, d2, v[8], v[9], v[24], v[25]);
          q8x4_split(rb.y, d2, v[10], v[11], v[26], v[27]);
          q8x4_split(rb.z, d2, v[12], v[13], v[28], v[29]);
          q8x4_split(rb.w, d2, v[14], v[15], v[30], v[31]);
          if (use > 0 && !mbar_wait_warp_sleep(&a_empty[slot], (use - 1) & 1, a.status, kErrX3AEmpty, kX3SleepWorker)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_st32(slot_base + slot * 32, v);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[slot]);
        }
        // this stage's weight records have been read
        __syncwarp();
        if (lane == 0) mbar_arrive(&wempty[s]);
        blk += kw;
      }
    }
  } else if (warp < kX3WarpCv) {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
    int j = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, ++j) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      const int buf = j % NACC;
      if (!mbar_wait_warp_sleep(&acc_full[buf], (j / NACC) & 1, a.status, kErrX3Acc, kX3SleepEpilogue)) break;
      tc_fence_after();
      const int64_t grow = static_cast<int64_t>(tile) * kTcRows + row;
      float* ys = a.y + static_cast<int64_t>(item % a.splits) * a.slice;
      constexpr int C8 = N / 8, GRP = C8 < 6 ? C8 : 6;
#pragma unroll
      for (int g0 = 0; g0 < C8; g0 += GRP) {
        uint32_t r[GRP][8];
#pragma unroll
        for (int q = 0; q < GRP; ++q)
          if (g0 + q < C8) tmem_ld8(lane_base + buf * ACCW + 8 * (g0 + q), r[q]);
        tmem_wait_ld();
        if (grow < a.rows) {
#pragma unroll
          for (int q = 0; q < GRP; ++q)
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const int t = 8 * (g0 + q) + jj;
              if (g0 + q < C8 && t < a.n) ys[static_cast<int64_t>(t) * a.ldy + grow] = __uint_as_float(r[q][jj]);
            }
        }
      }
      // the accumulator has been read: hand it back to the MMA issuer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else {
    // ---------------- activation converters ----------------
    // A block's int8 copy is 2N chunks of 16 values (token t, K half h) at chunk index c = 16 (t / 8) + 8 h + t % 8,
    // 16 bytes each; converter warp cw takes the 32-chunk rounds r = cw, cw + 4, ... The fp16 output of chunk c goes
    // to the K-major core-matrix layout: 8-value chunk k of token t at (t / 8) * 512 + k * 128 + (t % 8) * 16, B_hi
    // then B_lo (CSB / 2 bytes further).
    const int cw = warp - kX3WarpCv;
    int n = 0;
    uint32_t bad = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
      int tile, b0, b1;
      range(item, tile, b0, b1);
      for (int p = b0; p < b1; ++p, ++n) {
        const int rs = n % NRS, cs = n % NCS;
        if (!mbar_wait_warp_sleep(&rfull[rs], (n / NRS) & 1, a.status, kErrWaitFull, kX3SleepWorker) ||
            (n >= NCS &&
             !mbar_wait_warp_sleep(&cempty[cs], ((n / NCS) - 1) & 1, a.status, kErrWaitEmpty, kX3SleepWorker))) {
          ok = false;
          break;
        }
        const uint8_t* raw = smem + OFF_R + rs * RSB;
        const float* dxs = reinterpret_cast<const float*>(raw + N * 32);
        uint8_t* cv = smem + OFF_C + cs * CSB;
        for (int r = cw; r < NCH; r += kX3CvWarps) {
          const int c = 32 * r + lane;
          const int t = (c >> 4) * 8 + (c & 7), h = (c >> 3) & 1;
          uint32_t hi[8], lo[8];
          x16_split(*reinterpret_cast<const uint4*>(raw + c * 16), dxs[t], hi, lo, bad);
          uint8_t* o = cv + (c >> 4) * 512 + (2 * h) * 128 + (c & 7) * 16;
          *reinterpret_cast<uint4*>(o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(o + 128) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
          *reinterpret_cast<uint4*>(o + CSB / 2) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(o + CSB / 2 + 128) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
        }
        // the generic-proxy stores become visible to the tensor core (async proxy) before the stage is handed over
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&rempty[rs]);
          mbar_arrive(&cfull[cs]);
        }
      }
    }
    if (__any_sync(0xffffffffu, bad != 0) && lane == 0) atomicCAS(a.status, 0, kErrFp16Range);
  }
  // every warp reaches this point on every path, so TMEM is released exactly once
  tc_fence_before();
  __syncthreads();
  if (warp == kX3WarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kX3Cols);
  }
}

using X3Fn = void (*)(X3Args);
template <int... I>
constexpr std::array<X3Fn, sizeof...(I)> x3_table(std::integer_sequence<int, I...>) {
  return {&k_gemm_x3<I + 1>...};
}
constexpr int kX3Variants = kX3MaxN / 16;

}  // namespace

// Split-K for the persistent kernel at a nominal 128-token batch: the K split s that minimises the blocks the
// busiest SM streams, ceil(tiles * s / SMs) * ceil(kblocks / s), plus the partial-sum traffic of s output slices
// (written once, read once by the consumer, at about 8 TB/s, in units of one block's MMA time, ~0.24 us).
int gemm_x3_split_for(const DevWeight& w, int num_sms) {
  const int64_t tiles = (w.rows + kTcRows - 1) / kTcRows;
  const int kb = w.kunits;
  const double slice_cost = 128.0 * static_cast<double>(w.rows) * 8.0 / 8e12 / 0.24e-6;
  int best = 1;
  double best_cost = 1e300;
  for (int s = 1; s <= std::min(16, kb); ++s) {
    const int per = (kb + s - 1) / s;
    const int real = (kb + per - 1) / per;
    if (real != s) continue;
    const int64_t items = tiles * real;
    const double cost = static_cast<double>((items + num_sms - 1) / num_sms) * per + slice_cost * real;
    if (cost < best_cost - 1e-9) best_cost = cost, best = real;
  }
  return best;
}

void launch_gemm_x3(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                    int* status, cudaStream_t s) {
  if (n <= 0 || w.rows <= 0 || w.kunits <= 0) return;
  static constexpr auto fns = x3_table(std::make_integer_sequence<int, kX3Variants>{});
  static bool attr_set[kMaxDevices][kX3Variants] = {};
  static int sms[kMaxDevices] = {};
  const int kb = w.kunits;
  split = std::max(1, std::min(split, kb));
  const int per = (kb + split - 1) / split;
  const int gy = (kb + per - 1) / per;
  const int npad = act.nt8 * 8;
  int dev = 0;
  cudaGetDevice(&dev);
  int num_sms = 148;
  if (dev < kMaxDevices) {
    if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    num_sms = sms[dev];
  }
  X3Args a{};
  a.w = w.data;
  a.kblocks = kb;
  a.per_split = per;
  a.splits = gy;
  a.tiles = static_cast<int>((w.rows + kTcRows - 1) / kTcRows);
  a.npad = npad;
  a.ldy = ldy;
  a.rows = w.rows;
  a.slice = slice;
  a.status = status;
  const int items = a.tiles * gy;
  const unsigned grid = static_cast<unsigned>(std::min(items, num_sms));
  for (int t0 = 0; t0 < n; t0 += kX3MaxN) {
    const int N = (std::min(npad - t0, kX3MaxN) + 15) / 16 * 16;
    const int v = N / 16 - 1;
    if (dev < kMaxDevices && !attr_set[dev][v]) {
      cudaFuncSetAttribute(fns[v], cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(x3_smem(N)));
      attr_set[dev][v] = true;
    }
    X3Args ap = a;
    ap.qc = act.qc + static_cast<size_t>(t0) * 32;
    ap.dx = act.dx + t0;
    ap.y = y + static_cast<int64_t>(t0) * ldy;
    ap.n = std::min(kX3MaxN, n - t0);
    fns[v]<<<grid, kX3Threads, x3_smem(N), s>>>(ap);
  }
}

}  // namespace mkb
