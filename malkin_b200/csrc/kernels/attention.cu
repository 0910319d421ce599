// Attention side of a decoder layer (model.cpp:369-392): q/k head RMSNorm + NeoX RoPE + int8 KV write, then
// tree-masked GQA attention over the HBM-resident int8 KV cache (Model::attention + kern::attend_gqa,
// model.cpp:204-247, kernels_avx512.cpp:229-307).
//
// Key sets (model.cpp:306-321): token t attends keys [0, n_keys[t]) of its sequence, then its extra rows anc[...]
// (tree ancestors, root first, itself last). Rows of one sequence that share the prefix form a sub-group; one
// CTA takes a (sub-group, KV head, key chunk) and scores every (row, query head) of the sub-group against the
// chunk, so each prefix key is read once per sub-group and KV head (GQA: the G query heads share it).
// Per chunk it keeps an online softmax (running max m, sum l, weighted values o); the combine kernel merges the
// chunks and the extra rows. Arithmetic: score = (q . k_int8) * (k_scale * 1/sqrt(D)); p = exp(score - max)
// with malkin's exp; out = (sum p * v_scale * v_int8) / sum p.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include <cfloat>

#include "common.cuh"
#include "kernels.hpp"
#include "quant.cuh"
#include "pipeline.cuh"

namespace mkb {

namespace {

// ---------------- q/k norm + RoPE + KV write ----------------
// grid (n, ceil((H + 2 KV) / 4)), block 128: one warp per head. D % 64 == 0, D <= 256.
template <int D>
__global__ void k_qkv_post(Slices qk, int v_n, int64_t v_col0, int64_t ldy, int n, int H, int KV,
                           const float* __restrict__ q_norm, const float* __restrict__ k_norm, float eps,
                           const float* __restrict__ rope_cs, const int32_t* __restrict__ rpos,
                           const int32_t* __restrict__ kv_at, float* __restrict__ q_out, AttnLayer L) {
  constexpr int PER = D / 32, HALF = D / 2;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (head >= H + 2 * KV) return;
  const int64_t col = static_cast<int64_t>(head) * D;
  const int ns = col >= v_col0 ? v_n : qk.n;  // GEMM slices of this head's columns, summed in slice order
  const float* src = qk.p + static_cast<size_t>(t) * ldy + col;
  float v[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) v[m] = sum_strided16(src + lane + 32 * m, ns, qk.stride);
  const bool is_q = head < H, is_k = !is_q && head < H + KV;
  if (is_q || is_k) {
    const float* w = is_q ? q_norm : k_norm;
    // malkin's 16-lane dot over the head (rmsnorm -> kern::dot_f32): chain l sums elements l + 16 k in k order;
    // element l + 32 m is this lane's v[m] (k = 2 m) for l < 16, and lane l + 16's v[m] (k = 2 m + 1)
    float ss = 0.0f;
#pragma unroll
    for (int m = 0; m < PER; ++m) {
      const float u = __shfl_down_sync(0xffffffffu, v[m], 16);
      ss = __fmaf_rn(v[m], v[m], ss);
      ss = __fmaf_rn(u, u, ss);
    }
    ss = __shfl_sync(0xffffffffu, reduce16(ss), 0);
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps)));
#pragma unroll
    for (int m = 0; m < PER; ++m) v[m] = __fmul_rn(__fmul_rn(v[m], s), w[lane + 32 * m]);
    // NeoX RoPE on pairs (i, i + D/2): lane's values m < PER/2 are the first halves of its pairs. The products and
    // sums as g++ compiles model.cpp's rope (C++ contracts a * b - c * d into fma(a, b, -(c * d))).
    const float* cs = rope_cs + static_cast<size_t>(rpos[t]) * D;  // [cos D/2][sin D/2]
#pragma unroll
    for (int m = 0; m < PER / 2; ++m) {
      const int i = lane + 32 * m;
      const float c = cs[i], sn = cs[HALF + i];
      const float x0 = v[m], x1 = v[m + PER / 2];
      v[m] = __fmaf_rn(x0, c, -__fmul_rn(x1, sn));
      v[m + PER / 2] = __fmaf_rn(x0, sn, __fmul_rn(x1, c));
    }
  }
  if (is_q) {
    float* dst = q_out + (static_cast<size_t>(t) * H + head) * D;
#pragma unroll
    for (int m = 0; m < PER; ++m) dst[lane + 32 * m] = v[m];
    return;
  }
  // quantize_i8 (quant.cpp:134-140) into the cache row kv_at[t] of this KV head.
  float amax = 0.0f;
#pragma unroll
  for (int m = 0; m < PER; ++m) amax = fmaxf(amax, fabsf(v[m]));
  amax = warp_max(amax);
  const float d = __fdiv_rn(amax, 127.0f), id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const int kvh = is_k ? head - H : head - H - KV;
  const size_t row = static_cast<size_t>(kvh) * L.n_rows + kv_at[t];
  int8_t* qd = (is_k ? L.k : L.v) + row * D;
#pragma unroll
  for (int m = 0; m < PER; ++m) qd[lane + 32 * m] = static_cast<int8_t>(__float2int_rn(__fmul_rn(v[m], id)));
  if (lane == 0) (is_k ? L.ks : L.vs)[row] = d;
}

// ---------------- tree-masked GQA attention in malkin's operation order ----------------
// malkin's attend_t / softmax_inplace (kernels_avx512.cpp:205-268) per (token t, query head h), keys j = 0 .. n-1
// (the contiguous prefix 0 .. n_keys[t] - 1, then the token's extra rows anc[anc_off[t] ..], in that order):
//   s_j  = reduce16(chains) * (k_scale_j * scale), chain l = q[l] * k_j[l], then fma(q[l + 16 i], k_j[l + 16 i], .)
//   e_j  = exp(s_j - max_j s_j)                      (malkin's exp)
//   inv  = 1 / reduce16(sums), sum l adds e_j for j = l, l + 16, ... in order
//   out  = (acc over j in order: acc = fma(e_j * v_scale_j, v_j, acc), from 0) * inv
// Every float operation is malkin's, in malkin's order, so the output is bit-identical. Four kernels:
//   k_att_scores   a thread pair per two prefix keys of a (sub-group, KV head, half of its rows): each thread holds
//                  eight of the 16 chains of both keys in registers, the query vectors come from shared memory; the
//                  scores of 128 keys are staged in shared memory, written out as whole rows of the sub-group's
//                  key-major table ST[j][slot] (slot = row * GA + head, GA = G rounded up to even), followed by
//                  the chunk's maximum of every slot (a row after the table's maxk rows per 128 keys)
//   k_att_extras   one warp per (t, h): the scores of the token's extra (ancestor) keys, as 16 chains on a half-warp
//   k_att_softmax  a thread per (slot, malkin vector lane l), the table streamed through a cp.async ring: the maximum
//                  from the chunk maxima and the extras, then the lane-striped sum over keys l, l + 16, ... in order
//                  with e_j * v_scale_j in place of s_j
//   k_att_pv       one CTA per (sub-group, KV head, 32 of the D values): a producer warp keeps key tiles of the
//                  probabilities (ST rows) and of the int8 values in flight with TMA bulk copies and converts each
//                  landed value tile to floats; the consumer warps advance the chains of two heads in one f32x2 FMA
//                  (each lane of the pair its own IEEE fma, in key order); then each row's extras.
constexpr int kQMax = 96;         // query vectors (rows x G) per sub-group
constexpr int kScoreKeys = 128;   // keys per score CTA (and per chunk maximum)
constexpr int kScoreParts = 2;    // score CTAs that split a sub-group's rows
constexpr int kSmStages = 4;      // softmax cp.async ring depth
constexpr int kSmStageFloats = 2048;  // table floats per softmax stage (8 KB)
constexpr int kPvTile = 32;       // keys per P.V stage
constexpr int kPvStages = 3;      // P.V ring depth
constexpr int kPvSliceMax = 32;   // output values per P.V CTA (fewer when the grid would leave SMs idle)
constexpr int kErrAttWait = 24;   // status code: a P.V stage never landed or was never released

struct AttArgs {
  const float* q;  // [n][H][D]
  int H, KV, G;
  float scale;
  AttnLayer L;
  AttnPlan p;
  float* out;      // [n][H][D]
};

// Slots of a sub-group's key-major probability table: row r, head g at r * GA + g; rows padded to 4 slots.
__host__ __device__ constexpr int att_ga(int G) { return (G + 1) / 2 * 2; }
__host__ __device__ constexpr int att_nqp(int rows, int G) { return (rows * att_ga(G) + 3) / 4 * 4; }
// chunk maxima rows after a table of maxk key rows
__host__ __device__ constexpr int att_nch(int maxk) { return (maxk + kScoreKeys - 1) / kScoreKeys; }
// rows of one score CTA (a part of the sub-group) and its staging tile stride (odd: 32 keys at one slot, 32 banks)
__host__ __device__ constexpr int sc_part_rows(int G) { return (kQMax / G + kScoreParts - 1) / kScoreParts; }
__host__ __device__ constexpr int sc_stride(int G) { return sc_part_rows(G) * att_ga(G) + 1; }
__host__ __device__ constexpr int sc_smem(int G, int D) {
  return (sc_part_rows(G) * G * D + kScoreKeys * sc_stride(G)) * 4;
}

__device__ __forceinline__ float i8f(int8_t v) { return static_cast<float>(v); }

// ST of (sub-group sg, KV head kvh): maxk key rows of nqp floats, then att_nch(maxk) chunk-maximum rows.
__device__ __forceinline__ float* st_of(const AttArgs& a, int sg, int kvh, int maxk, int nqp) {
  return a.p.st + a.p.st_off[sg] + static_cast<int64_t>(kvh) * (maxk + att_nch(maxk)) * nqp;
}

// grid (key chunks, n_sg x kScoreParts, KV), block 2 x kScoreKeys / KP. Thread c (0, 1) of a pair holds the chain
// pairs m = c, c + 2, c + 4, c + 6 (chains 2m, 2m + 1, one f32x2 register per step of 16 values) of KP keys, so a
// 16-byte load of the query vector feeds 2 KP packed FMAs. malkin's horizontal sum pairs chain i + 8 with i, then
// i + 4 with i, then (0 + 2, 1 + 3), then 0 + 1: in chain pairs that is m + 4 with m, m + 2 with m (both inside a
// thread), then pair 0 with pair 1 (across the thread pair) and the two lanes - the same operations in the same
// order, so the scores are malkin's.
template <int D>
constexpr int sc_kp() { return D <= 128 ? 2 : 1; }
// three CTAs per SM for D <= 128 (167 registers, no spills): measured faster than two CTAs with more registers and
// than one key per thread
template <int D>
__global__ void __launch_bounds__(2 * kScoreKeys / sc_kp<D>(), D <= 128 ? 3 : 1) k_att_scores(AttArgs a) {
  constexpr int DC = D / 16, KP = sc_kp<D>(), NTH = 2 * kScoreKeys / KP;
  extern __shared__ __align__(16) float qs[];  // [v][D] permuted per step: (c, mm, lane) at c * 8 + mm * 2 + lane
  __shared__ int64_t qrow[kQMax];              // global offset of each query vector of this part
  const int G = a.G, GA = att_ga(G);
  const int sg = blockIdx.y / kScoreParts, part = blockIdx.y % kScoreParts, kvh = blockIdx.z;
  const int t0 = a.p.sg_first[sg], nr = a.p.sg_first[sg + 1] - t0;
  const int maxk = a.p.sg_maxk[sg];
  const int j0 = blockIdx.x * kScoreKeys;
  const int pr = (nr + kScoreParts - 1) / kScoreParts;
  const int ra = part * pr, rb = min(nr, ra + pr);
  if (j0 >= maxk || ra >= rb) return;
  const int nq = (rb - ra) * G, sst = sc_stride(G);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sc = qs + sc_part_rows(G) * G * D;  // [kScoreKeys][sst]: scores of this CTA's keys at its slots
  for (int r = warp; r < rb - ra; r += NTH / 32)
    if (lane < G) qrow[r * G + lane] = (static_cast<int64_t>(t0 + ra + r) * a.H + kvh * G + lane) * D;
  __syncthreads();
  // query vectors, 4 values per load: values e .. e + 3 are pairs m, m + 1 (m even) of a 16-value step
  for (int i = threadIdx.x; i < nq * (D / 4); i += NTH) {
    const int v = i / (D / 4), e = 4 * (i % (D / 4)), m = (e & 15) >> 1;
    const float4 x = *reinterpret_cast<const float4*>(a.q + qrow[v] + e);
    float* dst = qs + v * D + (e & ~15) + (m >> 1) * 2;
    *reinterpret_cast<float2*>(dst) = make_float2(x.x, x.y);      // pair m: c = 0
    *reinterpret_cast<float2*>(dst + 8) = make_float2(x.z, x.w);  // pair m + 1: c = 1
  }
  const int pi = threadIdx.x >> 1, c = threadIdx.x & 1;
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  f2 kf[KP][DC][4];
#pragma unroll
  for (int k = 0; k < KP; ++k) {
    const int j = min(j0 + pi * KP + k, maxk - 1);  // keys past the table compute on a real row and are not stored
    const int4* kr = reinterpret_cast<const int4*>(a.L.k + (hb + j) * D);
#pragma unroll
    for (int i = 0; i < DC; ++i) {
      const int4 w = kr[i];
      const int ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int mm = 0; mm < 4; ++mm) {  // pair m = c + 2 mm: bytes 2m, 2m + 1 = half c of word mm
        const int h = ws[mm] >> (16 * c);
        kf[k][i][mm] = f2_make(i8f(static_cast<int8_t>(h & 0xFF)), i8f(static_cast<int8_t>((h >> 8) & 0xFF)));
      }
    }
  }
  const int jl = pi * KP + (KP == 2 ? c : 0);  // the key this thread finishes
  const float ksc = __fmul_rn(a.L.ks[hb + min(j0 + jl, maxk - 1)], a.scale);
  __syncthreads();
  float* srow = sc + jl * sst;
  for (int r = 0; r < rb - ra; ++r) {
    for (int g = 0; g < G; ++g) {
      const ulonglong2* qv = reinterpret_cast<const ulonglong2*>(qs + (r * G + g) * D + c * 8);
      f2 acc[KP][4];
      {
        const ulonglong2 x0 = qv[0], x1 = qv[1];
#pragma unroll
        for (int k = 0; k < KP; ++k) {
          acc[k][0] = f2_mul(x0.x, kf[k][0][0]);
          acc[k][1] = f2_mul(x0.y, kf[k][0][1]);
          acc[k][2] = f2_mul(x1.x, kf[k][0][2]);
          acc[k][3] = f2_mul(x1.y, kf[k][0][3]);
        }
      }
#pragma unroll
      for (int i = 1; i < DC; ++i) {
        const ulonglong2 x0 = qv[4 * i], x1 = qv[4 * i + 1];
#pragma unroll
        for (int k = 0; k < KP; ++k) {
          acc[k][0] = f2_fma(x0.x, kf[k][i][0], acc[k][0]);
          acc[k][1] = f2_fma(x0.y, kf[k][i][1], acc[k][1]);
          acc[k][2] = f2_fma(x1.x, kf[k][i][2], acc[k][2]);
          acc[k][3] = f2_fma(x1.y, kf[k][i][3], acc[k][3]);
        }
      }
      f2 c2[KP];  // level 2 of the tree for pair c: (pairs c+2, c+6) + (pairs c, c+4)
#pragma unroll
      for (int k = 0; k < KP; ++k) c2[k] = f2_add(f2_add(acc[k][3], acc[k][1]), f2_add(acc[k][2], acc[k][0]));
      f2 mine, other;
      if constexpr (KP == 2) {  // thread c finishes key c of the pair
        mine = c ? c2[1] : c2[0];
        other = __shfl_xor_sync(0xffffffffu, c ? c2[0] : c2[1], 1);
      } else {
        mine = c2[0];
        other = __shfl_xor_sync(0xffffffffu, c2[0], 1);
      }
      const f2 d2 = f2_add(mine, other);
      if (KP == 2 || c == 0) srow[g] = __fmul_rn(__fadd_rn(f2_lo(d2), f2_hi(d2)), ksc);
    }
    srow += GA;
  }
  __syncthreads();
  // write-out: rows j0 .. j0 + kn - 1 of the table at this part's slots, a warp per row (GA even: 8-byte pairs)
  const int nqp = att_nqp(nr, G);
  float* st = st_of(a, sg, kvh, maxk, nqp);
  const int kn = min(kScoreKeys, maxk - j0), np = (rb - ra) * GA / 2;
  for (int k = warp; k < kn; k += NTH / 32) {
    float2* dst = reinterpret_cast<float2*>(st + static_cast<int64_t>(j0 + k) * nqp + ra * GA);
    for (int q = lane; q < np; q += 32) dst[q] = make_float2(sc[k * sst + 2 * q], sc[k * sst + 2 * q + 1]);
  }
  // chunk maxima: warp w takes slots w, w + NTH / 32, ...; lane l the keys l, l + 32, ... below the row's n_keys
  float* pm = st + static_cast<int64_t>(maxk + blockIdx.x) * nqp + ra * GA;
  for (int sl = warp; sl < (rb - ra) * GA; sl += NTH / 32) {
    const int r = sl / GA, g = sl - r * GA;
    const int lim = g < G ? min(kn, a.p.n_keys[t0 + ra + r] - j0) : 0;
    float mx = -INFINITY;
    for (int k = lane; k < lim; k += 32) mx = fmaxf(mx, sc[k * sst + sl]);
    mx = warp_max(mx);
    if (lane == 0) pm[sl] = mx;
  }
}

// grid (n, ceil(H / 4)), block 128: warp w computes the extra keys' scores of (t = blockIdx.x, h = blockIdx.y * 4 + w)
// into ex[t][h][e] and their maximum into exmax[t][h]: lane l < 16 runs chain l (the lanes of malkin's vector),
// reduce16 across the half-warp.
template <int D>
__global__ void __launch_bounds__(128) k_att_extras(AttArgs a) {
  constexpr int DC = D / 16;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (h >= a.H) return;
  const int e0 = a.p.anc_off[t], ne = a.p.anc_off[t + 1] - e0;
  if (ne == 0) return;
  const size_t hb = static_cast<size_t>(h / a.G) * a.L.n_rows + a.p.kv_base[t];
  const float* qv = a.q + (static_cast<size_t>(t) * a.H + h) * D;
  float q[DC];
#pragma unroll
  for (int i = 0; i < DC; ++i) q[i] = qv[16 * i + (lane & 15)];
  float* er = a.p.ex + (static_cast<size_t>(t) * a.H + h) * a.p.ex_stride;
  float mx = -INFINITY;
  for (int e = 0; e < ne; ++e) {
    const size_t row = hb + a.p.anc[e0 + e];
    const int8_t* kr = a.L.k + row * D;
    float acc = __fmul_rn(q[0], i8f(kr[lane & 15]));
#pragma unroll
    for (int i = 1; i < DC; ++i) acc = __fmaf_rn(q[i], i8f(kr[16 * i + (lane & 15)]), acc);
    acc = reduce16(acc);
    const float sc = __fmul_rn(acc, __fmul_rn(a.L.ks[row], a.scale));
    mx = fmaxf(mx, sc);
    if (lane == 0) er[e] = sc;
  }
  if (lane == 0) a.p.exmax[static_cast<size_t>(t) * a.H + h] = mx;
}

// Stage `it` of the softmax ring: table rows it * TK .. + TK - 1 at the CTA's SG slots (16-byte copies) and their
// value scales (4-byte copies; the cache rows have no 16-byte alignment), one commit group.
template <int SG>
__device__ __forceinline__ void sm_issue(const AttArgs& a, const float* st, int nqp, int s0, int maxk, size_t hb,
                                         int it, float* tile, float* vst) {
  constexpr int TK = kSmStageFloats / SG, CPR = SG / 4;
  const int jt = it * TK;
  for (int i = threadIdx.x; i < TK * CPR; i += 16 * SG) {
    const int rr = i / CPR, cc = i - rr * CPR, j = jt + rr;
    if (j < maxk && s0 + 4 * cc < nqp) cp_async16(tile + rr * SG + 4 * cc, st + static_cast<int64_t>(j) * nqp + s0 + 4 * cc);
  }
  for (int i = threadIdx.x; i < TK; i += 16 * SG)
    if (jt + i < maxk) cp_async4(vst + i, a.L.vs + hb + jt + i);
  cp_async_commit();
}

// grid (slot groups of SG, n_sg, KV), block 16 x SG: thread (l, sl) = threadIdx.x / SG, % SG runs malkin's vector lane
// l (0..15) of slot s0 + sl. The maximum over the slot's keys (any order: the chunk maxima of the score kernel, striped
// over the lanes, and the extras' maximum), then the table streams through shared memory in a kSmStages-deep cp.async
// ring of kSmStageFloats-float tiles, and each thread walks its keys j = l, l + 16, ... in order: e_j = exp(s_j - max),
// sum += e_j, p_j = e_j * v_scale_j written in place; then the extras (keys n0 .. nk - 1 of the stripe, from ex),
// and 1 / reduce16 of the slot's 16 lane sums into inv. SG (32, 16, 8 or 4 slots per CTA) is picked per launch so
// the grid covers the SMs.
template <int SG>
__global__ void __launch_bounds__(16 * SG) k_att_softmax(AttArgs a) {
  constexpr int TK = kSmStageFloats / SG;
  __shared__ __align__(16) float tile[kSmStages][kSmStageFloats];
  __shared__ float vst[kSmStages][TK];
  __shared__ float red[16][SG + 1], rsum[16][SG + 1];
  const int sg = blockIdx.y, kvh = blockIdx.z, s0 = blockIdx.x * SG;
  const int t0 = a.p.sg_first[sg], rows = a.p.sg_first[sg + 1] - t0;
  const int maxk = a.p.sg_maxk[sg], nch = att_nch(maxk);
  const int G = a.G, ga = att_ga(G), nqp = att_nqp(rows, G);
  if (s0 >= nqp) return;
  const int l = threadIdx.x / SG, sl = threadIdx.x - l * SG, slot = s0 + sl;
  const int r = slot / ga, g = slot - r * ga;
  const bool valid = slot < nqp && r < rows && g < G;
  const int t = t0 + (valid ? r : 0), h = kvh * G + (valid ? g : 0);
  const int n0 = valid ? a.p.n_keys[t] : 0;
  const int e0 = a.p.anc_off[t], ne = valid ? a.p.anc_off[t + 1] - e0 : 0, nk = n0 + ne;
  float* st = st_of(a, sg, kvh, maxk, nqp);
  const float* pm = st + static_cast<int64_t>(maxk) * nqp;
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  const int ntiles = (maxk + TK - 1) / TK;
  for (int it = 0; it < kSmStages - 1; ++it) {
    if (it < ntiles)
      sm_issue<SG>(a, st, nqp, s0, maxk, hb, it, tile[it], vst[it]);
    else
      cp_async_commit();
  }
  float mx = l == 0 && ne > 0 ? a.p.exmax[static_cast<size_t>(t) * a.H + h] : -INFINITY;
  const int nc = valid ? min(nch, (n0 + kScoreKeys - 1) / kScoreKeys) : 0;
  for (int cc = l; cc < nc; cc += 16) mx = fmaxf(mx, pm[static_cast<int64_t>(cc) * nqp + slot]);
  red[l][sl] = mx;
  __syncthreads();
  mx = red[0][sl];
#pragma unroll
  for (int i = 1; i < 16; ++i) mx = fmaxf(mx, red[i][sl]);
  float sum = 0.0f;
  for (int it = 0; it < ntiles; ++it) {
    cp_async_wait<kSmStages - 2>();
    __syncthreads();  // tile `it` landed for every thread; the stage of tile it - 1 is free
    const int nx = it + kSmStages - 1;
    if (nx < ntiles)
      sm_issue<SG>(a, st, nqp, s0, maxk, hb, nx, tile[nx % kSmStages], vst[nx % kSmStages]);
    else
      cp_async_commit();
    const int jt = it * TK;
    const float* tl = tile[it % kSmStages];
    const float* vl = vst[it % kSmStages];
    const int lim = min(TK, n0 - jt);
#pragma unroll 4
    for (int i = l; i < lim; i += 16) {
      const float e = exp_malkin(__fsub_rn(tl[i * SG + sl], mx));
      sum = __fadd_rn(sum, e);
      st[static_cast<int64_t>(jt + i) * nqp + slot] = __fmul_rn(e, vl[i]);
    }
  }
  cp_async_wait<0>();
  float* er = a.p.ex + (static_cast<size_t>(t) * a.H + h) * a.p.ex_stride;
  // the extras: from the first key >= n0 of lane l's stripe on
  for (int j = n0 + ((l - n0 % 16) + 16) % 16; j < nk; j += 16) {
    const float e = exp_malkin(__fsub_rn(er[j - n0], mx));
    sum = __fadd_rn(sum, e);
    er[j - n0] = __fmul_rn(e, a.L.vs[hb + a.p.anc[e0 + j - n0]]);
  }
  rsum[l][sl] = sum;
  __syncthreads();
  if (l == 0 && valid) {  // malkin's reduce_add of the 16 lane sums
    float b8[8], c4[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) b8[i] = __fadd_rn(rsum[i + 8][sl], rsum[i][sl]);
#pragma unroll
    for (int i = 0; i < 4; ++i) c4[i] = __fadd_rn(b8[i + 4], b8[i]);
    const float tot = __fadd_rn(__fadd_rn(c4[0], c4[2]), __fadd_rn(c4[1], c4[3]));
    a.p.inv[static_cast<size_t>(t) * a.H + h] = __fdiv_rn(1.0f, tot);
  }
}

// grid (n_sg, KV, D / S), block 32 + rows x S / 4 (rows = kQMax / G). Warp 0 is the producer: lane 0 keeps
// kPvStages tiles of kPvTile keys in flight with TMA bulk copies (the ST rows and the raw int8 value rows), the warp
// converts the slice of each landed value tile into floats held twice, (v, v), and signals `ready`. Consumer thread
// (r, u) owns values 4u .. 4u + 3 of the slice for the G heads of row t0 + r: one f32x2 FMA advances the chains of
// two heads (heads 2i, 2i + 1; for odd G the last pair's second lane is a padding slot whose result is discarded).
// Each lane of the pair is its own IEEE fma in key order: malkin's acc = fma(p_j, v_j, acc). Converted value row:
// (v0 v0 v1 v1) of every u in the first 4 S bytes, (v2 v2 v3 v3) in the next, so a warp's 16-byte loads read
// contiguous bytes. S (32, 16, 8 or 4 values per CTA) is picked per launch (pv_slice).
template <int D, int G, int S>
struct PvGeom {
  static constexpr int U = S / 4, VFROW = 2 * S;  // threads per row; floats per converted value row
  static constexpr int ROWS = kQMax / G, CW = (ROWS * U + 31) / 32, NT = 32 * (1 + CW);
  static constexpr int GA = att_ga(G), NQP = att_nqp(ROWS, G);
  static constexpr uint32_t PB = kPvTile * NQP * 4, VB = kPvTile * D, FB = kPvTile * VFROW * 4;
  static constexpr uint32_t STAGE = (PB + VB + FB + 127) / 128 * 128;  // P rows | raw values | converted values
  static constexpr uint32_t BAR = kPvStages * STAGE;
  static constexpr uint32_t SMEM = BAR + 3 * kPvStages * 8;
};
// Lane 0 of the producer: tile `it` (kPvTile keys from key it * kPvTile) of the P rows and the raw value rows into
// the stage at stg (values at stg + pb_off), completion counted on bar.
template <int D>
__device__ __forceinline__ void pv_issue(uint8_t* stg, uint32_t pb_off, uint64_t* bar, const float* st,
                                         const int8_t* vsrc, int it, int maxk, int nqp) {
  const int k0 = it * kPvTile, nkt = min(kPvTile, maxk - k0);
  const uint32_t pb = static_cast<uint32_t>(nkt) * nqp * 4, vb = static_cast<uint32_t>(nkt) * D;
  mbar_arrive_expect_tx(bar, pb + vb);
  bulk_g2s(stg, st + static_cast<int64_t>(k0) * nqp, pb, bar);
  bulk_g2s(stg + pb_off, vsrc + static_cast<int64_t>(k0) * D, vb, bar);
}

template <int D, int G, int S>
__global__ void __launch_bounds__(PvGeom<D, G, S>::NT) k_att_pv(AttArgs a) {
  using Gm = PvGeom<D, G, S>;
  constexpr int U = Gm::U, VFROW = Gm::VFROW;
  constexpr int GP = Gm::GA / 2;        // head pairs (the last one padded for odd G)
  constexpr int KB = G <= 4 ? 4 : 2;    // keys whose loads are issued together
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Gm::BAR);
  uint64_t* ready = full + kPvStages;
  uint64_t* empty = ready + kPvStages;
  const int sg = blockIdx.x, kvh = blockIdx.y, d0 = blockIdx.z * S;
  const int t0 = a.p.sg_first[sg], nr = a.p.sg_first[sg + 1] - t0;
  const int maxk = a.p.sg_maxk[sg];
  const int nqp = att_nqp(nr, G);
  const float* st = st_of(a, sg, kvh, maxk, nqp);
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  const int ntiles = (maxk + kPvTile - 1) / kPvTile;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cwarps = (nr * U + 31) / 32;  // consumer warps with at least one row
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPvStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 32);
      mbar_init(&empty[s], cwarps);
    }
    mbar_fence_init();
  }
  __syncthreads();
  if (warp == 0) {
    // ---------------- producer ----------------
    const int8_t* vsrc = a.L.v + hb * D;
    int issued = min(kPvStages, ntiles), landed = 0;
    if (lane == 0)
      for (int it = 0; it < issued; ++it) pv_issue<D>(sm + (it % kPvStages) * Gm::STAGE, Gm::PB, &full[it % kPvStages], st, vsrc, it, maxk, nqp);
    bool ok = true;
    for (int it = 0; it < ntiles; ++it) {
      const int s = it % kPvStages;
      if (!(ok = mbar_wait_warp(&full[s], (it / kPvStages) & 1, a.p.status, kErrAttWait))) break;
      landed = it + 1;
      const uint8_t* stg = sm + s * Gm::STAGE;
      const int8_t* vraw = reinterpret_cast<const int8_t*>(stg + Gm::PB);
      float4* vf = reinterpret_cast<float4*>(sm + s * Gm::STAGE + Gm::PB + Gm::VB);
      const int nkt = min(kPvTile, maxk - it * kPvTile);
      for (int i = lane; i < nkt * U; i += 32) {
        const int jj = i / U, u = i % U;
        const char4 w = *reinterpret_cast<const char4*>(vraw + jj * D + d0 + 4 * u);
        vf[jj * (VFROW / 4) + u] = make_float4(i8f(w.x), i8f(w.x), i8f(w.y), i8f(w.y));
        vf[jj * (VFROW / 4) + U + u] = make_float4(i8f(w.z), i8f(w.z), i8f(w.w), i8f(w.w));
      }
      mbar_arrive(&ready[s]);  // every lane: its conversions happen before the consumers' reads
      // refill the stage of the previous tile once its consumers have released it
      const int nxt = it - 1 + kPvStages;
      if (it >= 1 && nxt < ntiles) {
        const int sp = (it - 1) % kPvStages;
        if (!(ok = mbar_wait_warp(&empty[sp], ((it - 1) / kPvStages) & 1, a.p.status, kErrAttWait))) break;
        if (lane == 0) pv_issue<D>(sm + sp * Gm::STAGE, Gm::PB, &full[sp], st, vsrc, nxt, maxk, nqp);
        issued = nxt + 1;
      }
    }
    if (!ok)  // copies still in flight land before the CTA exits (bounded)
      for (int it = landed; it < issued; ++it)
        mbar_wait_warp(&full[it % kPvStages], (it / kPvStages) & 1, nullptr, 0);
    return;
  }
  // ---------------- consumers ----------------
  if (warp - 1 >= cwarps) return;
  const int ct = threadIdx.x - 32, r = ct / U, u = ct % U;
  const int t = t0 + r;
  const bool active = r < nr;
  const int n0 = active ? a.p.n_keys[t] : 0;
  f2 acc[GP][4];  // (head 2i, head 2i + 1) at output value 4u + e
#pragma unroll
  for (int i = 0; i < GP; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = f2_make(0.0f, 0.0f);
  bool ok = true;
  for (int it = 0; it < ntiles; ++it) {
    const int s = it % kPvStages;
    const uint32_t par = (it / kPvStages) & 1;
    if (!(ok = mbar_wait(&full[s], par, a.p.status, kErrAttWait) && mbar_wait(&ready[s], par, a.p.status, kErrAttWait)))
      break;
    const uint8_t* stg = sm + s * Gm::STAGE;
    const float* pt = reinterpret_cast<const float*>(stg) + r * Gm::GA;
    const float* vf = reinterpret_cast<const float*>(stg + Gm::PB + Gm::VB) + 4 * u;
    const int lim = active ? min(kPvTile, n0 - it * kPvTile) : 0;
    int jj = 0;
    for (; jj + KB <= lim; jj += KB) {
      f2 V[KB][4], P[KB][GP];
#pragma unroll
      for (int b = 0; b < KB; ++b) {
        const ulonglong2 va = *reinterpret_cast<const ulonglong2*>(vf + (jj + b) * VFROW);
        const ulonglong2 vb = *reinterpret_cast<const ulonglong2*>(vf + (jj + b) * VFROW + S);
        V[b][0] = va.x, V[b][1] = va.y, V[b][2] = vb.x, V[b][3] = vb.y;
        const float* pp = pt + (jj + b) * nqp;
        if constexpr (Gm::GA % 4 == 0) {
#pragma unroll
          for (int i = 0; i < GP / 2; ++i) {
            const ulonglong2 x = reinterpret_cast<const ulonglong2*>(pp)[i];
            P[b][2 * i] = x.x, P[b][2 * i + 1] = x.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < GP; ++i) P[b][i] = reinterpret_cast<const f2*>(pp)[i];
        }
      }
#pragma unroll
      for (int b = 0; b < KB; ++b)
#pragma unroll
        for (int i = 0; i < GP; ++i)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][e] = f2_fma(P[b][i], V[b][e], acc[i][e]);
    }
    for (; jj < lim; ++jj) {
      const ulonglong2 va = *reinterpret_cast<const ulonglong2*>(vf + jj * VFROW);
      const ulonglong2 vb = *reinterpret_cast<const ulonglong2*>(vf + jj * VFROW + S);
      const f2 V[4] = {va.x, va.y, vb.x, vb.y};
      const f2* pp = reinterpret_cast<const f2*>(pt + jj * nqp);
#pragma unroll
      for (int i = 0; i < GP; ++i) {
        const f2 P = pp[i];
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = f2_fma(P, V[e], acc[i][e]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!active || !ok) return;
  // the row's extra keys, in order
  const int e0 = a.p.anc_off[t], ne = a.p.anc_off[t + 1] - e0;
  const float* pr = a.p.ex + (static_cast<size_t>(t) * a.H + kvh * G) * a.p.ex_stride;
  for (int e = 0; e < ne; ++e) {
    const int8_t* vr = a.L.v + (hb + a.p.anc[e0 + e]) * D + d0 + 4 * u;
    const f2 V[4] = {f2_make(i8f(vr[0]), i8f(vr[0])), f2_make(i8f(vr[1]), i8f(vr[1])),
                     f2_make(i8f(vr[2]), i8f(vr[2])), f2_make(i8f(vr[3]), i8f(vr[3]))};
#pragma unroll
    for (int i = 0; i < GP; ++i) {
      const f2 P = f2_make(pr[(2 * i) * a.p.ex_stride + e], 2 * i + 1 < G ? pr[(2 * i + 1) * a.p.ex_stride + e] : 0.0f);
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][q] = f2_fma(P, V[q], acc[i][q]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const float iv = a.p.inv[static_cast<size_t>(t) * a.H + h];
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = __fmul_rn((g & 1) ? f2_hi(acc[g / 2][e]) : f2_lo(acc[g / 2][e]), iv);
    *reinterpret_cast<float4*>(a.out + (static_cast<size_t>(t) * a.H + h) * D + d0 + 4 * u) =
        make_float4(o[0], o[1], o[2], o[3]);
  }
}

template <int D, int G, int S>
void launch_pv_s(const AttArgs& a, cudaStream_t s) {
  using Gm = PvGeom<D, G, S>;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !attr[dev]) {
    cudaFuncSetAttribute(k_att_pv<D, G, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Gm::SMEM));
    attr[dev] = true;
  }
  const dim3 g(a.p.n_sg, a.KV, D / S);
  k_att_pv<D, G, S><<<g, Gm::NT, Gm::SMEM, s>>>(a);
}

// The value-slice width: 32 values per CTA unless that grid leaves SMs idle, then the widest that gives every SM a
// CTA (measured at the configurations' shapes: 32 is fastest from 256 CTAs up, 8B 132 vs 185 us at 16; one request of
// 17 rows, 32 CTAs at 32, runs 117 us at 4 vs 169 at 32); MALKIN_B200_PV_SLICE=<32|16|8|4> forces one.
inline int pv_slice(int ctas_at_32, int sms) {
  const char* e = std::getenv("MALKIN_B200_PV_SLICE");
  const int v = e ? std::atoi(e) : 0;
  const int forced = v == 32 || v == 16 || v == 8 || v == 4 ? v : 0;
  if (forced) return forced;
  int S = kPvSliceMax;
  while (S > 4 && ctas_at_32 * (kPvSliceMax / S) < sms) S /= 2;
  return S;
}

template <int D, int G>
void launch_pv(const AttArgs& a, cudaStream_t s) {
  static int sms[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int S = pv_slice(a.p.n_sg * a.KV * (D / kPvSliceMax), dev < kMaxDevices && sms[dev] ? sms[dev] : 148);
  switch (S) {
    case 32: launch_pv_s<D, G, 32>(a, s); break;
    case 16: launch_pv_s<D, G, 16>(a, s); break;
    case 8: launch_pv_s<D, G, 8>(a, s); break;
    default: launch_pv_s<D, G, 4>(a, s); break;
  }
}

// Slots per softmax CTA: 32, halved while the grid (sub-groups x KV heads x slot groups of the largest sub-group)
// would cover fewer than two CTAs per SM; MALKIN_B200_SM_SLOTS = 32 / 16 / 8 / 4 forces one.
template <int SG>
void launch_softmax_s(const AttArgs& a, int nqp, cudaStream_t s) {
  k_att_softmax<SG><<<dim3((nqp + SG - 1) / SG, a.p.n_sg, a.KV), 16 * SG, 0, s>>>(a);
}

void launch_softmax(const AttArgs& a, cudaStream_t s) {
  static int sms[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  const int nsm = dev < kMaxDevices && sms[dev] ? sms[dev] : 148;
  const int nqp = att_nqp(kQMax / a.G, a.G);  // the largest sub-group's slots; CTAs past a smaller one exit
  const char* e = std::getenv("MALKIN_B200_SM_SLOTS");
  const int v = e ? std::atoi(e) : 0;
  int SG = v == 32 || v == 16 || v == 8 || v == 4 ? v : 0;
  if (!SG) {
    SG = 32;
    while (SG > 4 && a.p.n_sg * a.KV * ((nqp + SG - 1) / SG) < 2 * nsm) SG /= 2;
  }
  switch (SG) {
    case 32: launch_softmax_s<32>(a, nqp, s); break;
    case 16: launch_softmax_s<16>(a, nqp, s); break;
    case 8: launch_softmax_s<8>(a, nqp, s); break;
    default: launch_softmax_s<4>(a, nqp, s); break;
  }
}

template <int D>
void run_attention(const float* q, int H, int KV, float scale, const AttnLayer& L, const AttnPlan& p, float* out,
                   const ActQ& act, cudaStream_t s) {
  AttArgs a{q, H, KV, H / KV, scale, L, p, out ? out : p.att};
  if (p.n <= 0) return;
  constexpr int KP = sc_kp<D>();
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !attr[dev]) {
    int mx = 0;
    for (int g = 1; g <= 8; ++g) mx = std::max(mx, sc_smem(g, D));
    cudaFuncSetAttribute(k_att_scores<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, mx);
    attr[dev] = true;
  }
  if (p.n_sg > 0 && p.kchunks > 0)
    k_att_scores<D><<<dim3(p.kchunks, p.n_sg * kScoreParts, KV), 2 * kScoreKeys / KP, sc_smem(a.G, D), s>>>(a);
  k_att_extras<D><<<dim3(p.n, (H + 3) / 4), 128, 0, s>>>(a);
  if (p.n_sg > 0) launch_softmax(a, s);
  switch (a.G) {
    case 1: launch_pv<D, 1>(a, s); break;
    case 2: launch_pv<D, 2>(a, s); break;
    case 3: launch_pv<D, 3>(a, s); break;
    case 4: launch_pv<D, 4>(a, s); break;
    case 5: launch_pv<D, 5>(a, s); break;
    case 6: launch_pv<D, 6>(a, s); break;
    case 7: launch_pv<D, 7>(a, s); break;
    case 8: launch_pv<D, 8>(a, s); break;
    default: break;
  }
  if (act.qx) launch_quant_rows(a.out, static_cast<int64_t>(H) * D, p.n, H * D, act, s);
}

}  // namespace

int attn_qmax() { return kQMax; }

int attn_key_chunks(int n_ctx) { return (n_ctx + kScoreKeys - 1) / kScoreKeys; }

int64_t attn_st_floats(int rows, int G, int KV, int maxk) {
  return static_cast<int64_t>(KV) * (maxk + att_nch(maxk)) * att_nqp(rows, G);
}

void launch_qkv_post(Slices qk, int v_n, int64_t v_col0, int64_t ldy, int n, int H, int KV, int D, const float* q_norm,
                     const float* k_norm, float eps, const float* rope_cs, const int32_t* rpos, const int32_t* kv_at,
                     float* q_out, const AttnLayer& L, cudaStream_t s) {
  const dim3 grid(n, (H + 2 * KV + 3) / 4);
  switch (D) {
    case 64:
      k_qkv_post<64><<<grid, 128, 0, s>>>(qk, v_n, v_col0, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at,
                                          q_out, L);
      break;
    case 128:
      k_qkv_post<128><<<grid, 128, 0, s>>>(qk, v_n, v_col0, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at,
                                           q_out, L);
      break;
    case 256:
      k_qkv_post<256><<<grid, 128, 0, s>>>(qk, v_n, v_col0, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at,
                                           q_out, L);
      break;
    default:
      break;
  }
}

void launch_attention(const float* q, int H, int KV, int D, float scale, const AttnLayer& L, const AttnPlan& p,
                      float* out, const ActQ& act, cudaStream_t s) {
  switch (D) {
    case 64:
      run_attention<64>(q, H, KV, scale, L, p, out, act, s);
      break;
    case 128:
      run_attention<128>(q, H, KV, scale, L, p, out, act, s);
      break;
    case 256:
      run_attention<256>(q, H, KV, scale, L, p, out, act, s);
      break;
    default:
      break;
  }
}

}  // namespace mkb
