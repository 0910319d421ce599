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
//   k_att_scores   one thread per prefix key of a (sub-group, KV head): the key row in registers, every query vector
//                  of the sub-group (rows x G heads) broadcast from shared memory; scores into the sub-group's
//                  key-major table ST[j][slot] (slot = row * GA + head, GA = G rounded up to even)
//   k_att_extras   one warp per (t, h): the scores of the token's extra (ancestor) keys, as 16 chains on a half-warp
//   k_att_softmax  one CTA per (sub-group, KV head): warp l runs malkin's vector lane l - the lane-striped maximum and
//                  sum of every slot - with 32 slots side by side, then e_j * v_scale_j in place of s_j and 1 / sum
//   k_att_pv       one CTA per (sub-group, KV head, 32 of the D values): TMA bulk copies bring key tiles of the
//                  probabilities (ST rows) and of the int8 values two tiles ahead; the chains of two heads advance
//                  in one f32x2 FMA (each lane of the pair its own IEEE fma, in key order); then each row's extras.
constexpr int kQMax = 96;         // query vectors (rows x G) per sub-group
constexpr int kScoreKeys = 128;   // keys (threads) per score CTA
constexpr int kPvTile = 64;       // keys per P.V tile
constexpr int kPvSlice = 32;      // output values per P.V CTA
constexpr int kErrAttWait = 24;   // status code: a P.V tile copy never landed

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

__device__ __forceinline__ float i8f(int8_t v) { return static_cast<float>(v); }

// ST of (sub-group sg, KV head kvh): maxk_sg rows of nqp floats.
__device__ __forceinline__ float* st_of(const AttArgs& a, int sg, int kvh, int maxk, int nqp) {
  return a.p.st + a.p.st_off[sg] + static_cast<int64_t>(kvh) * maxk * nqp;
}

// grid (key chunks, n_sg, KV), block kScoreKeys; dynamic smem: kQMax x D query floats + kQMax key limits. The 16 chains
// of a score run as 8 packed f32x2 pairs (chains 2m and 2m + 1 share an instruction; each lane of the pair is its
// own IEEE operation, so the values are malkin's) and the horizontal sum is done pairwise the same way.
template <int D>
__global__ void __launch_bounds__(kScoreKeys) k_att_scores(AttArgs a) {
  constexpr int DC = D / 16;
  extern __shared__ __align__(16) float qs[];
  int* nkq = reinterpret_cast<int*>(qs + kQMax * D);
  const int sg = blockIdx.y, kvh = blockIdx.z;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1];
  const int nq = (t1 - t0) * a.G;
  const int maxk = a.p.sg_maxk[sg];
  const int j0 = blockIdx.x * kScoreKeys;
  if (j0 >= maxk) return;
  for (int i = threadIdx.x; i < nq * D; i += kScoreKeys) {
    const int v = i / D, d = i % D;
    qs[i] = a.q[(static_cast<size_t>(t0 + v / a.G) * a.H + kvh * a.G + v % a.G) * D + d];
  }
  for (int v = threadIdx.x; v < nq; v += kScoreKeys) nkq[v] = a.p.n_keys[t0 + v / a.G];
  __syncthreads();
  const int j = j0 + threadIdx.x;
  if (j >= maxk) return;
  const size_t row = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0] + j;
  f2 kf[D / 2];  // (k[2m], k[2m + 1])
  {
    const int4* kr = reinterpret_cast<const int4*>(a.L.k + row * D);
#pragma unroll
    for (int c = 0; c < D / 16; ++c) {
      const int4 w = kr[c];
      const int8_t* b = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
      for (int e = 0; e < 8; ++e) kf[8 * c + e] = f2_make(i8f(b[2 * e]), i8f(b[2 * e + 1]));
    }
  }
  const float ks = __fmul_rn(a.L.ks[row], a.scale);
  const int ga = att_ga(a.G), nqp = att_nqp(t1 - t0, a.G);
  float* srow = st_of(a, sg, kvh, maxk, nqp) + static_cast<int64_t>(j) * nqp;
  for (int v = 0; v < nq; ++v) {
    if (j >= nkq[v]) continue;
    const ulonglong2* qv = reinterpret_cast<const ulonglong2*>(qs + v * D);  // pairs (q[2m], q[2m + 1])
    f2 acc[8];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const ulonglong2 x = qv[c];
      acc[2 * c] = f2_mul(x.x, kf[2 * c]);
      acc[2 * c + 1] = f2_mul(x.y, kf[2 * c + 1]);
    }
#pragma unroll
    for (int i = 1; i < DC; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const ulonglong2 x = qv[4 * i + c];
        acc[2 * c] = f2_fma(x.x, kf[8 * i + 2 * c], acc[2 * c]);
        acc[2 * c + 1] = f2_fma(x.y, kf[8 * i + 2 * c + 1], acc[2 * c + 1]);
      }
    // tree16 in pairs: lanes i + 8 and i (pairs p + 4 and p), then i + 4 and i, then (0 + 2, 1 + 3), then 0 + 1
    f2 b2[4], c2[2];
#pragma unroll
    for (int p = 0; p < 4; ++p) b2[p] = f2_add(acc[p + 4], acc[p]);
#pragma unroll
    for (int p = 0; p < 2; ++p) c2[p] = f2_add(b2[p + 2], b2[p]);
    const f2 d2 = f2_add(c2[0], c2[1]);
    srow[(v / a.G) * ga + v % a.G] = __fmul_rn(__fadd_rn(f2_lo(d2), f2_hi(d2)), ks);
  }
}

// grid (n, ceil(H / 4)), block 128: warp w computes the extra keys' scores of (t = blockIdx.x, h = blockIdx.y * 4 + w)
// into ex[t][h][e]: lane l < 16 runs chain l (the lanes of malkin's vector), reduce16 across the half-warp.
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
  for (int e = 0; e < ne; ++e) {
    const size_t row = hb + a.p.anc[e0 + e];
    const int8_t* kr = a.L.k + row * D;
    float acc = __fmul_rn(q[0], i8f(kr[lane & 15]));
#pragma unroll
    for (int i = 1; i < DC; ++i) acc = __fmaf_rn(q[i], i8f(kr[16 * i + (lane & 15)]), acc);
    acc = reduce16(acc);
    if (lane == 0) er[e] = __fmul_rn(acc, __fmul_rn(a.L.ks[row], a.scale));
  }
}

// grid (n_sg, KV, slot groups of 32), block 512: warp l (0..15) plays malkin's vector lane l for the CTA's 32 slots
// (lane = slot): the
// maximum over the slot's keys (any order), then e_j = exp(s_j - max) and the lane-striped sum over keys j = l, l + 16,
// ... in order (prefix keys from ST, extras from ex), p_j = e_j * v_scale_j written in place; then 1 / reduce16 of
// the 16 sums.
__global__ void __launch_bounds__(512) k_att_softmax(AttArgs a) {
  __shared__ float red[16][33];
  const int sg = blockIdx.x, kvh = blockIdx.y;
  const int l = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = a.p.sg_first[sg], rows = a.p.sg_first[sg + 1] - t0;
  const int maxk = a.p.sg_maxk[sg];
  const int ga = att_ga(a.G), nqp = att_nqp(rows, a.G);
  float* st = st_of(a, sg, kvh, maxk, nqp);
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  for (int s0 = blockIdx.z * 32; s0 < rows * ga && s0 < (blockIdx.z + 1) * 32; s0 += 32) {
    const int slot = s0 + lane, r = slot / ga, g = slot % ga;
    const bool valid = r < rows && g < a.G;
    const int t = t0 + (valid ? r : 0), h = kvh * a.G + (valid ? g : 0);
    const int n0 = valid ? a.p.n_keys[t] : 0;
    const int e0 = a.p.anc_off[t], ne = valid ? a.p.anc_off[t + 1] - e0 : 0, nk = n0 + ne;
    float* er = a.p.ex + (static_cast<size_t>(t) * a.H + h) * a.p.ex_stride;
    // maximum (of this lane's stripe, then over the 16 stripes)
    float mx = -INFINITY;
#pragma unroll 4
    for (int j = l; j < nk; j += 16) mx = fmaxf(mx, j < n0 ? st[static_cast<int64_t>(j) * nqp + slot] : er[j - n0]);
    red[l][lane] = mx;
    __syncthreads();
    mx = red[0][lane];
#pragma unroll
    for (int i = 1; i < 16; ++i) mx = fmaxf(mx, red[i][lane]);
    __syncthreads();
    // lane-striped sum in key order; eight keys of the stripe loaded at once, only the sum runs in sequence
    float sum = 0.0f;
    for (int jb = l; jb < nk; jb += 16 * 8) {
      float sv[8], vv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = jb + 16 * u;
        sv[u] = j < nk ? (j < n0 ? st[static_cast<int64_t>(j) * nqp + slot] : er[j - n0]) : 0.0f;
        vv[u] = j < nk ? a.L.vs[j < n0 ? hb + j : hb + a.p.anc[e0 + j - n0]] : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = jb + 16 * u;
        if (j < nk) {
          const float e = exp_malkin(__fsub_rn(sv[u], mx));
          sum = __fadd_rn(sum, e);
          const float p = __fmul_rn(e, vv[u]);
          if (j < n0)
            st[static_cast<int64_t>(j) * nqp + slot] = p;
          else
            er[j - n0] = p;
        }
      }
    }
    red[l][lane] = sum;
    __syncthreads();
    if (l == 0 && valid) {
      float b8[8], c4[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) b8[i] = __fadd_rn(red[i + 8][lane], red[i][lane]);
#pragma unroll
      for (int i = 0; i < 4; ++i) c4[i] = __fadd_rn(b8[i + 4], b8[i]);
      const float tot = __fadd_rn(__fadd_rn(c4[0], c4[2]), __fadd_rn(c4[1], c4[3]));
      a.p.inv[static_cast<size_t>(t) * a.H + h] = __fdiv_rn(1.0f, tot);
    }
    __syncthreads();
  }
}

// grid (n_sg, KV, D / kPvSlice), block rows x 8 (rows = kQMax / G): thread (r, u) owns values u*4 .. u*4+3 of the
// slice for the G heads of row t0 + r. Thread 0 keeps two tiles of kPvTile keys in flight with TMA bulk copies (the
// ST rows and the raw int8 value rows); every thread converts its share of a landed value tile into a shared float
// buffer holding each value twice (v, v), so one f32x2 FMA advances the chains of two heads (each lane of the pair
// is its own IEEE fma, in key order: malkin's acc = fma(p_j, v_j, acc)).
constexpr int kVS2 = 2 * kPvSlice + 8;  // float value buffer row stride (32 values duplicated + padding)
template <int D, int G>
struct PvGeom {
  static constexpr int ROWS = kQMax / G, NT = ROWS * 8, GA = att_ga(G);
  static constexpr int NQP = att_nqp(ROWS, G);                // largest P row (floats)
  static constexpr uint32_t PBYTES = kPvTile * NQP * 4, VBYTES = kPvTile * D;
  static constexpr uint32_t STAGE = PBYTES + VBYTES;           // one stage: P rows then raw values
  static constexpr uint32_t VF = 2 * STAGE;                    // float value buffer offset
  static constexpr uint32_t BAR = VF + kPvTile * kVS2 * 4;     // two mbarriers
  static constexpr uint32_t SMEM = BAR + 16;
};
template <int D, int G>
__global__ void __launch_bounds__(kQMax / G * 8) k_att_pv(AttArgs a) {
  using Gm = PvGeom<D, G>;
  constexpr int GP = G / 2;  // head pairs
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Gm::BAR);
  float* vf = reinterpret_cast<float*>(sm + Gm::VF);
  const int sg = blockIdx.x, kvh = blockIdx.y, d0 = blockIdx.z * kPvSlice;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1], nr = t1 - t0;
  const int r = threadIdx.x >> 3, u = threadIdx.x & 7;
  const int t = t0 + r;
  const bool active = r < nr;
  const int maxk = a.p.sg_maxk[sg];
  const int n0 = active ? a.p.n_keys[t] : 0;
  const int nqp = att_nqp(nr, G);
  const float* st = st_of(a, sg, kvh, maxk, nqp);
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  const int ntiles = (maxk + kPvTile - 1) / kPvTile;
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int it) {  // thread 0
    const int s = it & 1, k0 = it * kPvTile, nkt = min(kPvTile, maxk - k0);
    uint8_t* stg = sm + s * Gm::STAGE;
    const uint32_t pb = static_cast<uint32_t>(nkt) * nqp * 4, vb = static_cast<uint32_t>(nkt) * D;
    mbar_arrive_expect_tx(&full[s], pb + vb);
    bulk_g2s(stg, st + static_cast<int64_t>(k0) * nqp, pb, &full[s]);
    bulk_g2s(stg + Gm::PBYTES, a.L.v + (hb + k0) * D, vb, &full[s]);
  };
  if (threadIdx.x == 0)
    for (int it = 0; it < 2 && it < ntiles; ++it) issue(it);
  f2 acc2[GP > 0 ? GP : 1][4];  // (head 2 hp, head 2 hp + 1) at output value e
  float acc1[4];                // the last head when G is odd
#pragma unroll
  for (int e = 0; e < 4; ++e) {
#pragma unroll
    for (int hp = 0; hp < GP; ++hp) acc2[hp][e] = f2_make(0.0f, 0.0f);
    acc1[e] = 0.0f;
  }
  bool ok = true;
  for (int it = 0; it < ntiles; ++it) {
    const int s = it & 1, k0 = it * kPvTile, nkt = min(kPvTile, maxk - k0);
    ok = ok && mbar_wait(&full[s], (it >> 1) & 1, a.p.status, kErrAttWait);
    const uint8_t* stg = sm + s * Gm::STAGE;
    // value slice of the landed tile -> floats, each twice
    const int8_t* vraw = reinterpret_cast<const int8_t*>(stg + Gm::PBYTES);
    for (int i = threadIdx.x; i < nkt * (kPvSlice / 4); i += blockDim.x) {
      const int jj = i / (kPvSlice / 4), c = i % (kPvSlice / 4);
      const char4 w = *reinterpret_cast<const char4*>(vraw + jj * D + d0 + 4 * c);
      float4* dst = reinterpret_cast<float4*>(vf + jj * kVS2 + 8 * c);
      dst[0] = make_float4(i8f(w.x), i8f(w.x), i8f(w.y), i8f(w.y));
      dst[1] = make_float4(i8f(w.z), i8f(w.z), i8f(w.w), i8f(w.w));
    }
    __syncthreads();
    if (active && ok) {
      const float* pt = reinterpret_cast<const float*>(stg);
      const int lim = min(nkt, n0 - k0);
      // keys in groups of kB: every shared-memory load of the group is issued before its FMAs (which run in key order)
      constexpr int kB = 4;
      int jj = 0;
      for (; jj + kB <= lim; jj += kB) {
        f2 V[kB][4], P[kB][GP > 0 ? GP : 1];
        float P1[kB];
#pragma unroll
        for (int b = 0; b < kB; ++b) {
          const ulonglong2* vv = reinterpret_cast<const ulonglong2*>(vf + (jj + b) * kVS2 + 8 * u);
          const ulonglong2 va = vv[0], vb = vv[1];
          V[b][0] = va.x, V[b][1] = va.y, V[b][2] = vb.x, V[b][3] = vb.y;
          const float* pp = pt + (jj + b) * nqp + r * Gm::GA;
#pragma unroll
          for (int hp = 0; hp < GP; ++hp) P[b][hp] = *reinterpret_cast<const f2*>(pp + 2 * hp);
          P1[b] = (G % 2) ? pp[G - 1] : 0.0f;
        }
#pragma unroll
        for (int b = 0; b < kB; ++b) {
#pragma unroll
          for (int hp = 0; hp < GP; ++hp)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc2[hp][e] = f2_fma(P[b][hp], V[b][e], acc2[hp][e]);
          if constexpr (G % 2) {
#pragma unroll
            for (int e = 0; e < 4; ++e) acc1[e] = __fmaf_rn(P1[b], f2_lo(V[b][e]), acc1[e]);
          }
        }
      }
      for (; jj < lim; ++jj) {
        const ulonglong2* vv = reinterpret_cast<const ulonglong2*>(vf + jj * kVS2 + 8 * u);  // (v_e, v_e), e = 0..3
        const ulonglong2 va = vv[0], vb = vv[1];
        const float* pp = pt + jj * nqp + r * Gm::GA;
        const f2 V[4] = {va.x, va.y, vb.x, vb.y};
#pragma unroll
        for (int hp = 0; hp < GP; ++hp) {
          const f2 P = *reinterpret_cast<const f2*>(pp + 2 * hp);  // (p_2hp, p_2hp+1)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc2[hp][e] = f2_fma(P, V[e], acc2[hp][e]);
        }
        if constexpr (G % 2) {
          const float p = pp[G - 1];
#pragma unroll
          for (int e = 0; e < 4; ++e) acc1[e] = __fmaf_rn(p, f2_lo(V[e]), acc1[e]);
        }
      }
    }
    __syncthreads();  // stage s and the value buffer are free
    if (threadIdx.x == 0 && it + 2 < ntiles && ok) issue(it + 2);
  }
  if (!active || !ok) return;
  // the row's extra keys, in order
  const int e0 = a.p.anc_off[t], ne = a.p.anc_off[t + 1] - e0;
  for (int e = 0; e < ne; ++e) {
    const size_t row = hb + a.p.anc[e0 + e];
    const int8_t* vr = a.L.v + row * D + d0 + 4 * u;
    const f2 V[4] = {f2_make(i8f(vr[0]), i8f(vr[0])), f2_make(i8f(vr[1]), i8f(vr[1])),
                     f2_make(i8f(vr[2]), i8f(vr[2])), f2_make(i8f(vr[3]), i8f(vr[3]))};
    const float* pr = a.p.ex + (static_cast<size_t>(t) * a.H + kvh * G) * a.p.ex_stride + e;
#pragma unroll
    for (int hp = 0; hp < GP; ++hp) {
      const f2 P = f2_make(pr[(2 * hp) * a.p.ex_stride], pr[(2 * hp + 1) * a.p.ex_stride]);
#pragma unroll
      for (int q = 0; q < 4; ++q) acc2[hp][q] = f2_fma(P, V[q], acc2[hp][q]);
    }
    if constexpr (G % 2) {
      const float p = pr[(G - 1) * a.p.ex_stride];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc1[q] = __fmaf_rn(p, f2_lo(V[q]), acc1[q]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const float iv = a.p.inv[static_cast<size_t>(t) * a.H + h];
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x = (G % 2 && g == G - 1) ? acc1[e] : ((g & 1) ? f2_hi(acc2[g / 2 < GP ? g / 2 : 0][e])
                                                                  : f2_lo(acc2[g / 2 < GP ? g / 2 : 0][e]));
      o[e] = __fmul_rn(x, iv);
    }
    *reinterpret_cast<float4*>(a.out + (static_cast<size_t>(t) * a.H + h) * D + d0 + 4 * u) =
        make_float4(o[0], o[1], o[2], o[3]);
  }
}

template <int D, int G>
void launch_pv(const AttArgs& a, cudaStream_t s) {
  using Gm = PvGeom<D, G>;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !attr[dev]) {
    cudaFuncSetAttribute(k_att_pv<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(Gm::SMEM));
    attr[dev] = true;
  }
  const dim3 g(a.p.n_sg, a.KV, D / kPvSlice);
  k_att_pv<D, G><<<g, Gm::NT, Gm::SMEM, s>>>(a);
}

template <int D>
void run_attention(const float* q, int H, int KV, float scale, const AttnLayer& L, const AttnPlan& p, float* out,
                   const ActQ& act, cudaStream_t s) {
  AttArgs a{q, H, KV, H / KV, scale, L, p, out ? out : p.att};
  if (p.n <= 0) return;
  const size_t qsmem = kQMax * D * sizeof(float) + kQMax * sizeof(int);
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < kMaxDevices && !attr[dev]) {
    cudaFuncSetAttribute(k_att_scores<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(qsmem));
    attr[dev] = true;
  }
  if (p.n_sg > 0 && p.kchunks > 0) k_att_scores<D><<<dim3(p.kchunks, p.n_sg, KV), kScoreKeys, qsmem, s>>>(a);
  k_att_extras<D><<<dim3(p.n, (H + 3) / 4), 128, 0, s>>>(a);
  if (p.n_sg > 0) k_att_softmax<<<dim3(p.n_sg, KV, (kQMax / (H / KV) * att_ga(H / KV) + 31) / 32), 512, 0, s>>>(a);
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
  return static_cast<int64_t>(KV) * maxk * att_nqp(rows, G);
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
