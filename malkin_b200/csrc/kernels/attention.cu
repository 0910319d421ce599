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
// Every float operation is malkin's, in malkin's order, so the output is bit-identical. Three kernels:
//   k_att_scores   one thread per prefix key of a (sub-group, KV head): the key row in registers, every query vector
//                  of the sub-group (rows x G heads) broadcast from shared memory; scores to a workspace row per (t, h)
//   k_att_softmax  one warp per (t, h): the extra keys' scores, the maximum, e_j, the 16 lane-striped sums (one
//                  sequential chain per lane, as malkin's vector lanes), e_j * v_scale_j in place of s_j, and inv
//   k_att_pv       one thread per (row, 4 output values) of a (sub-group, KV head, 32-value slice of D): the G heads'
//                  chains over the shared prefix keys from shared-memory tiles, then each row's extra keys.
constexpr int kQMax = 96;         // query vectors (rows x G) per sub-group
constexpr int kScoreKeys = 128;   // keys (threads) per score CTA
constexpr int kPvTile = 64;       // keys per shared-memory tile of the P.V kernel
constexpr int kPvSlice = 32;      // output values per P.V CTA

struct AttArgs {
  const float* q;  // [n][H][D]
  int H, KV, G;
  float scale;
  AttnLayer L;
  AttnPlan p;
  float* out;      // [n][H][D]
};

// malkin's _mm512_reduce_add_ps on 16 values held by one thread: (0+8, 4+12, 2+10, 6+14, 1+9, 5+13, 3+11, 7+15)
// pairwise as the vector reduction pairs them.
__device__ __forceinline__ float tree16(const float (&a)[16]) {
  float b[8], c[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = __fadd_rn(a[i + 8], a[i]);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = __fadd_rn(b[i + 4], b[i]);
  return __fadd_rn(__fadd_rn(c[0], c[2]), __fadd_rn(c[1], c[3]));
}

__device__ __forceinline__ float i8f(int8_t v) { return static_cast<float>(v); }

// grid (key chunks, n_sg, KV), block kScoreKeys; dynamic smem: nq x D query floats + nq key limits.
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
  float kf[D];
  {
    const int4* kr = reinterpret_cast<const int4*>(a.L.k + row * D);
#pragma unroll
    for (int c = 0; c < D / 16; ++c) {
      const int4 w = kr[c];
      const int8_t* b = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
      for (int e = 0; e < 16; ++e) kf[16 * c + e] = i8f(b[e]);
    }
  }
  const float ks = __fmul_rn(a.L.ks[row], a.scale);
  for (int v = 0; v < nq; ++v) {
    if (j >= nkq[v]) continue;
    const float4* qv = reinterpret_cast<const float4*>(qs + v * D);
    float acc[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 x = qv[c];
      acc[4 * c] = __fmul_rn(x.x, kf[4 * c]);
      acc[4 * c + 1] = __fmul_rn(x.y, kf[4 * c + 1]);
      acc[4 * c + 2] = __fmul_rn(x.z, kf[4 * c + 2]);
      acc[4 * c + 3] = __fmul_rn(x.w, kf[4 * c + 3]);
    }
#pragma unroll
    for (int i = 1; i < DC; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float4 x = qv[4 * i + c];
        acc[4 * c] = __fmaf_rn(x.x, kf[16 * i + 4 * c], acc[4 * c]);
        acc[4 * c + 1] = __fmaf_rn(x.y, kf[16 * i + 4 * c + 1], acc[4 * c + 1]);
        acc[4 * c + 2] = __fmaf_rn(x.z, kf[16 * i + 4 * c + 2], acc[4 * c + 2]);
        acc[4 * c + 3] = __fmaf_rn(x.w, kf[16 * i + 4 * c + 3], acc[4 * c + 3]);
      }
    const int t = t0 + v / a.G, h = kvh * a.G + v % a.G;
    a.p.sbuf[(static_cast<size_t>(t) * a.H + h) * a.p.sstride + j] = __fmul_rn(tree16(acc), ks);
  }
}

// grid (n, ceil(H / 4)), block 128: warp w handles (t = blockIdx.x, h = blockIdx.y * 4 + w).
template <int D>
__global__ void __launch_bounds__(128) k_att_softmax(AttArgs a) {
  constexpr int DC = D / 16;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (h >= a.H) return;
  const int kvh = h / a.G;
  const int n0 = a.p.n_keys[t], e0 = a.p.anc_off[t], ne = a.p.anc_off[t + 1] - e0, nk = n0 + ne;
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t];
  float* sr = a.p.sbuf + (static_cast<size_t>(t) * a.H + h) * a.p.sstride;
  // extra keys: lane l < 16 runs chain l (the lanes of malkin's vector), reduce16 across the half-warp
  if (ne > 0) {
    const float* qv = a.q + (static_cast<size_t>(t) * a.H + h) * D;
    float q[DC];
#pragma unroll
    for (int i = 0; i < DC; ++i) q[i] = qv[16 * i + (lane & 15)];
    for (int e = 0; e < ne; ++e) {
      const size_t row = hb + a.p.anc[e0 + e];
      const int8_t* kr = a.L.k + row * D;
      float acc = __fmul_rn(q[0], i8f(kr[lane & 15]));
#pragma unroll
      for (int i = 1; i < DC; ++i) acc = __fmaf_rn(q[i], i8f(kr[16 * i + (lane & 15)]), acc);
      acc = reduce16(acc);
      if (lane == 0) sr[n0 + e] = __fmul_rn(acc, __fmul_rn(a.L.ks[row], a.scale));
    }
    __syncwarp();
  }
  float mx = -INFINITY;
  for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sr[j]);
  mx = warp_max(mx);
  for (int j = lane; j < nk; j += 32) sr[j] = exp_malkin(__fsub_rn(sr[j], mx));
  __syncwarp();
  // 16 lane-striped sums in key order (malkin's vector lanes), and p_j = e_j * v_scale_j for the P.V chains
  float sum = 0.0f;
  if (lane < 16) {
    for (int j = lane; j < nk; j += 16) {
      const float e = sr[j];
      sum = __fadd_rn(sum, e);
      const size_t row = j < n0 ? hb + j : hb + a.p.anc[e0 + j - n0];
      sr[j] = __fmul_rn(e, a.L.vs[row]);
    }
  }
  sum = reduce16(sum);
  if (lane == 0) a.p.inv[static_cast<size_t>(t) * a.H + h] = __fdiv_rn(1.0f, sum);
}

// grid (n_sg, KV, D / kPvSlice), block rows x 8 (rows = kQMax / G): thread (r, u) owns values u*4 .. u*4+3 of the
// slice for the G heads of row t0 + r. dynamic smem: V tile [kPvTile][kPvSlice] floats, P tile [kPvTile][rows * G].
template <int D, int G>
__global__ void k_att_pv(AttArgs a) {
  constexpr int ROWS = kQMax / G;
  extern __shared__ __align__(16) float pvs[];
  constexpr int PS = ROWS * G + 1;       // P tile row stride (odd: conflict-free stores)
  float* vt = pvs;                       // [kPvTile][kPvSlice]
  float* pt = pvs + kPvTile * kPvSlice;  // [kPvTile][PS]
  const int sg = blockIdx.x, kvh = blockIdx.y, d0 = blockIdx.z * kPvSlice;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1], nr = t1 - t0;
  const int r = threadIdx.x >> 3, u = threadIdx.x & 7;
  const int t = t0 + r;
  const bool active = r < nr;
  const int maxk = a.p.sg_maxk[sg];
  const int n0 = active ? a.p.n_keys[t] : 0;
  const size_t hb = static_cast<size_t>(kvh) * a.L.n_rows + a.p.kv_base[t0];
  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f;
  for (int k0 = 0; k0 < maxk; k0 += kPvTile) {
    const int nkt = min(kPvTile, maxk - k0);
    // V tile: 8-byte groups of the slice, converted exactly
    for (int i = threadIdx.x; i < kPvTile * (kPvSlice / 8); i += blockDim.x) {
      const int jj = i / (kPvSlice / 8), c = i % (kPvSlice / 8);
      float* dst = vt + jj * kPvSlice + 8 * c;
      if (jj < nkt) {
        const int2 w = *reinterpret_cast<const int2*>(a.L.v + (hb + k0 + jj) * D + d0 + 8 * c);
        const int8_t* b = reinterpret_cast<const int8_t*>(&w);
#pragma unroll
        for (int e = 0; e < 8; ++e) dst[e] = i8f(b[e]);
      }
    }
    // P tile: p_j of every (row, head) of the sub-group for these keys
    for (int i = threadIdx.x; i < nr * G * kPvTile; i += blockDim.x) {
      const int v = i / kPvTile, jj = i % kPvTile;
      if (jj < nkt)
        pt[jj * PS + v] =
            a.p.sbuf[(static_cast<size_t>(t0 + v / G) * a.H + kvh * G + v % G) * a.p.sstride + k0 + jj];
    }
    __syncthreads();
    if (active) {
      const int lim = min(nkt, n0 - k0);
      for (int jj = 0; jj < lim; ++jj) {
        const float4 vv = *reinterpret_cast<const float4*>(vt + jj * kPvSlice + 4 * u);
        const float* pp = pt + jj * PS + r * G;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float p = pp[g];
          acc[g][0] = __fmaf_rn(p, vv.x, acc[g][0]);
          acc[g][1] = __fmaf_rn(p, vv.y, acc[g][1]);
          acc[g][2] = __fmaf_rn(p, vv.z, acc[g][2]);
          acc[g][3] = __fmaf_rn(p, vv.w, acc[g][3]);
        }
      }
    }
    __syncthreads();
  }
  if (!active) return;
  // the row's extra keys, in order
  const int e0 = a.p.anc_off[t], ne = a.p.anc_off[t + 1] - e0;
  for (int e = 0; e < ne; ++e) {
    const size_t row = hb + a.p.anc[e0 + e];
    const int8_t* vr = a.L.v + row * D + d0 + 4 * u;
    const float v0 = i8f(vr[0]), v1 = i8f(vr[1]), v2 = i8f(vr[2]), v3 = i8f(vr[3]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float p = a.p.sbuf[(static_cast<size_t>(t) * a.H + kvh * G + g) * a.p.sstride + n0 + e];
      acc[g][0] = __fmaf_rn(p, v0, acc[g][0]);
      acc[g][1] = __fmaf_rn(p, v1, acc[g][1]);
      acc[g][2] = __fmaf_rn(p, v2, acc[g][2]);
      acc[g][3] = __fmaf_rn(p, v3, acc[g][3]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const float iv = a.p.inv[static_cast<size_t>(t) * a.H + h];
    float4 o;
    o.x = __fmul_rn(acc[g][0], iv);
    o.y = __fmul_rn(acc[g][1], iv);
    o.z = __fmul_rn(acc[g][2], iv);
    o.w = __fmul_rn(acc[g][3], iv);
    *reinterpret_cast<float4*>(a.out + (static_cast<size_t>(t) * a.H + h) * D + d0 + 4 * u) = o;
  }
}

template <int D, int G>
void launch_pv(const AttArgs& a, cudaStream_t s) {
  constexpr int ROWS = kQMax / G;
  const size_t smem = (kPvTile * kPvSlice + kPvTile * (ROWS * G + 1)) * sizeof(float);
  const dim3 g(a.p.n_sg, a.KV, D / kPvSlice);
  k_att_pv<D, G><<<g, ROWS * 8, smem, s>>>(a);
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
  k_att_softmax<D><<<dim3(p.n, (H + 3) / 4), 128, 0, s>>>(a);
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

size_t attn_ws_floats(int n, int H, int64_t sstride, int D) {
  return static_cast<size_t>(n) * H * static_cast<size_t>(sstride) + static_cast<size_t>(n) * H +
         static_cast<size_t>(n) * H * D;
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
