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
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <string>

#include <cfloat>

#include "common.cuh"
#include "kernels.hpp"
#include "quant.cuh"
#include "pipeline.cuh"
#include "tcgen05.cuh"

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
    float ss = 0.0f;
#pragma unroll
    for (int m = 0; m < PER; ++m) ss = __fmaf_rn(v[m], v[m], ss);
    ss = warp_sum(ss);
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps)));
#pragma unroll
    for (int m = 0; m < PER; ++m) v[m] = __fmul_rn(__fmul_rn(v[m], s), w[lane + 32 * m]);
    // NeoX RoPE on pairs (i, i + D/2): lane's values m < PER/2 are the first halves of its pairs.
    const float* cs = rope_cs + static_cast<size_t>(rpos[t]) * D;  // [cos D/2][sin D/2]
#pragma unroll
    for (int m = 0; m < PER / 2; ++m) {
      const int i = lane + 32 * m;
      const float c = cs[i], sn = cs[HALF + i];
      const float x0 = v[m], x1 = v[m + PER / 2];
      v[m] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      v[m + PER / 2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
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

// ---------------- partial attention over a key chunk (tensor cores) ----------------
// One CTA = (sub-group, KV head, key chunk). Query vectors (sub-group rows x G heads, at most kQMax) are split into
// m16 tiles, one per warp. Per tile of 64 keys: S = Q K^T with mma.sync m16n8k16 (fp16 in, fp32 accumulate), int8 K
// converted to fp16 exactly; then the online softmax in registers (a row lives in one quad of lanes); then
// O += P' V with P' = p * v_scale * 2^12 in fp16 (the power-of-two scale keeps P' in fp16's normal range; it is
// divided out exactly at the end) and int8 V in fp16. Q and P' are fp16 (11 significant bits): their rounding
// (relative 2^-12) stays well below the int8 quantization of K, V and of the attention output that feeds the next
// GEMM. kSplit = true keeps the earlier two-term form (fp16 hi + lo for Q and P', ~22 bits, twice the MMAs) for
// error measurements (MALKIN_B200_ATTN_SPLIT=1).
// K / V int8 tiles stream global -> registers one tile ahead and are converted into one of two shared-memory buffers,
// so each 64-key tile costs one CTA barrier: the warps that pass the barrier of tile i have all finished tile i - 1,
// whose buffer the next conversion reuses only after the barrier of tile i + 1.
constexpr int kQMax = 96;   // query vectors per sub-group (6 warps x 16)
constexpr int kKT = 64;     // keys per tile
constexpr int kAttWarps = kQMax / 16;
constexpr int kThreads = kAttWarps * 32;
constexpr float kPScale = 4096.0f;

struct PartArgs {
  const float* q;  // [n][H][D]
  int H, KV, G;
  float scale;
  AttnLayer L;
  AttnPlan p;
};

// e^x for the attention softmax through the hardware base-2 exponential (exp2f); its relative error (a few ulp)
// is far inside the attention tolerance, and it costs a few instructions instead of a polynomial.
__device__ __forceinline__ float exp_fast(float x) { return exp2f(__fmul_rn(x, 1.4426950408889634f)); }

// Four int8 values (one word) -> two fp16x2, exactly: the bytes become fp16 1152 + q (0x6400 | (q + 128)), one
// subtraction recovers q.
__device__ __forceinline__ void i8x4_to_h2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140), b = __byte_perm(u, 0x64646464u, 0x4342);
  const __half2 bias = __float2half2_rn(1152.0f);
  const __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), bias);
  const __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), bias);
  lo = *reinterpret_cast<const uint32_t*>(&ha);
  hi = *reinterpret_cast<const uint32_t*>(&hb);
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

// x = hi + lo in fp16 (both round to nearest).
__device__ __forceinline__ void split_h(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(__fsub_rn(x, __half2float(hi)));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int D, bool kSplit>
struct AttSmem {
  static constexpr int DP = D + 8;  // padded fp16 row (conflict-free ldmatrix)
  static constexpr size_t QTERM = sizeof(__half) * kQMax * DP, KVTILE = sizeof(__half) * kKT * DP;
  static constexpr size_t QH = 0, QL = QH + QTERM, K = QL + (kSplit ? QTERM : 0), V = K + 2 * KVTILE,
                          KS = V + 2 * KVTILE, VS = KS + 2 * 4 * kKT, NK = VS + 2 * 4 * kKT, BYTES = NK + 4 * kQMax;
};

template <int D, bool kSplit>
__global__ void __launch_bounds__(kThreads, kSplit ? 1 : 2) k_attn_part(PartArgs a) {
  using SM = AttSmem<D, kSplit>;
  constexpr int DP = SM::DP;
  constexpr int NDT = D / 8;          // d tiles (n8) of O
  constexpr int CH = D / 16;          // 16-byte int8 chunks per key row
  constexpr int PF = (2 * kKT * CH + kThreads - 1) / kThreads;  // prefetch chunks per thread (K and V)
  constexpr int TP = kSplit ? 2 : 1;  // fp16 terms of Q and P'
  extern __shared__ __align__(128) uint8_t sm[];
  __half* Qh = reinterpret_cast<__half*>(sm + SM::QH);
  __half* Ql = reinterpret_cast<__half*>(sm + SM::QL);
  int* Nk = reinterpret_cast<int*>(sm + SM::NK);

  const int chunk = blockIdx.x, sg = blockIdx.y, kvh = blockIdx.z;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1];
  const int nq = (t1 - t0) * a.G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, c = lane & 3;
  const int maxk = a.p.sg_maxk[sg];
  const int k0 = chunk * a.p.chunk;
  if (k0 >= maxk) return;
  const int k1 = min(maxk, k0 + a.p.chunk);
  const int base = a.p.kv_base[t0];

  // Q in fp16 (hi / lo when split), zero rows past nq: warp w loads its 16 query vectors, lanes over d
  {
    constexpr int PL = D / 32;  // values per lane
    float qv[16][PL];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int qi = warp * 16 + i;
      const int t = t0 + qi / a.G, h = kvh * a.G + qi % a.G;
      const float* src = a.q + (static_cast<size_t>(t) * a.H + h) * D;
#pragma unroll
      for (int m = 0; m < PL; ++m) qv[i][m] = qi < nq ? src[lane + 32 * m] : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int qi = warp * 16 + i;
#pragma unroll
      for (int m = 0; m < PL; ++m) {
        if constexpr (kSplit) {
          __half hi, lo;
          split_h(qv[i][m], hi, lo);
          Qh[qi * DP + lane + 32 * m] = hi;
          Ql[qi * DP + lane + 32 * m] = lo;
        } else {
          Qh[qi * DP + lane + 32 * m] = __float2half_rn(qv[i][m]);
        }
      }
    }
  }
  for (int qi = tid; qi < kQMax; qi += kThreads) Nk[qi] = qi < nq ? a.p.n_keys[t0 + qi / a.G] : 0;

  const int8_t* kh = a.L.k + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const int8_t* vh = a.L.v + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const float* ksh = a.L.ks + static_cast<size_t>(kvh) * a.L.n_rows + base;
  const float* vsh = a.L.vs + static_cast<size_t>(kvh) * a.L.n_rows + base;

  // register prefetch of one 64-key tile: chunk i < kKT*CH is K, else V
  int4 pre[PF];
  float pks = 0.0f, pvs = 0.0f;
  auto fetch = [&](int kt) {
    const int nk = min(kKT, k1 - kt);
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int i = tid + u * kThreads;
      int4 v = make_int4(0, 0, 0, 0);
      if (i < 2 * kKT * CH) {
        const bool isv = i >= kKT * CH;
        const int ii = isv ? i - kKT * CH : i;
        const int j = ii / CH, ch = ii % CH;
        if (j < nk) v = *reinterpret_cast<const int4*>((isv ? vh : kh) + static_cast<size_t>(kt + j) * D + ch * 16);
      }
      pre[u] = v;
    }
    if (tid < kKT) {
      pks = tid < nk ? __fmul_rn(ksh[kt + tid], a.scale) : 0.0f;
      pvs = tid < nk ? __fmul_rn(vsh[kt + tid], kPScale) : 0.0f;
    }
  };
  // registers -> shared buffer b (fp16 K / V rows, scales)
  auto commit = [&](int b) {
    __half* Kb = reinterpret_cast<__half*>(sm + SM::K + b * SM::KVTILE);
    __half* Vb = reinterpret_cast<__half*>(sm + SM::V + b * SM::KVTILE);
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int i = tid + u * kThreads;
      if (i < 2 * kKT * CH) {
        const bool isv = i >= kKT * CH;
        const int ii = isv ? i - kKT * CH : i;
        const int j = ii / CH, ch = ii % CH;
        __half* dst = (isv ? Vb : Kb) + j * DP + ch * 16;
        uint4 h0, h1;
        i8x4_to_h2(static_cast<uint32_t>(pre[u].x), h0.x, h0.y);
        i8x4_to_h2(static_cast<uint32_t>(pre[u].y), h0.z, h0.w);
        i8x4_to_h2(static_cast<uint32_t>(pre[u].z), h1.x, h1.y);
        i8x4_to_h2(static_cast<uint32_t>(pre[u].w), h1.z, h1.w);
        reinterpret_cast<uint4*>(dst)[0] = h0;
        reinterpret_cast<uint4*>(dst)[1] = h1;
      }
    }
    if (tid < kKT) {
      reinterpret_cast<float*>(sm + SM::KS)[b * kKT + tid] = pks;
      reinterpret_cast<float*>(sm + SM::VS)[b * kKT + tid] = pvs;
    }
  };

  const int r0 = warp * 16;
  const bool active = r0 < nq;
  float o[NDT][4];
#pragma unroll
  for (int j = 0; j < NDT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;
  fetch(k0);
  __syncthreads();
  const int nkA = Nk[min(r0 + g, kQMax - 1)], nkB = Nk[min(r0 + g + 8, kQMax - 1)];

  int buf = 0;
  for (int kt = k0; kt < k1; kt += kKT, buf ^= 1) {
    commit(buf);
    __syncthreads();
    if (kt + kKT < k1) fetch(kt + kKT);
    if (!active) continue;
    const __half* Kh = reinterpret_cast<const __half*>(sm + SM::K + buf * SM::KVTILE);
    const __half* Vh = reinterpret_cast<const __half*>(sm + SM::V + buf * SM::KVTILE);
    const float* ksc = reinterpret_cast<const float*>(sm + SM::KS) + buf * kKT;
    const float* vsc = reinterpret_cast<const float*>(sm + SM::VS) + buf * kKT;
    // S = Q K^T for this warp's 16 query vectors x 64 keys
    float sacc[kKT / 8][4];
#pragma unroll
    for (int j = 0; j < kKT / 8; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t aq[TP][4];
      const int qr = r0 + (lane & 15), qc = kk * 16 + (lane >> 4) * 8;
      ldsm_x4(aq[0], Qh + qr * DP + qc);
      if constexpr (kSplit) ldsm_x4(aq[TP - 1], Ql + qr * DP + qc);
      uint32_t b[kKT / 16][4];
#pragma unroll
      for (int nj = 0; nj < kKT / 16; ++nj) {  // two n8 tiles per ldmatrix.x4
        const int kr = nj * 16 + (lane >> 4) * 8 + (lane & 7), kc = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(b[nj], Kh + kr * DP + kc);
      }
      // one pass per term over every n tile: dependent MMAs on one accumulator are 8 apart
#pragma unroll
      for (int tp = 0; tp < TP; ++tp)
#pragma unroll
        for (int nj = 0; nj < kKT / 16; ++nj) {
          mma_f16(sacc[2 * nj], aq[tp], b[nj][0], b[nj][1]);
          mma_f16(sacc[2 * nj + 1], aq[tp], b[nj][2], b[nj][3]);
        }
    }
    // scale, mask, online softmax
    float tmA = -INFINITY, tmB = -INFINITY;
#pragma unroll
    for (int j = 0; j < kKT / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = 8 * j + 2 * c + e, key = kt + col;
        const float ks = ksc[col];
        const bool okA = key < k1 && key < nkA, okB = key < k1 && key < nkB;
        sacc[j][e] = okA ? __fmul_rn(sacc[j][e], ks) : -INFINITY;
        sacc[j][2 + e] = okB ? __fmul_rn(sacc[j][2 + e], ks) : -INFINITY;
        tmA = fmaxf(tmA, sacc[j][e]);
        tmB = fmaxf(tmB, sacc[j][2 + e]);
      }
    }
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 1));
    tmA = fmaxf(tmA, __shfl_xor_sync(0xffffffffu, tmA, 2));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 1));
    tmB = fmaxf(tmB, __shfl_xor_sync(0xffffffffu, tmB, 2));
    const float nmA = fmaxf(mA, tmA), nmB = fmaxf(mB, tmB);
    const float alA = (mA == -INFINITY || nmA == -INFINITY) ? (nmA == -INFINITY ? 1.0f : 0.0f)
                                                            : exp_fast(__fsub_rn(mA, nmA));
    const float alB = (mB == -INFINITY || nmB == -INFINITY) ? (nmB == -INFINITY ? 1.0f : 0.0f)
                                                            : exp_fast(__fsub_rn(mB, nmB));
    mA = nmA;
    mB = nmB;
    float sA = 0.0f, sB = 0.0f;
    uint32_t pp[TP][kKT / 16][4];
#pragma unroll
    for (int j = 0; j < kKT / 8; ++j) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool rowA = e < 2;
        const float x = sacc[j][e], m = rowA ? mA : mB;
        const float p = x == -INFINITY ? 0.0f : exp_fast(__fsub_rn(x, m));
        if (rowA)
          sA += p;
        else
          sB += p;
        pv[e] = __fmul_rn(p, vsc[8 * j + 2 * c + (e & 1)]);
      }
      // C layout of n-tile j -> A fragment of k16 step j / 2 (regs 0/1 from the even tile, 2/3 from the odd)
      const int kq = j >> 1, hi = (j & 1) * 2;
      if constexpr (kSplit) {
        __half h0, l0, h1, l1, h2, l2, h3, l3;
        split_h(pv[0], h0, l0);
        split_h(pv[1], h1, l1);
        split_h(pv[2], h2, l2);
        split_h(pv[3], h3, l3);
        pp[0][kq][hi] = pack_h2(h0, h1);
        pp[0][kq][hi + 1] = pack_h2(h2, h3);
        pp[TP - 1][kq][hi] = pack_h2(l0, l1);
        pp[TP - 1][kq][hi + 1] = pack_h2(l2, l3);
      } else {
        const __half2 p01 = __floats2half2_rn(pv[0], pv[1]), p23 = __floats2half2_rn(pv[2], pv[3]);
        pp[0][kq][hi] = *reinterpret_cast<const uint32_t*>(&p01);
        pp[0][kq][hi + 1] = *reinterpret_cast<const uint32_t*>(&p23);
      }
    }
    sA += __shfl_xor_sync(0xffffffffu, sA, 1);
    sA += __shfl_xor_sync(0xffffffffu, sA, 2);
    sB += __shfl_xor_sync(0xffffffffu, sB, 1);
    sB += __shfl_xor_sync(0xffffffffu, sB, 2);
    lA = __fmaf_rn(lA, alA, sA);
    lB = __fmaf_rn(lB, alB, sB);
#pragma unroll
    for (int j = 0; j < NDT; ++j) {
      o[j][0] *= alA, o[j][1] *= alA, o[j][2] *= alB, o[j][3] *= alB;
    }
    // O += P' V: one pass per term over every d tile (V fragments loaded again for the second term)
#pragma unroll
    for (int kq = 0; kq < kKT / 16; ++kq) {
#pragma unroll
      for (int tp = 0; tp < TP; ++tp) {
#pragma unroll
        for (int dj = 0; dj < NDT / 2; ++dj) {  // two d tiles per ldmatrix.x4.trans
          uint32_t b[4];
          const int vr = kq * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = dj * 16 + (lane >> 4) * 8;
          ldsm_x4_t(b, Vh + vr * DP + vc);
          mma_f16(o[2 * dj], pp[tp][kq], b[0], b[1]);
          mma_f16(o[2 * dj + 1], pp[tp][kq], b[2], b[3]);
        }
      }
    }
  }
  // Partials: [((sg * n_chunks + chunk) * KV + kvh) * kQMax + qi][D + 2] = o[D], m, l.
  if (active) {
    float* part = a.p.part + ((static_cast<size_t>(sg) * a.p.n_chunks + chunk) * a.KV + kvh) * kQMax * (D + 2);
    const int qa = r0 + g, qb = r0 + g + 8;
    constexpr float inv = 1.0f / kPScale;
#pragma unroll
    for (int j = 0; j < NDT; ++j) {
      if (qa < nq) {
        part[static_cast<size_t>(qa) * (D + 2) + 8 * j + 2 * c] = o[j][0] * inv;
        part[static_cast<size_t>(qa) * (D + 2) + 8 * j + 2 * c + 1] = o[j][1] * inv;
      }
      if (qb < nq) {
        part[static_cast<size_t>(qb) * (D + 2) + 8 * j + 2 * c] = o[j][2] * inv;
        part[static_cast<size_t>(qb) * (D + 2) + 8 * j + 2 * c + 1] = o[j][3] * inv;
      }
    }
    if (c == 0) {
      if (qa < nq) part[static_cast<size_t>(qa) * (D + 2) + D] = mA, part[static_cast<size_t>(qa) * (D + 2) + D + 1] = lA;
      if (qb < nq) part[static_cast<size_t>(qb) * (D + 2) + D] = mB, part[static_cast<size_t>(qb) * (D + 2) + D + 1] = lB;
    }
  }
}

// ---------------- combine chunks + extra (ancestor) keys ----------------
// grid (n, ceil(H / 4)), block 128: one warp per (token, head).
// out (nullable): [n][H][D] floats. act (act.qx nullable): the same rows quantized to Q8 blocks straight into the
// GEMM activation layouts (head h = blocks h * D / 32 ..), rows n .. npad - 1 zero-filled (blockIdx.x >= n).
template <int D>
__global__ void k_attn_combine(PartArgs a, const int32_t* __restrict__ tok_sg, float* __restrict__ out, ActQ act) {
  constexpr int PER = D / 32;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (h >= a.H) return;
  if (t >= a.p.n) {
#pragma unroll
    for (int m = 0; m < PER; ++m) store_act(act, h * PER + m, t, QBlock{0, 0.0f, 0, 0}, lane);
    return;
  }
  const int kvh = h / a.G;
  const int sg = tok_sg[t];
  const int t0 = a.p.sg_first[sg];
  const int nck = (a.p.sg_maxk[sg] + a.p.chunk - 1) / a.p.chunk;
  const int qi = (t - t0) * a.G + (h - kvh * a.G);
  const float* part = a.p.part + (static_cast<size_t>(sg) * a.p.n_chunks * a.KV + kvh) * kQMax * (D + 2) +
                      static_cast<size_t>(qi) * (D + 2);
  const size_t cstride = static_cast<size_t>(a.KV) * kQMax * (D + 2);
  const int base = a.p.kv_base[t];
  const int e0 = a.p.anc_off[t], e1 = a.p.anc_off[t + 1];
  const float* qv = a.q + (static_cast<size_t>(t) * a.H + h) * D;
  float q[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) q[m] = qv[lane + 32 * m];
  const int8_t* kh = a.L.k + static_cast<size_t>(kvh) * a.L.n_rows * D;
  const int8_t* vh = a.L.v + static_cast<size_t>(kvh) * a.L.n_rows * D;
  const float* ksh = a.L.ks + static_cast<size_t>(kvh) * a.L.n_rows;
  const float* vsh = a.L.vs + static_cast<size_t>(kvh) * a.L.n_rows;
  // chunk maxima: lane c holds chunk c (up to 32 chunks per pass)
  float M = -INFINITY;
  for (int cb = 0; cb < nck; cb += 32) {
    const float mc = cb + lane < nck ? part[(cb + lane) * cstride + D] : -INFINITY;
    M = fmaxf(M, warp_max(mc));
  }
  // extra-key scores: lane e holds extra e (up to 32 extras per pass); dots in batches of 8 whose loads and
  // butterfly reductions run side by side (the same xor order as warp_sum)
  float se_reg = -INFINITY;
  for (int eb = e0; eb < e1; eb += 8) {
    float s8[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      s8[u] = 0.0f;
      if (eb + u < e1) {
        const size_t row = static_cast<size_t>(base) + a.p.anc[eb + u];
#pragma unroll
        for (int m = 0; m < PER; ++m) s8[u] = __fmaf_rn(q[m], static_cast<float>(kh[row * D + lane + 32 * m]), s8[u]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 8; ++u) s8[u] += __shfl_xor_sync(0xffffffffu, s8[u], o);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (eb + u < e1) {
        const size_t row = static_cast<size_t>(base) + a.p.anc[eb + u];
        const float sc = __fmul_rn(s8[u], __fmul_rn(ksh[row], a.scale));
        if (((eb + u - e0) & 31) == lane) se_reg = sc;
        M = fmaxf(M, sc);
      }
    }
  }
  float o[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) o[m] = 0.0f;
  float L = 0.0f;
  for (int cb = 0; cb < nck; cb += 4) {
    float mc[4], lc[4], oc[4][PER];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const bool ok = cb + u < nck;
      const float* pr = part + (cb + u) * cstride;
      mc[u] = ok ? pr[D] : -INFINITY;
      lc[u] = ok ? pr[D + 1] : 0.0f;
#pragma unroll
      for (int m = 0; m < PER; ++m) oc[u][m] = ok ? pr[lane + 32 * m] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (mc[u] == -INFINITY) continue;
      const float f = exp_malkin(__fsub_rn(mc[u], M));
      L = __fmaf_rn(lc[u], f, L);
#pragma unroll
      for (int m = 0; m < PER; ++m) o[m] = __fmaf_rn(oc[u][m], f, o[m]);
    }
  }
  for (int e = e0; e < e1; ++e) {
    const size_t row = static_cast<size_t>(base) + a.p.anc[e];
    float s;
    if (e - e0 < 32) {
      s = __shfl_sync(0xffffffffu, se_reg, e - e0);
    } else {  // more than 32 extras: recompute
      s = 0.0f;
#pragma unroll
      for (int m = 0; m < PER; ++m) s = __fmaf_rn(q[m], static_cast<float>(kh[row * D + lane + 32 * m]), s);
      s = warp_sum(s);
      s = __fmul_rn(s, __fmul_rn(ksh[row], a.scale));
    }
    const float p = exp_malkin(__fsub_rn(s, M));
    L = __fadd_rn(L, p);
    const float pv = __fmul_rn(p, vsh[row]);
#pragma unroll
    for (int m = 0; m < PER; ++m) o[m] = __fmaf_rn(pv, static_cast<float>(vh[row * D + lane + 32 * m]), o[m]);
  }
  const float inv = __fdiv_rn(1.0f, L);
  if (out) {
    float* dst = out + (static_cast<size_t>(t) * a.H + h) * D;
#pragma unroll
    for (int m = 0; m < PER; ++m) dst[lane + 32 * m] = __fmul_rn(o[m], inv);
  }
  if (act.qx) {
#pragma unroll
    for (int m = 0; m < PER; ++m) store_act(act, h * PER + m, t, quant_block32(__fmul_rn(o[m], inv), lane), lane);
  }
}

// ---------------- partial attention over a key chunk on tcgen05 (D = 128) ----------------
// One CTA = (sub-group, KV head, key chunk), like k_attn_part, with the products on the 5th-generation tensor core:
// S = Q Kᵀ (M = 128 query rows, the sub-group's G x rows zero-padded; N = 64 keys; K = 128) accumulates into one of
// two TMEM buffers from Q hi and Q lo (fp16, ~22 bits together) against the int8 K tile converted exactly to fp16;
// O += P' V (M = 128, N = 128 = D, K = 64 keys) accumulates into a TMEM O from P' = p · v_scale · 2^12 split into fp16
// hi + lo, against the int8 V tile in fp16 (read MN-major). Warp roles (320 threads, one CTA per SM):
//   0      TMEM owner; lane 0 issues the MMAs (S of tile j, then P'V of tile j - 1) and the commits
//   1      TMA producer: the raw int8 K / V rows of each tile and their scales into a 2-stage staging ring
//   2..5   converters: Q (once) and each staged tile into fp16 UMMA core-matrix layouts (2 buffers)
//   6..9   softmax: one query row per thread (TMEM lane quarter warp % 4): scale, mask, online max / sum, P' hi/lo
//          into shared memory, rescale O in TMEM when the row maximum grows; at the end O, m, l -> partials
// Every wait is bounded; TMEM is released on every path. Partials use k_attn_part's format (combined unchanged).
namespace tc_attn {
constexpr int kM = 128, kN = 64, kDh = 128;
constexpr int kThreads = 320;
constexpr uint32_t kCols = 256;  // S0 [0, 64), S1 [64, 128), O [128, 256)
constexpr int kErrBase = 16;     // status codes 16.. (bounded waits)
// shared-memory map (bytes)
constexpr uint32_t QH = 0, QL = QH + kM * kDh * 2, KF = QL + kM * kDh * 2, VF = KF + 2 * kN * kDh * 2,
                   PH = VF + 2 * kN * kDh * 2, PL = PH + kM * kN * 2, RAW = PL + kM * kN * 2,
                   RAWB = 2 * kN * kDh,  // one staged tile: K rows then V rows (int8)
                   SCF = RAW + 2 * RAWB,  // scales: [2][ks * scale 64 | vs * 2^12 64]
                   NKR = SCF + 2 * 2 * kN * 4,  // n_keys per query row [128]
                   BAR = NKR + kM * 4, BYTES = BAR + 32 * 8 + 16;
// K-major core-matrix offsets (bytes) of an fp16 tile whose rows are `r` and K index `k`, 16 K-chunks per row group
__device__ __forceinline__ uint32_t kmaj(int r, int k, int kchunks) {
  return static_cast<uint32_t>((r >> 3) * (kchunks * 128) + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
}  // namespace tc_attn

__global__ void __launch_bounds__(tc_attn::kThreads, 1) k_attn_part_tc(PartArgs a) {
  using namespace tc_attn;
  constexpr int D = kDh;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + BAR);
  uint64_t *raw_full = bar, *raw_free = bar + 2, *kv_full = bar + 4, *kv_free = bar + 6, *s_full = bar + 8,
           *s_free = bar + 10, *p_ready = bar + 12, *o_done = bar + 13, *mma_done = bar + 14;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sm + BAR + 32 * 8);
  int* nkr = reinterpret_cast<int*>(sm + NKR);

  const int chunk = blockIdx.x, sg = blockIdx.y, kvh = blockIdx.z;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1];
  const int nq = (t1 - t0) * a.G;
  const int maxk = a.p.sg_maxk[sg];
  const int k0 = chunk * a.p.chunk;
  if (k0 >= maxk) return;  // whole CTA, before any barrier or TMEM
  const int k1 = min(maxk, k0 + a.p.chunk);
  const int T = (k1 - k0 + kN - 1) / kN;  // key tiles
  const int base = a.p.kv_base[t0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = a.p.status;  // bounded waits record the first timeout here (nullable)

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_free[i], 4);
      mbar_init(&kv_full[i], 4);
      mbar_init(&kv_free[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_ready, 4);
    mbar_init(o_done, 1);
    mbar_init(mma_done, 1);
    mbar_fence_init();
  }
  for (int r = threadIdx.x; r < kM; r += blockDim.x) nkr[r] = r < nq ? a.p.n_keys[t0 + r / a.G] : 0;
  if (warp == 0) tmem_alloc(tmem_holder, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int8_t* kh = a.L.k + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const int8_t* vh = a.L.v + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const float* ksh = a.L.ks + static_cast<size_t>(kvh) * a.L.n_rows + base;
  const float* vsh = a.L.vs + static_cast<size_t>(kvh) * a.L.n_rows + base;

  if (warp == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc_s = umma_idesc_f16_f32(kM, kN);
    const uint32_t idesc_pv = umma_idesc_f16_f32(kM, D) | (1u << 16);  // B (V) MN-major
    const uint32_t qh = smem_addr(sm + QH), ql = smem_addr(sm + QL);
    bool ok = true;
    auto pv = [&](int i) {  // O += P'(tile i) V(tile i)
      if (!mbar_wait_warp(p_ready, i & 1, status, kErrBase + 6)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vb = smem_addr(sm + VF + (i & 1) * kN * D * 2);
        for (int pass = 0; pass < 2; ++pass) {
          const uint32_t pb = smem_addr(sm + (pass ? PL : PH));
          for (int ks = 0; ks < kN / 16; ++ks)
            tc_mma_f16_ss(tmem + 128, umma_desc_kmajor(pb + ks * 256, 128, 1024),
                          umma_desc_kmajor(vb + ks * 256, 128, 1024), idesc_pv, (i > 0 || pass > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
        tc_commit(&kv_free[i & 1]);
      }
      __syncwarp();
      return true;
    };
    for (int j = 0; j < T && ok; ++j) {
      const int b = j & 1;
      if (!mbar_wait_warp(&kv_full[b], (j >> 1) & 1, status, kErrBase + 0)) break;
      if (j >= 2 && !mbar_wait_warp(&s_free[b], ((j >> 1) - 1) & 1, status, kErrBase + 1)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kb = smem_addr(sm + KF + b * kN * D * 2);
        for (int pass = 0; pass < 2; ++pass)
          for (int kk = 0; kk < D / 16; ++kk)
            tc_mma_f16_ss(tmem + b * kN, umma_desc_kmajor((pass ? ql : qh) + kk * 256, 128, 2048),
                          umma_desc_kmajor(kb + kk * 256, 128, 2048), idesc_s, (pass > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&s_full[b]);
      }
      __syncwarp();
      if (j >= 1) ok = pv(j - 1);
    }
    if (ok) pv(T - 1);
    if (lane == 0) tc_commit(mma_done);
    __syncwarp();
    mbar_wait_warp(mma_done, 0, status, kErrBase + 7);
  } else if (warp == 1) {
    // ---------------- TMA producer: raw int8 rows + scales of each tile ----------------
    int issued = 0;
    for (int j = 0; j < T; ++j, ++issued) {
      const int b = j & 1, kt = k0 + j * kN, nk = min(kN, k1 - kt);
      if (j >= 2 && !mbar_wait_warp(&raw_free[b], ((j >> 1) - 1) & 1, status, kErrBase + 2)) break;
      uint8_t* raw = sm + RAW + b * RAWB;
      if (lane == 0) {
        // the tile's nk valid rows of K and of V (128 bytes each; row addresses are 128-byte aligned)
        mbar_arrive_expect_tx(&raw_full[b], static_cast<uint32_t>(2 * nk * D));
        bulk_g2s(raw, kh + static_cast<size_t>(kt) * D, nk * D, &raw_full[b]);
        bulk_g2s(raw + kN * D, vh + static_cast<size_t>(kt) * D, nk * D, &raw_full[b]);
      }
      __syncwarp();
    }
    for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
      if (!mbar_wait_warp(&raw_full[j & 1], (j >> 1) & 1, status, kErrBase + 3)) break;
  } else if (warp < 6) {
    // ---------------- converters ----------------
    const int ct = threadIdx.x - 64;  // 0..127
    // Q rows (query r = token (r / G), head kvh * G + r % G) as fp16 hi + lo, zero past nq; each warp takes rows
    // warp - 2 + 4 i, eight rows' loads in flight at a time
    for (int r0 = warp - 2; r0 < kM; r0 += 32) {
      float4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = r0 + 4 * i;
        v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nq) {
          const int t = t0 + r / a.G, h = kvh * a.G + r % a.G;
          v[i] = reinterpret_cast<const float4*>(a.q + (static_cast<size_t>(t) * a.H + h) * D)[lane];
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = r0 + 4 * i;
        const float x[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        __half hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) split_h(x[e], hi[e], lo[e]);
        const uint32_t off = kmaj(r, 4 * lane, D / 8);
        *reinterpret_cast<uint2*>(sm + QH + off) = make_uint2(pack_h2(hi[0], hi[1]), pack_h2(hi[2], hi[3]));
        *reinterpret_cast<uint2*>(sm + QL + off) = make_uint2(pack_h2(lo[0], lo[1]), pack_h2(lo[2], lo[3]));
      }
    }
    bool ok = true;
    // scales of the next tile prefetched into registers (threads ct < 64: key ct)
    float ks_next = 0.0f, vs_next = 0.0f;
    if (ct < kN && ct < min(kN, k1 - k0)) ks_next = ksh[k0 + ct], vs_next = vsh[k0 + ct];
    for (int j = 0; j < T && ok; ++j) {
      const int b = j & 1, kt = k0 + j * kN, nk = min(kN, k1 - kt);
      const float ks_cur = ks_next, vs_cur = vs_next;
      if (ct < kN && j + 1 < T && ct < min(kN, k1 - kt - kN)) ks_next = ksh[kt + kN + ct], vs_next = vsh[kt + kN + ct];
      if (!mbar_wait_warp(&raw_full[b], (j >> 1) & 1, status, kErrBase + 4)) break;
      if (j >= 2 && !mbar_wait_warp(&kv_free[b], ((j >> 1) - 1) & 1, status, kErrBase + 5)) break;
      const uint8_t* raw = sm + RAW + b * RAWB;
      uint8_t* kf = sm + KF + b * kN * D * 2;
      uint8_t* vf = sm + VF + b * kN * D * 2;
      // 64 keys x 8 chunks of 16 values, K and V: 4 chunks of each per thread, rows past nk zero. Thread ct takes
      // key ct % 64 and chunks (j + key) % 8: eight consecutive threads then read and write eight different bank
      // groups (staged rows are 128 bytes apart; the core-matrix rows 16 bytes apart).
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int key = ct & (kN - 1), d16 = (((ct >> 6) * 4 + u) + key) & 7;
        uint4 wk = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
        if (key < nk) {
          wk = *reinterpret_cast<const uint4*>(raw + key * D + d16 * 16);
          wv = *reinterpret_cast<const uint4*>(raw + kN * D + key * D + d16 * 16);
        }
        uint4 k0h, k1h, v0h, v1h;
        i8x4_to_h2(wk.x, k0h.x, k0h.y);
        i8x4_to_h2(wk.y, k0h.z, k0h.w);
        i8x4_to_h2(wk.z, k1h.x, k1h.y);
        i8x4_to_h2(wk.w, k1h.z, k1h.w);
        i8x4_to_h2(wv.x, v0h.x, v0h.y);
        i8x4_to_h2(wv.y, v0h.z, v0h.w);
        i8x4_to_h2(wv.z, v1h.x, v1h.y);
        i8x4_to_h2(wv.w, v1h.z, v1h.w);
        // K: K-major (rows = keys, 16 chunks of 8 dims); V: MN-major (8 dims contiguous, 8 keys per core matrix)
        *reinterpret_cast<uint4*>(kf + kmaj(key, d16 * 16, D / 8)) = k0h;
        *reinterpret_cast<uint4*>(kf + kmaj(key, d16 * 16 + 8, D / 8)) = k1h;
        *reinterpret_cast<uint4*>(vf + (2 * d16) * 1024 + (key >> 3) * 128 + (key & 7) * 16) = v0h;
        *reinterpret_cast<uint4*>(vf + (2 * d16 + 1) * 1024 + (key >> 3) * 128 + (key & 7) * 16) = v1h;
      }
      if (ct < kN) {  // scales: k * softmax scale, v * 2^12; zero past nk
        float* scf = reinterpret_cast<float*>(sm + SCF + b * 2 * kN * 4);
        scf[ct] = ct < nk ? __fmul_rn(ks_cur, a.scale) : 0.0f;
        scf[kN + ct] = ct < nk ? __fmul_rn(vs_cur, kPScale) : 0.0f;
      }
      // generic-proxy writes -> visible to the tensor core (async proxy); staging free for the producer
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&kv_full[b]);
        mbar_arrive(&raw_free[b]);
      }
      ok = true;
    }
  } else {
    // ---------------- softmax: query row r of this thread ----------------
    const int quarter = warp & 3, r = 32 * quarter + lane;
    const uint32_t lane_base = static_cast<uint32_t>(32 * quarter) << 16;
    const int nk_r = nkr[r];
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < T && ok; ++j) {
      const int b = j & 1, kt = k0 + j * kN;
      // the tile's scales (written by the converters) and its scores
      if (!mbar_wait_warp(&kv_full[b], (j >> 1) & 1, status, kErrBase + 11) ||
          !mbar_wait_warp(&s_full[b], (j >> 1) & 1, status, kErrBase + 8)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sc[kN];  // this row's scores of the tile (bits from TMEM, then scaled and masked in place)
      tmem_ld32(tmem + lane_base + b * kN, *reinterpret_cast<uint32_t(*)[32]>(&sc[0]));
      tmem_ld32(tmem + lane_base + b * kN + 32, *reinterpret_cast<uint32_t(*)[32]>(&sc[32]));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      const float* scf = reinterpret_cast<const float*>(sm + SCF + b * 2 * kN * 4);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kN; ++c) {
        const int key = kt + c;
        const bool valid = key < k1 && key < nk_r;
        sc[c] = valid ? __fmul_rn(sc[c], scf[c]) : -INFINITY;
        mt = fmaxf(mt, sc[c]);
      }
      // Lazy rescaling: the reference maximum m moves (and O, l are rescaled) only when a score exceeds it by more than
      // kLazy nats, so p = e^(s - m) <= e^kLazy and P' = p * v_scale * 2^12 stays inside fp16 for |v| < 254; O and l
      // are always relative to the same m, which the partial stores. The decision is per warp (TMEM access is
      // warp-wide); rows with no new maximum get a factor 1.
      constexpr float kLazy = 2.0f;
      const bool grow = mt > m + kLazy || (m == -INFINITY && mt != -INFINITY);
      const bool resc = __any_sync(0xffffffffu, grow);
      float mn = m, alpha = 1.0f;
      if (resc && mt > m) {
        mn = mt;
        alpha = m == -INFINITY ? 0.0f : exp_fast(__fsub_rn(m, mn));
      }
      m = mn;
      float sum = 0.0f;
      uint32_t ph[kN / 2], pl[kN / 2];
#pragma unroll
      for (int c = 0; c < kN; c += 2) {
        float pv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float x = sc[c + u];
          const float p = x == -INFINITY ? 0.0f : exp_fast(__fsub_rn(x, mn));
          sum += p;
          pv[u] = __fmul_rn(p, scf[kN + c + u]);
        }
        __half h0, l0, h1, l1;
        split_h(pv[0], h0, l0);
        split_h(pv[1], h1, l1);
        ph[c / 2] = pack_h2(h0, h1);
        pl[c / 2] = pack_h2(l0, l1);
      }
      l = __fmaf_rn(l, alpha, sum);
      // P'V of the previous tile must be done before O is rescaled and P is overwritten
      if (j >= 1 && !mbar_wait_warp(o_done, (j - 1) & 1, status, kErrBase + 9)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j >= 1 && resc) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t ov[32];
          tmem_ld32(tmem + lane_base + 128 + c0, ov);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__fmul_rn(__uint_as_float(ov[e]), alpha));
          tmem_st32(tmem + lane_base + 128 + c0, ov);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c8 = 0; c8 < kN / 8; ++c8) {
        const uint32_t off = kmaj(r, c8 * 8, kN / 8);
        *reinterpret_cast<uint4*>(sm + PH + off) = make_uint4(ph[4 * c8], ph[4 * c8 + 1], ph[4 * c8 + 2], ph[4 * c8 + 3]);
        *reinterpret_cast<uint4*>(sm + PL + off) = make_uint4(pl[4 * c8], pl[4 * c8 + 1], pl[4 * c8 + 2], pl[4 * c8 + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
    }
    // final O (after the last P'V) -> partials, like k_attn_part: o / 2^12, m, l
    if (ok && mbar_wait_warp(o_done, (T - 1) & 1, status, kErrBase + 10)) {
      tc_fence_after();
      float* part = a.p.part + ((static_cast<size_t>(sg) * a.p.n_chunks + chunk) * a.KV + kvh) * kQMax * (D + 2);
      constexpr float inv = 1.0f / kPScale;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t ov[32];
        tmem_ld32(tmem + lane_base + 128 + c0, ov);
        tmem_wait_ld();
        if (r < nq)
#pragma unroll
          for (int e = 0; e < 32; ++e) part[static_cast<size_t>(r) * (D + 2) + c0 + e] = __uint_as_float(ov[e]) * inv;
      }
      if (r < nq) {
        part[static_cast<size_t>(r) * (D + 2) + D] = m;
        part[static_cast<size_t>(r) * (D + 2) + D + 1] = l;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// Tree attention partials: the mma.sync kernel by default; MALKIN_B200_ATTN=tc selects the tcgen05 one (D = 128).
// Both pass the same oracle tests; on the 8B verify shape the tcgen05 kernel is slower today (95 us vs 67 us per
// layer): one query tile per CTA leaves S -> softmax -> P'V a serial chain per key tile at one CTA per SM, where the
// mma.sync kernel runs two CTAs per SM.
bool attn_use_tc() {
  const char* e = std::getenv("MALKIN_B200_ATTN");
  return e && std::string(e) == "tc";
}

// MALKIN_B200_ATTN_SPLIT=1: two-term fp16 Q and P' (error measurements); default one term.
bool attn_split() {
  static const bool on = [] {
    const char* e = std::getenv("MALKIN_B200_ATTN_SPLIT");
    return e && std::string(e) == "1";
  }();
  return on;
}

template <int D>
void run_attention(const float* q, int H, int KV, float scale, const AttnLayer& L, const AttnPlan& p, float* out,
                   const ActQ& act, cudaStream_t s) {
  PartArgs a{q, H, KV, H / KV, scale, L, p};
  const bool split = attn_split();
  const size_t smem = split ? AttSmem<D, true>::BYTES : AttSmem<D, false>::BYTES;
  auto part_fn = split ? k_attn_part<D, true> : k_attn_part<D, false>;
  static bool attr[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev][split]) {
    cudaFuncSetAttribute(part_fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    cudaFuncSetAttribute(part_fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attr[dev][split] = true;
  }
  if (p.n_sg > 0 && p.n_chunks > 0) {
    const dim3 g1(p.n_chunks, p.n_sg, KV);
    if constexpr (D == tc_attn::kDh) {
      if (attn_use_tc()) {
        static bool tc_attr[kMaxDevices] = {};
        if (dev < kMaxDevices && !tc_attr[dev]) {
          cudaFuncSetAttribute(k_attn_part_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tc_attn::BYTES));
          tc_attr[dev] = true;
        }
        k_attn_part_tc<<<g1, tc_attn::kThreads, tc_attn::BYTES, s>>>(a);
      } else {
        part_fn<<<g1, kThreads, smem, s>>>(a);
      }
    } else {
      part_fn<<<g1, kThreads, smem, s>>>(a);
    }
  }
  const dim3 g2(act.qx ? act.nt8 * 8 : p.n, (H + 3) / 4);
  k_attn_combine<D><<<g2, 128, 0, s>>>(a, p.tok_sg, out, act);
}

}  // namespace

int attn_qmax() { return kQMax; }

int attn_chunk_for(int max_keys, int n_sg, int KV, int num_sms) {
  const int pairs = std::max(1, n_sg * KV);
  const int target = std::max(1, 2 * num_sms / pairs);  // chunks per (sub-group, kv head)
  const int per = (std::max(1, max_keys) + target - 1) / target;
  return std::max(kKT, (per + kKT - 1) / kKT * kKT);
}

size_t attn_part_floats(int n_sg, int n_chunks, int KV, int D) {
  return static_cast<size_t>(n_sg) * n_chunks * KV * kQMax * (D + 2);
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
