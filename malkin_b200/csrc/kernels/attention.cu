// Attention side of a decoder layer (model.cpp:468-496): q/k head RMSNorm + NeoX RoPE + int8 KV write, then
// tree-masked GQA attention over the HBM-resident int8 KV cache (Model::attention + kern::attend_gqa,
// model.cpp:303-346, kernels_avx512.cpp:228-306).
//
// Key sets (model.cpp:405-420): token t attends keys [0, n_keys[t]) of its sequence, then its extra rows anc[...]
// (tree ancestors, root first, itself last). Rows of one sequence that share the prefix form a sub-group; one
// CTA takes a (sub-group, KV head, key chunk) and scores every (row, query head) of the sub-group against the
// chunk, so each prefix key is read once per sub-group and KV head (GQA: the G query heads share it).
// Per chunk it keeps an online softmax (running max m, sum l, weighted values o); the combine kernel merges the
// chunks and the extra rows. Arithmetic: score = (q . k_int8) * (k_scale * 1/sqrt(D)); p = exp(score - max)
// with malkin's exp; out = (sum p * v_scale * v_int8) / sum p.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

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
  // quantize_i8 (quant.cpp:216-222) into the cache row kv_at[t] of this KV head.
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
// m16 tiles, one per warp. Per tile of 64 keys: S = Q K^T with mma.sync m16n8k16 (fp16 in, fp32 accumulate) where Q
// is split into fp16 hi + lo parts (q = hi + lo to ~22 bits) and int8 K converts to fp16 exactly; then the online
// softmax in registers (a row lives in one quad of lanes); then O += P V with P' = p * v_scale * 2^12 split into fp16
// hi + lo (the power-of-two scale keeps P' in fp16's normal range; it is divided out exactly at the end) and int8 V
// in fp16. K / V int8 tiles for the next 64 keys are prefetched into registers while the current tile computes.
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

template <int D>
struct AttSmem {
  static constexpr int DP = D + 8;  // padded fp16 row (conflict-free ldmatrix)
  static constexpr size_t QH = 0, QL = QH + sizeof(__half) * kQMax * DP, K = QL + sizeof(__half) * kQMax * DP,
                          V = K + sizeof(__half) * kKT * DP, KS = V + sizeof(__half) * kKT * DP, VS = KS + 4 * kKT,
                          NK = VS + 4 * kKT, BYTES = NK + 4 * kQMax;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 2) k_attn_part(PartArgs a) {  // two CTAs per SM
  using SM = AttSmem<D>;
  constexpr int DP = SM::DP;
  constexpr int NDT = D / 8;          // d tiles (n8) of O
  constexpr int CH = D / 16;          // 16-byte int8 chunks per key row
  constexpr int PF = (2 * kKT * CH + kThreads - 1) / kThreads;  // prefetch chunks per thread (K and V)
  extern __shared__ __align__(128) uint8_t sm[];
  __half* Qh = reinterpret_cast<__half*>(sm + SM::QH);
  __half* Ql = reinterpret_cast<__half*>(sm + SM::QL);
  __half* Kh = reinterpret_cast<__half*>(sm + SM::K);
  __half* Vh = reinterpret_cast<__half*>(sm + SM::V);
  float* ksc = reinterpret_cast<float*>(sm + SM::KS);
  float* vsc = reinterpret_cast<float*>(sm + SM::VS);
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

  // Q (hi / lo fp16), zero rows past nq: warp w loads its 16 query vectors, lanes over d (independent loads first)
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
        __half hi, lo;
        split_h(qv[i][m], hi, lo);
        Qh[qi * DP + lane + 32 * m] = hi;
        Ql[qi * DP + lane + 32 * m] = lo;
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
  auto commit = [&]() {
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      const int i = tid + u * kThreads;
      if (i < 2 * kKT * CH) {
        const bool isv = i >= kKT * CH;
        const int ii = isv ? i - kKT * CH : i;
        const int j = ii / CH, ch = ii % CH;
        __half* dst = (isv ? Vh : Kh) + j * DP + ch * 16;
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
      ksc[tid] = pks;
      vsc[tid] = pvs;
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

  for (int kt = k0; kt < k1; kt += kKT) {
    commit();
    __syncthreads();
    if (kt + kKT < k1) fetch(kt + kKT);
    if (active) {
      // S = Q K^T for this warp's 16 query vectors x 64 keys
      float sacc[kKT / 8][4];
#pragma unroll
      for (int j = 0; j < kKT / 8; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t ah[4], al[4];
        const int qr = r0 + (lane & 15), qc = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(ah, Qh + qr * DP + qc);
        ldsm_x4(al, Ql + qr * DP + qc);
        uint32_t b[kKT / 16][4];
#pragma unroll
        for (int nj = 0; nj < kKT / 16; ++nj) {  // two n8 tiles per ldmatrix.x4
          const int kr = nj * 16 + (lane >> 4) * 8 + (lane & 7), kc = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(b[nj], Kh + kr * DP + kc);
        }
        // the hi pass over every n tile, then the lo pass: dependent MMAs on one accumulator are 8 apart
#pragma unroll
        for (int nj = 0; nj < kKT / 16; ++nj) {
          mma_f16(sacc[2 * nj], ah, b[nj][0], b[nj][1]);
          mma_f16(sacc[2 * nj + 1], ah, b[nj][2], b[nj][3]);
        }
#pragma unroll
        for (int nj = 0; nj < kKT / 16; ++nj) {
          mma_f16(sacc[2 * nj], al, b[nj][0], b[nj][1]);
          mma_f16(sacc[2 * nj + 1], al, b[nj][2], b[nj][3]);
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
      uint32_t ph[kKT / 16][4], pl[kKT / 16][4];
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
        __half h0, l0, h1, l1, h2, l2, h3, l3;
        split_h(pv[0], h0, l0);
        split_h(pv[1], h1, l1);
        split_h(pv[2], h2, l2);
        split_h(pv[3], h3, l3);
        // C layout of n-tile j -> A fragment of k16 step j / 2 (regs 0/1 from the even tile, 2/3 from the odd)
        const int kq = j >> 1, hi = (j & 1) * 2;
        ph[kq][hi] = pack_h2(h0, h1);
        ph[kq][hi + 1] = pack_h2(h2, h3);
        pl[kq][hi] = pack_h2(l0, l1);
        pl[kq][hi + 1] = pack_h2(l2, l3);
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
      // O += P' V
#pragma unroll
      for (int kq = 0; kq < kKT / 16; ++kq) {
        // hi pass over every d tile, then the lo pass (V fragments loaded again): dependent MMAs 16 apart
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
          for (int dj = 0; dj < NDT / 2; ++dj) {  // two d tiles per ldmatrix.x4.trans
            uint32_t b[4];
            const int vr = kq * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, vc = dj * 16 + (lane >> 4) * 8;
            ldsm_x4_t(b, Vh + vr * DP + vc);
            mma_f16(o[2 * dj], pass ? pl[kq] : ph[kq], b[0], b[1]);
            mma_f16(o[2 * dj + 1], pass ? pl[kq] : ph[kq], b[2], b[3]);
          }
        }
      }
    }
    __syncthreads();
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

template <int D>
size_t part_smem() {
  return AttSmem<D>::BYTES;
}

template <int D>
void run_attention(const float* q, int H, int KV, float scale, const AttnLayer& L, const AttnPlan& p, float* out,
                   const ActQ& act, cudaStream_t s) {
  PartArgs a{q, H, KV, H / KV, scale, L, p};
  const size_t smem = part_smem<D>();
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(k_attn_part<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    cudaFuncSetAttribute(k_attn_part<D>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attr[dev] = true;
  }
  if (p.n_sg > 0 && p.n_chunks > 0) {
    const dim3 g1(p.n_chunks, p.n_sg, KV);
    k_attn_part<D><<<g1, kThreads, smem, s>>>(a);
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
