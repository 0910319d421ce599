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
#include <cuda_runtime.h>

#include <cfloat>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

namespace {

// ---------------- q/k norm + RoPE + KV write ----------------
// grid (n, ceil((H + 2 KV) / 4)), block 128: one warp per head. D % 64 == 0, D <= 256.
template <int D>
__global__ void k_qkv_post(const float* __restrict__ y, int64_t ldy, int n, int H, int KV,
                           const float* __restrict__ q_norm, const float* __restrict__ k_norm, float eps,
                           const float* __restrict__ rope_cs, const int32_t* __restrict__ rpos,
                           const int32_t* __restrict__ kv_at, float* __restrict__ q_out, AttnLayer L) {
  constexpr int PER = D / 32, HALF = D / 2;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (head >= H + 2 * KV) return;
  const float* src = y + static_cast<size_t>(t) * ldy + static_cast<size_t>(head) * D;
  float v[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) v[m] = src[lane + 32 * m];
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

// ---------------- partial attention over a key chunk ----------------
constexpr int kQMax = 72;   // query vectors per sub-group
constexpr int kKT = 32;     // keys per tile
constexpr int kThreads = 256;

struct PartArgs {
  const float* q;  // [n][H][D]
  int H, KV, G;
  float scale;
  AttnLayer L;
  AttnPlan p;
};

template <int D>
__global__ void __launch_bounds__(kThreads) k_attn_part(PartArgs a) {
  constexpr int DP = D + 4;            // padded smem row (floats)
  constexpr int DV = D / 4;            // threads per query for the PV product (4 dims each)
  constexpr int QG = kThreads / DV;    // query groups in PV
  constexpr int QI = (kQMax + QG - 1) / QG;
  constexpr int SI = kQMax / 8;        // queries per thread in the score product (8 warps)
  extern __shared__ float smem[];
  float* Qs = smem;                      // [kQMax][DP]
  float* Kf = Qs + kQMax * DP;           // [kKT][DP]
  float* Vf = Kf + kKT * DP;             // [kKT][DP]
  float* Ps = Vf + kKT * DP;             // [kQMax][kKT + 4]   p * v_scale
  float* Ms = Ps + kQMax * (kKT + 4);    // [kQMax] running max
  float* Ls = Ms + kQMax;                // [kQMax] running sum
  float* Al = Ls + kQMax;                // [kQMax] rescale of this tile
  int* Nk = reinterpret_cast<int*>(Al + kQMax);  // [kQMax] keys of the query's token

  const int chunk = blockIdx.x, sg = blockIdx.y, kvh = blockIdx.z;
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1];
  const int nq = (t1 - t0) * a.G;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Keys of this sub-group: the longest prefix among its rows.
  int maxk = 0;
  for (int t = t0; t < t1; ++t) maxk = max(maxk, a.p.n_keys[t]);
  const int k0 = chunk * a.p.chunk;
  if (k0 >= maxk) return;
  const int k1 = min(maxk, k0 + a.p.chunk);
  const int base = a.p.kv_base[t0];

  for (int i = tid; i < nq * D; i += kThreads) {
    const int qi = i / D, d = i % D;
    const int t = t0 + qi / a.G, h = kvh * a.G + qi % a.G;
    Qs[qi * DP + d] = a.q[(static_cast<size_t>(t) * a.H + h) * D + d];
  }
  for (int qi = tid; qi < kQMax; qi += kThreads) {
    Ms[qi] = -INFINITY;
    Ls[qi] = 0.0f;
    Nk[qi] = qi < nq ? a.p.n_keys[t0 + qi / a.G] : 0;
  }
  float o[QI][4];
#pragma unroll
  for (int i = 0; i < QI; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  const int8_t* kh = a.L.k + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const int8_t* vh = a.L.v + (static_cast<size_t>(kvh) * a.L.n_rows + base) * D;
  const float* ksh = a.L.ks + static_cast<size_t>(kvh) * a.L.n_rows + base;
  const float* vsh = a.L.vs + static_cast<size_t>(kvh) * a.L.n_rows + base;
  __syncthreads();

  for (int kt = k0; kt < k1; kt += kKT) {
    const int nk = min(kKT, k1 - kt);
    // int8 K / V tile -> float smem (unscaled), 4 values per thread-iteration.
    for (int i = tid; i < kKT * D / 4; i += kThreads) {
      const int j = i / (D / 4), d4 = (i % (D / 4)) * 4;
      char4 kv = make_char4(0, 0, 0, 0), vv = make_char4(0, 0, 0, 0);
      if (j < nk) {
        kv = *reinterpret_cast<const char4*>(kh + static_cast<size_t>(kt + j) * D + d4);
        vv = *reinterpret_cast<const char4*>(vh + static_cast<size_t>(kt + j) * D + d4);
      }
      float* kr = Kf + j * DP + d4;
      float* vr = Vf + j * DP + d4;
      kr[0] = kv.x, kr[1] = kv.y, kr[2] = kv.z, kr[3] = kv.w;
      vr[0] = vv.x, vr[1] = vv.y, vr[2] = vv.z, vr[3] = vv.w;
    }
    __syncthreads();
    // Scores: lane = key, warp w -> queries w + 8 i.
    {
      const int j = lane;
      const bool kvalid = j < nk;
      const float ks = kvalid ? __fmul_rn(ksh[kt + j], a.scale) : 0.0f;
      const float vs = kvalid ? vsh[kt + j] : 0.0f;
      float s[SI];
#pragma unroll
      for (int i = 0; i < SI; ++i) s[i] = 0.0f;
      const float* kr = Kf + j * DP;
#pragma unroll 4
      for (int d = 0; d < D; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
#pragma unroll
        for (int i = 0; i < SI; ++i) {
          const float4 q4 = *reinterpret_cast<const float4*>(Qs + (warp + 8 * i) * DP + d);
          s[i] = __fmaf_rn(q4.x, k4.x, s[i]);
          s[i] = __fmaf_rn(q4.y, k4.y, s[i]);
          s[i] = __fmaf_rn(q4.z, k4.z, s[i]);
          s[i] = __fmaf_rn(q4.w, k4.w, s[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < SI; ++i) {
        const int qi = warp + 8 * i;
        const bool valid = kvalid && qi < nq && (kt + j) < Nk[qi];
        const float sc = valid ? __fmul_rn(s[i], ks) : -INFINITY;
        const float mt = warp_max(sc);
        const float mo = Ms[qi];
        const float mn = fmaxf(mo, mt);
        float p = 0.0f, alpha = 1.0f;
        if (mn != -INFINITY) {
          p = valid ? exp_malkin(__fsub_rn(sc, mn)) : 0.0f;
          alpha = mo == -INFINITY ? 0.0f : exp_malkin(__fsub_rn(mo, mn));
        }
        const float ps = warp_sum(p);
        Ps[qi * (kKT + 4) + j] = __fmul_rn(p, vs);
        __syncwarp();
        if (lane == 0) {
          Ms[qi] = mn;
          Ls[qi] = __fmaf_rn(Ls[qi], alpha, ps);
          Al[qi] = alpha;
        }
      }
    }
    __syncthreads();
    // o = o * alpha + sum_j (p_j * vs_j) * v_j
    {
      const int dq = tid % DV, qg = tid / DV;
#pragma unroll
      for (int i = 0; i < QI; ++i) {
        const int qi = qg + QG * i;
        if (qi < kQMax) {
          const float al = Al[qi];
          o[i][0] *= al, o[i][1] *= al, o[i][2] *= al, o[i][3] *= al;
        }
      }
      for (int j = 0; j < nk; j += 4) {
        float4 v4[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) v4[jj] = *reinterpret_cast<const float4*>(Vf + (j + jj) * DP + 4 * dq);
#pragma unroll
        for (int i = 0; i < QI; ++i) {
          const int qi = qg + QG * i;
          if (qi < kQMax) {
            const float4 p4 = *reinterpret_cast<const float4*>(Ps + qi * (kKT + 4) + j);
            const float pp[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              o[i][0] = __fmaf_rn(pp[jj], v4[jj].x, o[i][0]);
              o[i][1] = __fmaf_rn(pp[jj], v4[jj].y, o[i][1]);
              o[i][2] = __fmaf_rn(pp[jj], v4[jj].z, o[i][2]);
              o[i][3] = __fmaf_rn(pp[jj], v4[jj].w, o[i][3]);
            }
          }
        }
      }
    }
    __syncthreads();
  }
  // Partials: [((sg * n_chunks + chunk) * KV + kvh) * qmax + qi][D + 2] = o[D], m, l.
  {
    const int dq = tid % DV, qg = tid / DV;
    float* part = a.p.part + ((static_cast<size_t>(sg) * a.p.n_chunks + chunk) * a.KV + kvh) * kQMax * (D + 2);
#pragma unroll
    for (int i = 0; i < QI; ++i) {
      const int qi = qg + QG * i;
      if (qi < nq) {
        float* pr = part + static_cast<size_t>(qi) * (D + 2);
        pr[4 * dq + 0] = o[i][0];
        pr[4 * dq + 1] = o[i][1];
        pr[4 * dq + 2] = o[i][2];
        pr[4 * dq + 3] = o[i][3];
        if (dq == 0) {
          pr[D] = Ms[qi];
          pr[D + 1] = Ls[qi];
        }
      }
    }
  }
}

// ---------------- combine chunks + extra (ancestor) keys ----------------
// grid (n, ceil(H / 4)), block 128: one warp per (token, head).
template <int D>
__global__ void k_attn_combine(PartArgs a, const int32_t* __restrict__ tok_sg, float* __restrict__ out) {
  constexpr int PER = D / 32;
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + (threadIdx.x >> 5);
  if (h >= a.H) return;
  const int kvh = h / a.G;
  const int sg = tok_sg[t];
  const int t0 = a.p.sg_first[sg], t1 = a.p.sg_first[sg + 1];
  int maxk = 0;
  for (int u = t0; u < t1; ++u) maxk = max(maxk, a.p.n_keys[u]);
  const int nck = (maxk + a.p.chunk - 1) / a.p.chunk;
  const int qi = (t - t0) * a.G + (h - kvh * a.G);
  const float* part = a.p.part + (static_cast<size_t>(sg) * a.p.n_chunks * a.KV + kvh) * kQMax * (D + 2) +
                      static_cast<size_t>(qi) * (D + 2);
  const size_t cstride = static_cast<size_t>(a.KV) * kQMax * (D + 2);
  const int base = a.p.kv_base[t];
  const int e0 = a.p.anc_off[t], e1 = a.p.anc_off[t + 1];
  // extra-key scores
  const float* qv = a.q + (static_cast<size_t>(t) * a.H + h) * D;
  float q[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) q[m] = qv[lane + 32 * m];
  float M = -INFINITY;
  for (int c = 0; c < nck; ++c) M = fmaxf(M, part[c * cstride + D]);
  const int8_t* kh = a.L.k + static_cast<size_t>(kvh) * a.L.n_rows * D;
  const int8_t* vh = a.L.v + static_cast<size_t>(kvh) * a.L.n_rows * D;
  const float* ksh = a.L.ks + static_cast<size_t>(kvh) * a.L.n_rows;
  const float* vsh = a.L.vs + static_cast<size_t>(kvh) * a.L.n_rows;
  float se_reg = -INFINITY;  // score of extra e0 + lane (<= 32 extras per token handled per pass)
  for (int e = e0; e < e1; ++e) {
    const size_t row = static_cast<size_t>(base) + a.p.anc[e];
    float s = 0.0f;
#pragma unroll
    for (int m = 0; m < PER; ++m) s = __fmaf_rn(q[m], static_cast<float>(kh[row * D + lane + 32 * m]), s);
    s = warp_sum(s);
    s = __fmul_rn(s, __fmul_rn(ksh[row], a.scale));
    if (((e - e0) & 31) == lane) se_reg = s;
    M = fmaxf(M, s);
  }
  float o[PER];
#pragma unroll
  for (int m = 0; m < PER; ++m) o[m] = 0.0f;
  float L = 0.0f;
  for (int c = 0; c < nck; ++c) {
    const float* pr = part + c * cstride;
    const float mc = pr[D];
    if (mc == -INFINITY) continue;
    const float f = exp_malkin(__fsub_rn(mc, M));
    L = __fmaf_rn(pr[D + 1], f, L);
#pragma unroll
    for (int m = 0; m < PER; ++m) o[m] = __fmaf_rn(pr[lane + 32 * m], f, o[m]);
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
  float* dst = out + (static_cast<size_t>(t) * a.H + h) * D;
#pragma unroll
  for (int m = 0; m < PER; ++m) dst[lane + 32 * m] = __fmul_rn(o[m], inv);
}

template <int D>
size_t part_smem() {
  constexpr int DP = D + 4;
  return sizeof(float) * (kQMax * DP + 2 * kKT * DP + kQMax * (kKT + 4) + 3 * kQMax) + sizeof(int) * kQMax;
}

template <int D>
void run_attention(const float* q, int H, int KV, float scale, const AttnLayer& L, const AttnPlan& p, float* out,
                   cudaStream_t s) {
  PartArgs a{q, H, KV, H / KV, scale, L, p};
  const size_t smem = part_smem<D>();
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attn_part<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    attr = true;
  }
  if (p.n_sg > 0 && p.n_chunks > 0) {
    const dim3 g1(p.n_chunks, p.n_sg, KV);
    k_attn_part<D><<<g1, kThreads, smem, s>>>(a);
  }
  const dim3 g2(p.n, (H + 3) / 4);
  k_attn_combine<D><<<g2, 128, 0, s>>>(a, p.tok_sg, out);
}

}  // namespace

int attn_qmax() { return kQMax; }

size_t attn_part_floats(int n_sg, int n_chunks, int KV, int D) {
  return static_cast<size_t>(n_sg) * n_chunks * KV * kQMax * (D + 2);
}

void launch_qkv_post(const float* y, int64_t ldy, int n, int H, int KV, int D, const float* q_norm, const float* k_norm,
                     float eps, const float* rope_cs, const int32_t* rpos, const int32_t* kv_at, float* q_out,
                     const AttnLayer& L, cudaStream_t s) {
  const dim3 grid(n, (H + 2 * KV + 3) / 4);
  switch (D) {
    case 64:
      k_qkv_post<64><<<grid, 128, 0, s>>>(y, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at, q_out, L);
      break;
    case 128:
      k_qkv_post<128><<<grid, 128, 0, s>>>(y, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at, q_out, L);
      break;
    case 256:
      k_qkv_post<256><<<grid, 128, 0, s>>>(y, ldy, n, H, KV, q_norm, k_norm, eps, rope_cs, rpos, kv_at, q_out, L);
      break;
    default:
      break;
  }
}

void launch_attention(const float* q, int H, int KV, int D, float scale, const AttnLayer& L, const AttnPlan& p,
                      float* out, cudaStream_t s) {
  switch (D) {
    case 64:
      run_attention<64>(q, H, KV, scale, L, p, out, s);
      break;
    case 128:
      run_attention<128>(q, H, KV, scale, L, p, out, s);
      break;
    case 256:
      run_attention<256>(q, H, KV, scale, L, p, out, s);
      break;
    default:
      break;
  }
}

}  // namespace mkb
