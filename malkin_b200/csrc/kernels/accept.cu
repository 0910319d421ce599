// Acceptance on device, no logits round trip: per-row argmax / top-k candidates over the logits, then per request
// malkin's greedy tree walk (Engine::accept_greedy, engine.cpp:441-479) or the exact rejection chain
// (Engine::accept_sampled + Sampler::distribution / verify / draw, engine.cpp:482-507, sampler.cpp:22-97), and the
// KV moves of the accepted tree path (Model::move_kv).
//
// Tie rules: argmax takes the lowest index of the maximum (std::max_element). Top-k ranks by (value desc, index asc);
// malkin's std::partial_sort leaves the order of equal values unspecified, so rows with ties at the k-th value may
// keep different (equally valid) members there.
#include <cuda_runtime.h>

#include <cfloat>

#include "common.cuh"
#include "kernels.hpp"

namespace mkb {

namespace {

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// ---------------- argmax ----------------
__global__ void k_argmax(const float* __restrict__ logits, int64_t ld, int V, int vbase, int kc, float* __restrict__ ov,
                         int32_t* __restrict__ oi) {
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* l = logits + static_cast<size_t>(row) * ld;
  float bv = -INFINITY;
  int bi = INT32_MAX;
  // (value, lowest index) is order independent, so the row may be read in any order: 16-byte loads, four in flight
  // per thread, when the row is 16-byte aligned; the scalar tail (and unaligned rows) after.
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(l) & 15) == 0) {
    const float4* l4 = reinterpret_cast<const float4*>(l);
    const int n4 = V / 4;
    const int step = static_cast<int>(blockDim.x);
    for (int b = tid; b < n4; b += 4 * step) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        q[u] = b + u * step < n4 ? l4[b + u * step] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (b + u * step >= n4) break;
        const int i = 4 * (b + u * step);
        if (better(q[u].x, i, bv, bi)) bv = q[u].x, bi = i;
        if (better(q[u].y, i + 1, bv, bi)) bv = q[u].y, bi = i + 1;
        if (better(q[u].z, i + 2, bv, bi)) bv = q[u].z, bi = i + 2;
        if (better(q[u].w, i + 3, bv, bi)) bv = q[u].w, bi = i + 3;
      }
    }
    done = n4 * 4;
  }
  for (int i = done + tid; i < V; i += blockDim.x) {
    const float v = l[i];
    if (better(v, i, bv, bi)) bv = v, bi = i;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(v, i, bv, bi)) bv = v, bi = i;
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((tid & 31) == 0) sv[tid >> 5] = bv, si[tid >> 5] = bi;
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) bv = sv[w], bi = si[w];
    ov[static_cast<size_t>(row) * kc] = bv;
    oi[static_cast<size_t>(row) * kc] = bi == INT32_MAX ? vbase : bi + vbase;
  }
}

// ---------------- top-k: 4-pass radix select on order-preserving keys ----------------
__device__ __forceinline__ uint32_t fkey(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kTopkThreads = 1024;

__global__ void __launch_bounds__(kTopkThreads) k_topk(const float* __restrict__ logits, int64_t ld, int V, int vbase,
                                                        int k, int kc, float* __restrict__ ov, int32_t* __restrict__ oi) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_krem, s_cnt;
  __shared__ int wsum[32];
  __shared__ float cv[MK_TOPK_CAP];
  __shared__ int ci[MK_TOPK_CAP];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* l = logits + static_cast<size_t>(row) * ld;
  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_krem = k;
    s_cnt = 0;
  }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < V; i += blockDim.x) {
      const uint32_t key = fkey(l[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int krem = s_krem;
      int b = 255;
      for (; b > 0; --b) {
        if (static_cast<int>(hist[b]) >= krem) break;
        krem -= static_cast<int>(hist[b]);
      }
      s_krem = krem;
      s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int need_eq = s_krem;  // elements equal to T to take (lowest indices); k - need_eq are greater
  for (int i = tid; i < V; i += blockDim.x) {
    const float v = l[i];
    if (fkey(v) > T) {
      const int pos = atomicAdd(&s_cnt, 1);
      cv[pos] = v;
      ci[pos] = i;
    }
  }
  __syncthreads();
  // Equal keys in index order: thread t scans the contiguous range [t * per, (t + 1) * per).
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int lo = tid * per, hi = min(V, lo + per);
  int my = 0;
  for (int i = lo; i < hi; ++i) my += fkey(l[i]) == T;
  // exclusive scan of my over the block
  int incl = my;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if ((tid & 31) >= o) incl += y;
  }
  if ((tid & 31) == 31) wsum[tid >> 5] = incl;
  __syncthreads();
  if (tid < 32) {
    int w = tid < static_cast<int>(blockDim.x >> 5) ? wsum[tid] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (tid >= o) w += y;
    }
    wsum[tid] = w;  // inclusive warp totals
  }
  __syncthreads();
  int rank = incl - my + ((tid >> 5) ? wsum[(tid >> 5) - 1] : 0);
  const int gt = k - need_eq;
  for (int i = lo; i < hi && rank < need_eq; ++i) {
    const float v = l[i];
    if (fkey(v) == T) {
      cv[gt + rank] = v;
      ci[gt + rank] = i;
      ++rank;
    }
  }
  __syncthreads();
  if (tid < k) {
    const float v = cv[tid];
    const int i = ci[tid];
    int r = 0;
    for (int j = 0; j < k; ++j) r += better(cv[j], ci[j], v, i);
    ov[static_cast<size_t>(row) * kc + r] = v;
    oi[static_cast<size_t>(row) * kc + r] = i + vbase;
  }
}

// ---------------- merge tensor-parallel candidate lists ----------------
__global__ void k_merge(const float* __restrict__ iv, const int32_t* __restrict__ ii, int tp, int m, int k, int kc,
                        float* __restrict__ ov, int32_t* __restrict__ oi) {
  extern __shared__ float sm[];
  const int row = blockIdx.x, N = tp * k;
  float* v = sm;
  int* id = reinterpret_cast<int*>(sm + N);
  for (int x = threadIdx.x; x < N; x += blockDim.x) {
    const int r = x / k, j = x % k;
    v[x] = iv[(static_cast<size_t>(r) * m + row) * kc + j];
    id[x] = ii[(static_cast<size_t>(r) * m + row) * kc + j];
  }
  __syncthreads();
  for (int x = threadIdx.x; x < N; x += blockDim.x) {
    int r = 0;
    for (int y = 0; y < N; ++y) r += better(v[y], id[y], v[x], id[x]);
    if (r < k) {
      ov[static_cast<size_t>(row) * kc + r] = v[x];
      oi[static_cast<size_t>(row) * kc + r] = id[x];
    }
  }
}

// ---------------- acceptance ----------------
struct Dist {
  int n;
  float p[MK_TOPK_CAP];
  int id[MK_TOPK_CAP];
};

// Sampler::distribution (sampler.cpp:22-62) from the row's top-k candidates (sorted value desc).
__device__ void distribution(const float* cv, const int32_t* ci, int k, float temp, float top_p, float min_p, Dist& out) {
  float e[MK_TOPK_CAP];
  const float mx = cv[0];
  double sum = 0.0;
  for (int j = 0; j < k; ++j) {
    const float z = __fdiv_rn(__fsub_rn(cv[j], mx), temp);
    e[j] = static_cast<float>(exp(static_cast<double>(z)));
    sum += static_cast<double>(e[j]);
  }
  const double floor = static_cast<double>(min_p) * static_cast<double>(e[0]);
  double kept = 0.0;
  int n = 0;
  for (; n < k; ++n) {
    if (n > 0 && static_cast<double>(e[n]) < floor) break;
    kept += static_cast<double>(e[n]);
    if (kept >= static_cast<double>(top_p) * sum) {
      ++n;
      break;
    }
  }
  n = max(n, 1);
  double total = 0.0;
  for (int j = 0; j < n; ++j) total += static_cast<double>(e[j]);
  out.n = n;
  for (int j = 0; j < n; ++j) {
    out.p[j] = static_cast<float>(static_cast<double>(e[j]) / total);
    out.id[j] = ci[j];
  }
}

__device__ float prob_of(const float* p, const int* id, int n, int d) {
  for (int j = 0; j < n; ++j)
    if (id[j] == d) return p[j];
  return 0.0f;
}

// Sampler::draw (sampler.cpp:64-72): no uniform consumed for a one-entry distribution.
__device__ int draw(const float* p, const int* id, int n, const double* U, int nu, int& u, int& status) {
  if (n == 1) return id[0];
  if (u >= nu) {
    status = 1;
    return id[0];
  }
  double r = U[u++];
  for (int j = 0; j < n; ++j) {
    r -= static_cast<double>(p[j]);
    if (r <= 0.0) return id[j];
  }
  return id[n - 1];
}

__global__ void k_accept(const AcceptReq* __restrict__ reqs, const float* __restrict__ cv,
                         const int32_t* __restrict__ ci, int kc, const int32_t* __restrict__ chain,
                         const int32_t* __restrict__ alt, const float* __restrict__ q_p, const int32_t* __restrict__ q_id,
                         const int32_t* __restrict__ q_n, const double* __restrict__ U, int n_ctx,
                         AcceptOut* __restrict__ out, int32_t* __restrict__ from, int32_t* __restrict__ to,
                         int32_t* __restrict__ count) {
  if (threadIdx.x != 0) return;
  const int r = blockIdx.x;
  const AcceptReq q = reqs[r];
  AcceptOut o{};
  const int P = q.cache_len;
  int moves = 0;
  if (q.greedy) {
    const int64_t base = static_cast<int64_t>(q.seq) * n_ctx;
    int size = P + 1, cur = 0, n = 0;
    bool bonus = false;
    for (int i = 0; i < q.kk; ++i) {
      const int a = ci[static_cast<size_t>(q.row0 + cur) * kc];
      int slot = -1;
      if (a == chain[q.chain_off + i])
        slot = 1 + 2 * i;
      else if (a == alt[q.chain_off + i])
        slot = 2 + 2 * i;
      if (slot < 0) {
        o.next = a;
        bonus = true;
        break;
      }
      from[r * 32 + moves] = static_cast<int32_t>(base + P + slot);
      to[r * 32 + moves] = static_cast<int32_t>(base + size);
      ++moves;
      ++size;
      o.ids[n++] = a;
      cur = slot;
      if (slot == 2 + 2 * i) break;
    }
    if (!bonus) o.next = ci[static_cast<size_t>(q.row0 + cur) * kc];
    o.n_acc = n;
    o.cache_len = size;
    o.last_node = cur;
  } else {
    Dist p;
    int u = 0, i = 0, n = 0, status = 0, qo = q.q_off;
    const double* Ur = U + q.u_off;
    for (; i < q.kk; ++i) {
      const size_t row = static_cast<size_t>(q.row0 + i) * kc;
      distribution(cv + row, ci + row, q.top_k, q.temperature, q.top_p, q.min_p, p);
      const int d = chain[q.chain_off + i];
      const int qn = q_n[q.qn_off + i];
      const float pd = prob_of(p.p, p.id, p.n, d), qd = prob_of(q_p + qo, q_id + qo, qn, d);
      if (u >= q.n_u) {
        status = 1;
        break;
      }
      const double uu = Ur[u++];
      const bool ok = qd > 0.0f && uu * static_cast<double>(qd) < static_cast<double>(pd);
      if (ok) {
        o.ids[n++] = d;
        qo += qn;
        continue;
      }
      float rp[MK_TOPK_CAP];
      int rid[MK_TOPK_CAP], nr = 0;
      double total = 0.0;
      for (int j = 0; j < p.n; ++j) {
        const float rr = __fsub_rn(p.p[j], prob_of(q_p + qo, q_id + qo, qn, p.id[j]));
        if (rr > 0.0f) {
          rp[nr] = rr;
          rid[nr++] = p.id[j];
          total += static_cast<double>(rr);
        }
      }
      int t;
      if (nr == 0) {
        t = draw(p.p, p.id, p.n, Ur, q.n_u, u, status);
      } else {
        for (int j = 0; j < nr; ++j) rp[j] = static_cast<float>(static_cast<double>(rp[j]) / total);
        t = draw(rp, rid, nr, Ur, q.n_u, u, status);
      }
      o.next = t;
      break;
    }
    if (i == q.kk && status == 0) {
      const size_t row = static_cast<size_t>(q.row0 + q.kk) * kc;
      distribution(cv + row, ci + row, q.top_k, q.temperature, q.top_p, q.min_p, p);
      o.next = draw(p.p, p.id, p.n, Ur, q.n_u, u, status);
    }
    o.n_acc = n;
    o.cache_len = P + 1 + n;
    o.u_used = u;
    o.last_node = n;
    o.status = status;
  }
  count[r] = moves;
  out[r] = o;
}

// ---------------- log-sum-exp for perplexity ----------------
// Engine::perplexity (engine.cpp:545-552) per logits row: sum over the row of exp(double(l[v] - mx)) with the row's
// maximum mx (over every vocabulary shard), and the row's logit of its target token when this shard holds it (else 0).
// The double sum is a tree over the block, not malkin's sequential loop: the two agree to about 1e-15 relative.
__global__ void k_row_lse(const float* __restrict__ logits, int64_t ld, int V, int vbase, const float* __restrict__ mx,
                          const int32_t* __restrict__ tgt, double* __restrict__ sum, float* __restrict__ tl) {
  __shared__ double part[32];
  const int row = blockIdx.x, tid = threadIdx.x;
  const float* l = logits + static_cast<size_t>(row) * ld;
  const float m = mx[row];
  double s = 0.0;
  for (int i = tid; i < V; i += blockDim.x) s += exp(static_cast<double>(__fsub_rn(l[i], m)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((tid & 31) == 0) part[tid >> 5] = s;
  __syncthreads();
  if (tid < 32) {
    s = tid < static_cast<int>(blockDim.x >> 5) ? part[tid] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (tid == 0) {
      sum[row] = s;
      const int t = tgt[row] - vbase;
      tl[row] = t >= 0 && t < V ? l[t] : 0.0f;
    }
  }
}

}  // namespace

void launch_row_lse(const float* logits, int64_t ld, int m, int V, int vbase, const float* mx, const int32_t* tgt,
                    double* sum, float* tl, cudaStream_t s) {
  if (m > 0) k_row_lse<<<m, 512, 0, s>>>(logits, ld, V, vbase, mx, tgt, sum, tl);
}

void launch_argmax(const float* logits, int64_t ld, int m, int V, int vbase, float* best_v, int32_t* best_i,
                   cudaStream_t s) {
  launch_argmax_kc(logits, ld, m, V, vbase, 1, best_v, best_i, s);
}

void launch_argmax_kc(const float* logits, int64_t ld, int m, int V, int vbase, int kc, float* best_v, int32_t* best_i,
                      cudaStream_t s) {
  if (m > 0) k_argmax<<<m, 1024, 0, s>>>(logits, ld, V, vbase, kc, best_v, best_i);
}

void launch_topk(const float* logits, int64_t ld, int m, int V, int vbase, int k, int kc, float* cand_v,
                 int32_t* cand_i, cudaStream_t s) {
  if (m > 0) k_topk<<<m, kTopkThreads, 0, s>>>(logits, ld, V, vbase, k, kc, cand_v, cand_i);
}

void launch_merge_cand(const float* in_v, const int32_t* in_i, int tp, int m, int k, int kc, float* out_v,
                       int32_t* out_i, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(tp) * k * (sizeof(float) + sizeof(int));
  if (m > 0) k_merge<<<m, 256, smem, s>>>(in_v, in_i, tp, m, k, kc, out_v, out_i);
}

void launch_accept(const AcceptReq* reqs, int n_req, const float* cand_v, const int32_t* cand_i, int kc,
                   const int32_t* chain, const int32_t* alt, const float* q_p, const int32_t* q_id, const int32_t* q_n,
                   const double* uniforms, int n_ctx, AcceptOut* out, int32_t* from, int32_t* to, int32_t* count,
                   cudaStream_t s) {
  if (n_req > 0)
    k_accept<<<n_req, 32, 0, s>>>(reqs, cand_v, cand_i, kc, chain, alt, q_p, q_id, q_n, uniforms, n_ctx, out, from, to,
                                  count);
}

}  // namespace mkb
