// Tensor-parallel sum of the row-split GEMM partials (attention output and ffn down) over NVLink peer memory:
// the B200-native replacement of "sum the split-K slices, then ncclAllReduce" (malkin has no tensor parallelism; the
// sum is the allreduce of the Megatron split of wo / down).
//
// Every rank owns an exchange buffer (two halves of `cap` floats, a flag word per rank, an epoch counter and a CTA
// arrival counter), mapped into every other rank with CUDA IPC. One call is two kernels on the rank's stream:
//   publish: sums this rank's split-K slices (slice order) into half (epoch & 1) of its own buffer; each CTA
//            fences system-wide and counts its arrival, and the last one advances the epoch and stores it with
//            release semantics into flag[rank] of every rank's buffer;
//   gather:  waits (bounded) until every rank's flag in this rank's buffer has reached the epoch, then sums the
//            ranks' halves in rank order 0..size-1, so every rank gets bit-identical results.
// A half is rewritten two calls later; by then every rank has published the call in between, which it does only
// after its gather of the earlier call finished, so no rank still reads it. A wait that runs out records
// kErrTpWait in the status word and the kernel returns (a rank that died or never launched); a wait gives up after
// x.wait_polls polls.
// Two-shot (opt-in): after publish, reduce sums this rank's 1/size of the rows over all ranks into its red half and
// releases flags2; allgather waits for every rank's flags2 and copies each rank's reduced rows. Each rank reads
// 2 (size - 1) / size of the data from peers (one-shot: size - 1 times it); the sums are the same, bit for bit. The
// red half of a call is rewritten two calls later, after every rank published the next call (after its allgather).
#include <cuda_runtime.h>

#include <algorithm>

#include "kernels.hpp"

namespace mkb {

namespace {

constexpr unsigned kTpCallFailed = 0x80000000u;  // counter2 bit: a CTA of this reduce gave up waiting

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void k_tp_publish(TpExchange x, Slices src, int64_t ld, int n, int cols) {
  const int e = *x.epoch + 1;  // the previous call's kernels have finished (stream order)
  float* dst = x.data[x.rank] + static_cast<int64_t>(e & 1) * x.cap;
  const int c4 = cols / 4;
  const int64_t total4 = static_cast<int64_t>(n) * c4;  // cols % 4 == 0
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / c4, c = (i % c4) * 4;
    const float4* p = reinterpret_cast<const float4*>(src.p + t * ld + c);
    float4 v = p[0];
    for (int s = 1; s < src.n; ++s) {
      const float4 u = *reinterpret_cast<const float4*>(src.p + s * src.stride + t * ld + c);
      v.x = __fadd_rn(v.x, u.x);
      v.y = __fadd_rn(v.y, u.y);
      v.z = __fadd_rn(v.z, u.z);
      v.w = __fadd_rn(v.w, u.w);
    }
    reinterpret_cast<float4*>(dst)[i] = v;
  }
  // the CTA's stores, made visible to the CTA by the barrier, are ordered before the arrival by thread 0's fence
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned prev = atomicAdd(x.counter, 1u);
    if (prev == gridDim.x - 1) {  // every CTA's part of the half is written and fenced
      __threadfence_system();
      *x.counter = 0;
      *x.epoch = e;
      for (int r = 0; r < x.size; ++r) st_release_sys(x.flags[r] + x.rank, e);
    }
  }
}

// Bounded wait (thread 0 of the CTA) until flags[0..size) all reach e; false (and status) if one never does.
__device__ bool wait_flags(const int* flags, int size, int e, uint32_t polls, int* status) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int r = 0; r < size && ok; ++r) {
      uint32_t it = 0;
      while (ld_acquire_sys(flags + r) < e) {
        if (++it >= polls) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
    if (!ok && status) atomicCAS(status, 0, kErrTpWait);
    ready = ok;
  }
  __syncthreads();
  return ready != 0;
}

__global__ void k_tp_gather(TpExchange x, int n, int cols, float* __restrict__ dst, int* status) {
  const int e = *x.epoch;  // set by this rank's publish (stream order)
  if (!wait_flags(x.flags[x.rank], x.size, e, x.wait_polls, status)) return;
  const int64_t off = static_cast<int64_t>(e & 1) * x.cap;
  const int64_t total4 = static_cast<int64_t>(n) * cols / 4;  // cols % 4 == 0
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 v[kMaxTp];
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r)  // every rank's load in flight at once
      if (r < x.size) v[r] = __ldcv(reinterpret_cast<const float4*>(x.data[r] + off) + i);
    float4 acc = v[0];
#pragma unroll
    for (int r = 1; r < kMaxTp; ++r)
      if (r < x.size) {
        acc.x = __fadd_rn(acc.x, v[r].x);
        acc.y = __fadd_rn(acc.y, v[r].y);
        acc.z = __fadd_rn(acc.z, v[r].z);
        acc.w = __fadd_rn(acc.w, v[r].w);
      }
    reinterpret_cast<float4*>(dst)[i] = acc;
  }
}

// Rows of rank q's share of the reduction, in float4 units: [q * total4 / size, (q + 1) * total4 / size).
__device__ __forceinline__ int64_t share_begin(int64_t total4, int q, int size) { return total4 * q / size; }

__global__ void k_tp_reduce(TpExchange x, int n, int cols, int* status) {
  const int e = *x.epoch;  // set by this rank's publish (stream order)
  const bool ok = wait_flags(x.flags[x.rank], x.size, e, x.wait_polls, status);
  const int64_t off = static_cast<int64_t>(e & 1) * x.cap;
  const int64_t total4 = static_cast<int64_t>(n) * cols / 4;
  const int64_t b = share_begin(total4, x.rank, x.size), end = ok ? share_begin(total4, x.rank + 1, x.size) : b;
  for (int64_t i = b + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < end;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 v[kMaxTp];
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r)
      if (r < x.size) v[r] = __ldcv(reinterpret_cast<const float4*>(x.data[r] + off) + i);
    float4 acc = v[0];
#pragma unroll
    for (int r = 1; r < kMaxTp; ++r)
      if (r < x.size) {
        acc.x = __fadd_rn(acc.x, v[r].x);
        acc.y = __fadd_rn(acc.y, v[r].y);
        acc.z = __fadd_rn(acc.z, v[r].z);
        acc.w = __fadd_rn(acc.w, v[r].w);
      }
    reinterpret_cast<float4*>(x.red[x.rank] + off)[i] = acc;
  }
  // Every CTA arrives, also one whose wait gave up (it marks the call failed first), so the counter is back at zero
  // for the next call; the share is released to the peers only when every CTA reduced its part.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (!ok) atomicOr(x.counter2, kTpCallFailed);
    const unsigned prev = atomicAdd(x.counter2, 1u);
    if ((prev & ~kTpCallFailed) == gridDim.x - 1) {  // last arrival: the whole share is reduced and fenced
      __threadfence_system();
      *x.counter2 = 0;
      if (!(prev & kTpCallFailed))
        for (int r = 0; r < x.size; ++r) st_release_sys(x.flags2[r] + x.rank, e);
    }
  }
}

__global__ void k_tp_allgather(TpExchange x, int n, int cols, float* __restrict__ dst, int* status) {
  const int e = *x.epoch;
  if (!wait_flags(x.flags2[x.rank], x.size, e, x.wait_polls, status)) return;
  const int64_t off = static_cast<int64_t>(e & 1) * x.cap;
  const int64_t total4 = static_cast<int64_t>(n) * cols / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int q = static_cast<int>(i * x.size / total4);  // owner of row i: the share with begin <= i < end
    while (q > 0 && i < share_begin(total4, q, x.size)) --q;
    while (q + 1 < x.size && i >= share_begin(total4, q + 1, x.size)) ++q;
    reinterpret_cast<float4*>(dst)[i] = __ldcv(reinterpret_cast<const float4*>(x.red[q] + off) + i);
  }
}

int tp_grid(int64_t items, int per_cta) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t g = (items + per_cta - 1) / per_cta;
  return static_cast<int>(g < 1 ? 1 : (g > 4 * sms ? 4 * sms : g));
}

}  // namespace

void launch_tp_publish(const TpExchange& x, Slices src, int64_t ld, int n, int cols, cudaStream_t s) {
  if (n <= 0) return;
  k_tp_publish<<<tp_grid(static_cast<int64_t>(n) * cols / 4, 256), 256, 0, s>>>(x, src, ld, n, cols);
}

void launch_tp_gather(const TpExchange& x, int n, int cols, float* dst, int* status, cudaStream_t s) {
  if (n <= 0) return;
  k_tp_gather<<<tp_grid(static_cast<int64_t>(n) * cols / 4, 256), 256, 0, s>>>(x, n, cols, dst, status);
}

void launch_tp_reduce(const TpExchange& x, int n, int cols, int* status, cudaStream_t s) {
  if (n <= 0) return;
  k_tp_reduce<<<tp_grid(static_cast<int64_t>(n) * cols / 4 / x.size + 1, 256), 256, 0, s>>>(x, n, cols, status);
}

void launch_tp_allgather(const TpExchange& x, int n, int cols, float* dst, int* status, cudaStream_t s) {
  if (n <= 0) return;
  k_tp_allgather<<<tp_grid(static_cast<int64_t>(n) * cols / 4, 256), 256, 0, s>>>(x, n, cols, dst, status);
}

namespace {
// float4 per thread: el % 4 == 0 (whole 16-row panels per rank).
__global__ void k_tp_concat(const float4* __restrict__ src, int tp, int n, int el4, float4* __restrict__ dst) {
  const int64_t e4 = static_cast<int64_t>(tp) * el4, total = static_cast<int64_t>(n) * e4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / e4, e = i % e4, r = e / el4;
    dst[i] = src[(r * n + t) * el4 + (e - r * el4)];
  }
}
}  // namespace

void launch_tp_concat(const float* src, int tp, int n, int el, float* dst, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(n) * tp * el / 4;
  if (total <= 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 8));
  k_tp_concat<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(src), tp, n, el / 4,
                                     reinterpret_cast<float4*>(dst));
}

}  // namespace mkb
