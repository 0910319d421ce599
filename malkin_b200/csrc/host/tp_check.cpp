// mk_tp_exchange_check: the tensor-parallel rank-sum kernels of one rank, run on one device against emulated peers.
//
// Rank 0's exchange buffer and those of `size - 1` emulated ranks all live on the current device. Before each call
// the host plays the peers: it writes their partial sums and the flags they would release (and, two-shot, their
// reduced shares), except for a rank marked absent for that call. Rank 0 then runs its real publish + gather (or
// publish + reduce + allgather) on one stream, exactly as Model::tp_sum launches them. No kernel waits on another
// kernel: every flag a wait can succeed on is written by the host before the launch, and a missing one makes the
// bounded wait give up after `wait_polls` polls with kErrTpWait.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "../../../include/malkin_b200.h"
#include "../kernels/kernels.hpp"
#include "model.hpp"

namespace mkb {

namespace {

// Float4 share boundaries of the two-shot reduce (k_tp_reduce's share_begin).
int64_t share_begin(int64_t total4, int q, int size) { return total4 * q / size; }

}  // namespace

void tp_exchange_check(int size, bool twoshot, int n, int cols, int n_calls, const int* absent, uint32_t wait_polls,
                       const float* parts, float* out, int* call_status) {
  if (size < 2 || size > kMaxTp) throw ArgError("tp_exchange_check: size must be 2..8");
  if (n <= 0 || cols <= 0 || cols % 4 || n_calls <= 0 || wait_polls == 0)
    throw ArgError("tp_exchange_check: bad shape (n > 0, cols % 4 == 0, calls > 0, wait_polls > 0)");
  if (!parts || !out || !call_status) throw ArgError("tp_exchange_check: null buffer");
  const int64_t elems = static_cast<int64_t>(n) * cols, total4 = elems / 4;
  const size_t cap = static_cast<size_t>((elems + 63) / 64 * 64);
  // per rank, the layout Model::setup_tp_exchange maps: [data 2 halves | red 2 halves | flags | flags2 | epoch ...]
  const size_t bytes = 4 * cap * sizeof(float) + 2 * kMaxTp * sizeof(int) + 128;
  std::vector<DevBuf> bufs;
  for (int r = 0; r < size; ++r) {
    bufs.emplace_back(bytes);
    cuda_check(cudaMemset(bufs.back().get(), 0, bytes), "tp check memset");
  }
  TpExchange x;
  for (int r = 0; r < size; ++r) {
    auto* base = bufs[static_cast<size_t>(r)].get<uint8_t>();
    x.data[r] = reinterpret_cast<float*>(base);
    x.red[r] = reinterpret_cast<float*>(base + 2 * cap * sizeof(float));
    x.flags[r] = reinterpret_cast<int*>(base + 4 * cap * sizeof(float));
    x.flags2[r] = x.flags[r] + kMaxTp;
  }
  auto* own = bufs[0].get<uint8_t>() + 4 * cap * sizeof(float) + 2 * kMaxTp * sizeof(int);
  x.epoch = reinterpret_cast<int*>(own);
  x.counter = reinterpret_cast<unsigned*>(own + 32);
  x.counter2 = reinterpret_cast<unsigned*>(own + 64);
  x.rank = 0;
  x.size = size;
  x.cap = static_cast<int64_t>(cap);
  x.wait_polls = wait_polls;

  DevBuf d_part(static_cast<size_t>(elems) * 4), d_out(static_cast<size_t>(elems) * 4), d_status(sizeof(int));
  cuda_check(cudaMemset(d_status.get(), 0, sizeof(int)), "tp check memset");
  std::vector<float> red(static_cast<size_t>(elems));
  for (int k = 0; k < n_calls; ++k) {
    const int e = k + 1;  // rank 0's publish advances its epoch once per call, also in a call that later fails
    const size_t half = static_cast<size_t>(e & 1) * cap;
    const float* pk = parts + static_cast<size_t>(k) * size * elems;
    for (int r = 1; r < size; ++r) {
      if (absent && absent[k] == r) continue;
      cuda_check(cudaMemcpy(x.data[r] + half, pk + static_cast<size_t>(r) * elems, elems * 4, cudaMemcpyHostToDevice),
                 "tp check peer half");
      cuda_check(cudaMemcpy(x.flags[0] + r, &e, sizeof e, cudaMemcpyHostToDevice), "tp check peer flag");
    }
    if (twoshot) {
      // every present peer's reduced share: the sum over ranks in rank order, as k_tp_reduce forms it
      for (int64_t i = 0; i < elems; ++i) {
        float acc = pk[i];
        for (int r = 1; r < size; ++r) acc += pk[static_cast<size_t>(r) * elems + i];
        red[static_cast<size_t>(i)] = acc;
      }
      for (int q = 1; q < size; ++q) {
        if (absent && absent[k] == q) continue;
        const int64_t b = share_begin(total4, q, size) * 4, end = share_begin(total4, q + 1, size) * 4;
        cuda_check(cudaMemcpy(x.red[q] + half + b, red.data() + b, (end - b) * 4, cudaMemcpyHostToDevice),
                   "tp check peer share");
        cuda_check(cudaMemcpy(x.flags2[0] + q, &e, sizeof e, cudaMemcpyHostToDevice), "tp check peer flag2");
      }
    }
    cuda_check(cudaMemcpy(d_part.get(), pk, elems * 4, cudaMemcpyHostToDevice), "tp check part");
    cuda_check(cudaMemset(d_out.get(), 0, elems * 4), "tp check memset");
    launch_tp_publish(x, Slices{d_part.get<float>(), 1, 0}, cols, n, cols, nullptr);
    if (twoshot) {
      launch_tp_reduce(x, n, cols, d_status.get<int>(), nullptr);
      launch_tp_allgather(x, n, cols, d_out.get<float>(), d_status.get<int>(), nullptr);
    } else {
      launch_tp_gather(x, n, cols, d_out.get<float>(), d_status.get<int>(), nullptr);
    }
    cuda_check(cudaGetLastError(), "tp check launch");
    cuda_check(cudaDeviceSynchronize(), "tp check");
    int st = 0;
    cuda_check(cudaMemcpy(&st, d_status.get(), sizeof st, cudaMemcpyDeviceToHost), "tp check status");
    cuda_check(cudaMemset(d_status.get(), 0, sizeof(int)), "tp check status reset");
    call_status[k] = st == 0 ? MK_OK : (st == kErrTpWait ? MK_ERR_TIMEOUT : MK_ERR_CUDA);
    cuda_check(cudaMemcpy(out + static_cast<size_t>(k) * elems, d_out.get(), elems * 4, cudaMemcpyDeviceToHost),
               "tp check out");
  }
}

}  // namespace mkb
