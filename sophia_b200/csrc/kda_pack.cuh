// Document boundaries of packed pretraining windows, on the device.
//
// Sophia's pretraining data path packs documents into fixed windows of
// tokens and runs each window as one sequence, with no reset at document ends
// (ml/training/pretrain/engine/sm120_graph_runner.py:244-259, static
// [1, 4096] int32 token slabs replayed through a CUDA graph).  This kernel
// turns such token windows into the cu_seqlens table of the packed KDA layer,
// so that the recurrent state and the conv history restart at every document,
// without a host synchronisation: the table has a fixed capacity (N is known
// when the graph is captured) and unused entries describe empty sequences.
//
// A document starts at every window start and at the token after every EOS
// token (the EOS closes its document).  Boundary b (in token order) goes to
// cu_seqlens[b] while b < capacity; cu_seqlens[b] = total_tokens for every
// later entry up to cu_seqlens[capacity].  When a batch holds more documents
// than the capacity, the boundaries past the capacity are dropped -- those
// documents run on from their predecessor with no reset, the reference's own
// behaviour -- and *n_docs reports the true count so the caller can size the
// capacity.  One CTA of 1024 threads scans the tokens in tiles.
#pragma once

#include "kda_common.cuh"

namespace kda {

constexpr int PACK_THREADS = 1024;
constexpr int PACK_PER_THREAD = 8;  // tokens per thread per tile

__global__ void __launch_bounds__(PACK_THREADS) kda_doc_bounds_kernel(const int* tokens, long long total, int window,
                                                                      int eos_id, int capacity, int* cu_seqlens,
                                                                      int* n_docs) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  constexpr long long TILE = (long long)PACK_THREADS * PACK_PER_THREAD;
  for (long long base = 0; base < total; base += TILE) {
    const long long t0 = base + (long long)tid * PACK_PER_THREAD;
    unsigned flags = 0;
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < PACK_PER_THREAD; ++i) {
      const long long t = t0 + i;
      if (t < total) {
        const bool start = (t % window) == 0 || tokens[t - 1] == eos_id;
        if (start) {
          flags |= 1u << i;
          ++cnt;
        }
      }
    }
    // exclusive prefix of the per-thread counts over the CTA, plus the carry
    int x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    int idx = x - cnt + (wid > 0 ? warp_sums[wid - 1] : 0) + carry;
#pragma unroll
    for (int i = 0; i < PACK_PER_THREAD; ++i) {
      if (flags & (1u << i)) {
        if (idx < capacity) cu_seqlens[idx] = (int)(t0 + i);
        ++idx;
      }
    }
    __syncthreads();
    if (tid == PACK_THREADS - 1) carry = idx;
    __syncthreads();
  }
  const int count = carry;
  for (int b = min(count, capacity) + tid; b <= capacity; b += PACK_THREADS) cu_seqlens[b] = (int)total;
  if (tid == 0) *n_docs = count;
}

}  // namespace kda
