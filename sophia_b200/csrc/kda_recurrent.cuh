// Token-by-token KDA recurrence for decode (fp32 state and arithmetic).
//
// One CTA (128 threads) per (sequence, head).  The 128x128 state S[k][v] sits
// in shared memory (64 KB, so three CTAs share an SM and their state loads
// overlap each other's work) and thread v updates column v in place.  Per token, the
// CTA builds the normalised q (times scale), the normalised k and the decay
// alpha_k = exp(lb * sigmoid(exp(A_log) (g_k + dt_bias_k))) in shared memory,
// then every thread runs the reference's update on its column:
//   S <- diag(alpha) S;  pred = k^T S;  u = beta (v - pred);
//   S <- S + k u^T;      o = q^T S
// (ml/runtime/model/attention.py:286-292, the order of the reference loop).
// Inputs may be bf16 or fp32; o takes v's dtype; the final state is fp32.
//
// With conv taps and a conv history (the decode step of a cached
// SophiaKDA.forward: _short_convolution with history, attention.py:226-258),
// q, k and v are the pre-conv projections: thread v keeps the last three
// inputs of channel v of q, k and v in registers, forms
//   c = w0 x_(t-3) + w1 x_(t-2) + w2 x_(t-1) + w3 x_t,  x <- silu(c)
// per token, and writes the history back at the end (the module's conv_state,
// [B][3][H*128][3], oldest position first).
#pragma once

#include "kda_fwd_state_tc.cuh"  // g_kda_device_error

namespace kda {

constexpr int REC_THREADS = 128;
constexpr int REC_SMEM = D * D * 4;  // the fp32 state, dynamic shared memory

struct RecurrentParams {
  SeqInfo seq;
  int H;
  bool fp32_inputs;
  const void *q, *k, *v, *g, *beta;  // [T_total][H][128] ([T_total][H] for beta)
  const float *A_log, *dt_bias;      // [H], [H*128]
  const float* h0;                   // [N][H][128][128] or null
  float scale, lower_bound;
  void* o;                           // [T_total][H][128], v's dtype
  float* ht;                         // [N][H][128][128] or null
  long long total_tokens;            // B*T: sequence bounds are checked against it
  const float *conv_q, *conv_k, *conv_v;  // [H*128][4] taps, or null (inputs are post-conv)
  float* conv_state;                 // [N][3][H*128][3] history in/out (with the taps)
};

// One conv step of channel `ch` given its three previous inputs (updated).
__device__ __forceinline__ float rec_conv_silu(const float* taps, size_t ch, float (&hist)[3], float x) {
  const float4 w = __ldg(reinterpret_cast<const float4*>(taps) + ch);
  const float c = w.x * hist[0] + w.y * hist[1] + w.z * hist[2] + w.w * x;
  hist[0] = hist[1];
  hist[1] = hist[2];
  hist[2] = x;
  return c / (1.f + expf(-c));
}

__device__ __forceinline__ float rec_load(const void* p, size_t i, bool f32) {
  return f32 ? static_cast<const float*>(p)[i] : __bfloat162float(static_cast<const bf16*>(p)[i]);
}

// Sum over the CTA (128 threads = 4 warps); red holds 4 floats per call site.
__device__ __forceinline__ float rec_block_sum(float x, float* red) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}

__global__ void __launch_bounds__(REC_THREADS) kda_recurrent_kernel(RecurrentParams P) {
  extern __shared__ __align__(16) float rec_state[];  // [128][128]: row k, column v
  __shared__ float qn[D], kn[D], alpha[D];
  __shared__ float red[2][4];
  const int n = blockIdx.x, h = blockIdx.y, H = P.H, vi = threadIdx.x;
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  if (bos < 0 || eos < bos || (long long)eos > P.total_tokens) {  // malformed cu_seqlens: touch nothing
    if (vi == 0) atomicExch(&g_kda_device_error, 3);
    return;
  }
  const size_t stateoff = ((size_t)n * H + h) * D * D;

  // the state -> shared memory (cp.async, 16-byte chunks, when aligned)
  float* const S = rec_state;
  if (P.h0) {
    const float* src = P.h0 + stateoff;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      for (int i = vi; i < D * D / 4; i += REC_THREADS) cp_async16(S + 4 * i, src + 4 * i, true);
    } else {
      for (int i = vi; i < D * D; i += REC_THREADS) S[i] = src[i];
    }
  } else {
    for (int i = vi; i < D * D / 4; i += REC_THREADS)
      reinterpret_cast<float4*>(S)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  cp_async_commit();

  const float eA = expf(P.A_log[h]);
  const float bias = P.dt_bias[(size_t)h * D + vi];
  const bool conv = P.conv_state != nullptr;
  const size_t ch = (size_t)h * D + vi, inner = (size_t)H * D;
  float hq[3] = {0.f, 0.f, 0.f}, hk[3] = {0.f, 0.f, 0.f}, hv[3] = {0.f, 0.f, 0.f};
  if (conv) {
    const float* cs = P.conv_state + (size_t)n * 3 * inner * 3 + ch * 3;
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      hq[s] = cs[s];
      hk[s] = cs[inner * 3 + s];
      hv[s] = cs[2 * inner * 3 + s];
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // (each thread then reads and writes only its own column)
  for (int t = bos; t < eos; ++t) {
    const size_t row = ((size_t)t * H + h) * D + vi;
    float qx = rec_load(P.q, row, P.fp32_inputs), kx = rec_load(P.k, row, P.fp32_inputs);
    float vx = rec_load(P.v, row, P.fp32_inputs);
    const float gx = rec_load(P.g, row, P.fp32_inputs);
    if (conv) {
      qx = rec_conv_silu(P.conv_q, ch, hq, qx);
      kx = rec_conv_silu(P.conv_k, ch, hk, kx);
      vx = rec_conv_silu(P.conv_v, ch, hv, vx);
    }
    const float bx = rec_load(P.beta, (size_t)t * H + h, P.fp32_inputs);
    const float sq = rec_block_sum(qx * qx, red[0]);
    const float sk = rec_block_sum(kx * kx, red[1]);
    qn[vi] = qx / fmaxf(sqrtf(sq), 1e-12f) * P.scale;
    kn[vi] = kx / fmaxf(sqrtf(sk), 1e-12f);
    alpha[vi] = expf(P.lower_bound / (1.f + expf(-eA * (gx + bias))));
    const float beta = 1.f / (1.f + expf(-bx));
    __syncthreads();
    float pred = 0.f;
#pragma unroll 16
    for (int kk = 0; kk < D; ++kk) {
      const float sv = S[kk * D + vi] * alpha[kk];
      S[kk * D + vi] = sv;
      pred = fmaf(kn[kk], sv, pred);
    }
    const float u = (vx - pred) * beta;
    float out = 0.f;
#pragma unroll 16
    for (int kk = 0; kk < D; ++kk) {
      const float sv = fmaf(kn[kk], u, S[kk * D + vi]);
      S[kk * D + vi] = sv;
      out = fmaf(qn[kk], sv, out);
    }
    if (P.fp32_inputs)
      static_cast<float*>(P.o)[row] = out;
    else
      static_cast<bf16*>(P.o)[row] = __float2bfloat16(out);
    __syncthreads();  // qn/kn/alpha/red are rewritten by the next token
  }
  if (P.ht) {
#pragma unroll 16
    for (int kk = 0; kk < D; ++kk) P.ht[stateoff + (size_t)kk * D + vi] = S[kk * D + vi];
  }
  if (conv) {
    float* cs = P.conv_state + (size_t)n * 3 * inner * 3 + ch * 3;
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      cs[s] = hq[s];
      cs[inner * 3 + s] = hk[s];
      cs[2 * inner * 3 + s] = hv[s];
    }
  }
}

}  // namespace kda
