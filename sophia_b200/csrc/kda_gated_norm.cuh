// Gated output norm of the KDA mixer: per head row of 128 channels,
//   y = rms_norm(o) * w * sigmoid(g),   rms_norm(o) = o / sqrt(mean(o^2) + eps)
// (attention.py:416-419 with the RMSNorm of ops.py:49-64), forward and
// backward in one pass each.  HBM-bound elementwise work with two row
// reductions: 16 lanes own a row (8 channels each, 16-byte loads for bf16), a
// warp takes two rows per step, CTAs stride over row pairs.  Arithmetic is
// fp32; inputs and outputs are bf16 or fp32 (all the same dtype), w is fp32.
//
// Backward, with n = o r (r = 1 / sqrt(mean(o^2) + eps)), s = sigmoid(g):
//   dg = dy n w s (1 - s);   u = dy s (gradient of n w);   dw += sum_rows u n
//   do = r (u w - n mean(u w n))
// The weight gradient leaves as one partial row per CTA, summed in a fixed
// order by kda_gated_norm_reduce_kernel.
#pragma once

#include "kda_common.cuh"

namespace kda {

constexpr int GN_THREADS = 256;

struct GatedNormParams {
  const void *o, *g, *dy;
  const float* w;
  void *y, *d_o, *d_g;
  float* partial;  // [gridDim.x][128]
  long long rows;
  float eps;
  bool fp32;
};

__device__ __forceinline__ void gn_load8(const void* base, long long row, int c0, bool ok, bool f32, float (&v)[8]) {
  if (!ok) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  if (f32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + row * D + c0);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    unpack8(*reinterpret_cast<const bf16x8*>(static_cast<const bf16*>(base) + row * D + c0), v);
  }
}

__device__ __forceinline__ void gn_store8(void* base, long long row, int c0, bool f32, const float (&v)[8]) {
  if (f32) {
    float4* p = reinterpret_cast<float4*>(static_cast<float*>(base) + row * D + c0);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    *reinterpret_cast<bf16x8*>(static_cast<bf16*>(base) + row * D + c0) = pack8(v);
  }
}

// Sum over the 16 lanes that own a row.
__device__ __forceinline__ float gn_row_sum(float x) {
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
  return x;
}

__global__ void __launch_bounds__(GN_THREADS) kda_gated_norm_fwd_kernel(GatedNormParams P) {
  const int c0 = 8 * (threadIdx.x & 15);
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = __ldg(P.w + c0 + i);
  const long long pairs = (P.rows + 1) / 2;
  const int half = (threadIdx.x >> 4) & 1, warp = threadIdx.x >> 5;
  // every lane of a warp runs the same number of steps (shuffles are full-warp)
  for (long long pr = (long long)blockIdx.x * (GN_THREADS / 32) + warp; pr < pairs;
       pr += (long long)gridDim.x * (GN_THREADS / 32)) {
    const long long row = 2 * pr + half;
    const bool ok = row < P.rows;
    float o[8], g[8];
    gn_load8(P.o, row, c0, ok, P.fp32, o);
    gn_load8(P.g, row, c0, ok, P.fp32, g);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(o[i], o[i], ss);
    const float r = rsqrtf(gn_row_sum(ss) * (1.f / D) + P.eps);
    float y[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) y[i] = o[i] * r * w[i] * sigmoidf_(g[i]);
    if (ok) gn_store8(P.y, row, c0, P.fp32, y);
  }
}

__global__ void __launch_bounds__(GN_THREADS) kda_gated_norm_bwd_kernel(GatedNormParams P) {
  __shared__ float red[GN_THREADS / 16][D];
  const int c0 = 8 * (threadIdx.x & 15);
  float w[8], dw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    w[i] = __ldg(P.w + c0 + i);
    dw[i] = 0.f;
  }
  const long long pairs = (P.rows + 1) / 2;
  const int half = (threadIdx.x >> 4) & 1, warp = threadIdx.x >> 5;
  for (long long pr = (long long)blockIdx.x * (GN_THREADS / 32) + warp; pr < pairs;
       pr += (long long)gridDim.x * (GN_THREADS / 32)) {
    const long long row = 2 * pr + half;
    const bool ok = row < P.rows;
    float o[8], g[8], dy[8];
    gn_load8(P.o, row, c0, ok, P.fp32, o);
    gn_load8(P.g, row, c0, ok, P.fp32, g);
    gn_load8(P.dy, row, c0, ok, P.fp32, dy);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(o[i], o[i], ss);
    const float r = rsqrtf(gn_row_sum(ss) * (1.f / D) + P.eps);
    float n[8], u[8], dgv[8], dot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float s = sigmoidf_(g[i]);
      n[i] = o[i] * r;
      u[i] = dy[i] * s;
      dgv[i] = dy[i] * n[i] * w[i] * s * (1.f - s);
      dot = fmaf(u[i] * w[i], n[i], dot);
      dw[i] = fmaf(u[i], n[i], dw[i]);
    }
    const float mdot = gn_row_sum(dot) * (1.f / D);
    float dov[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) dov[i] = r * (u[i] * w[i] - n[i] * mdot);
    if (ok) {
      gn_store8(P.d_o, row, c0, P.fp32, dov);
      gn_store8(P.d_g, row, c0, P.fp32, dgv);
    }
  }
  // the CTA's weight-gradient partial: the 16 row slots in a fixed order
  const int slot = threadIdx.x >> 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) red[slot][c0 + i] = dw[i];
  __syncthreads();
  if (threadIdx.x < D) {
    float acc = 0.f;
#pragma unroll
    for (int s = 0; s < GN_THREADS / 16; ++s) acc += red[s][threadIdx.x];
    P.partial[(size_t)blockIdx.x * D + threadIdx.x] = acc;
  }
}

// dw[c] = sum over CTAs of partial[b][c]: eight strided slices of the CTAs
// summed in order, then the eight slice sums in order (a fixed order for a
// given CTA count).
constexpr int GN_REDUCE_SLICES = 8;
__global__ void __launch_bounds__(D * GN_REDUCE_SLICES) kda_gated_norm_reduce_kernel(const float* partial, int nparts,
                                                                                     float* dw) {
  __shared__ float part[GN_REDUCE_SLICES][D];
  const int c = threadIdx.x % D, sl = threadIdx.x / D;
  float acc = 0.f;
  for (int b = sl; b < nparts; b += GN_REDUCE_SLICES) acc += partial[(size_t)b * D + c];
  part[sl][c] = acc;
  __syncthreads();
  if (sl == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < GN_REDUCE_SLICES; ++i) t += part[i][c];
    dw[c] = t;
  }
}

}  // namespace kda
