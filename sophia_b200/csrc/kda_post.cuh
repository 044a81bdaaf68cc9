// Backward epilogue: L2-norm and ShortConv(+SiLU) backward, and the final
// deterministic reductions of the per-chunk partial sums.
//
//   kda_bwd_post_kernel  (one CTA per (chunk, head, tensor))
//     given dq_hat / dk_hat (gradients of the normalised inputs) and dv from
//     the chunk kernel, recomputes the conv output c = conv(x), y = silu(c)
//     and the norms, then
//       dy  = (dn - n (n . dn)) / max(|y|, eps)     (q: dn = scale dq_hat)
//       dc  = dy * silu'(c)
//       dx_t = sum_s w_s dc_(t+3-s),   dw_s += sum_t dc_t x_(t-3+s)
//     Without the conv, only the L2-norm backward runs (dv passes through).
//   kda_reduce_kernel: dA_log, dt_bias and conv-tap gradients, summed over
//     chunks in a fixed order.
#pragma once

#include "kda_common.cuh"

namespace kda {

struct PostParams {
  SeqInfo seq;
  int H;
  bool conv;
  float scale;
  const bf16 *q, *k, *v;                        // inputs as given to the layer
  const float *conv_q, *conv_k, *conv_v;        // [H*128][4]
  const bf16 *dq_hat, *dk_hat, *dv_hat;         // [T_total][H][128]
  bf16 *dq, *dk, *dv;                           // outputs
  float* partW;                                 // [chunks][3][H][128][4]
};

// One CTA per (chunk, head, tensor), 256 threads: warp w owns dc rows
// 8w .. 8w+7 and lane l channels 4l .. 4l+3, so a warp covers whole rows (the
// L2 norm of a row is a warp shuffle reduction) and each 8-byte load of a row
// is part of one 256-byte coalesced access.  A thread's conv input rows (x rows
// 8w-3 .. 8w+7) and gradient rows are loaded straight from global memory into
// registers, all in flight together.  The fp32 dc tile goes through shared
// memory because the conv backward of row t needs dc rows t .. t+3; rows
// 64 .. 66 are the next chunk's first rows and are computed by warp 7.
constexpr int POST_THREADS = 256;
constexpr int POST_DC_BYTES = 67 * D * 4;

struct alignas(8) bf16x4 { uint32_t u[2]; };

__device__ __forceinline__ void unpack4(const bf16x4& v, float (&f)[4]) {
  const float2 a = unpack_bf16(v.u[0]), b = unpack_bf16(v.u[1]);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
__device__ __forceinline__ bf16x4 pack4(const float (&f)[4]) {
  bf16x4 v;
  v.u[0] = pack_bf16(f[0], f[1]);
  v.u[1] = pack_bf16(f[2], f[3]);
  return v;
}

__device__ __forceinline__ bf16x4 post_ld(const bf16* base, int t, bool ok, size_t rowH, int h, int lane) {
  uint2 u = make_uint2(0u, 0u);
  if (ok) u = __ldg(reinterpret_cast<const uint2*>(base + (size_t)t * rowH + (size_t)h * D + 4 * lane));
  bf16x4 v;
  v.u[0] = u.x; v.u[1] = u.y;
  return v;
}

// L2-norm backward of one row (full-warp shuffles): dn = dscale g,
// n = y / |y|, result (dn - n (n . dn)) / |y|.
__device__ __forceinline__ void post_norm_bwd(const float (&y)[4], const float (&g)[4], float dscale,
                                              float (&dyv)[4]) {
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) { ss += y[ch] * y[ch]; dot += y[ch] * g[ch]; }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, m);
    dot += __shfl_xor_sync(0xffffffffu, dot, m);
  }
  const float nrm = sqrtf(ss);
  if (nrm > 1e-12f) {
    const float inv = 1.f / nrm, nd = dot * inv * dscale;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dyv[ch] = (dscale * g[ch] - y[ch] * inv * nd) * inv;
  } else {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dyv[ch] = dscale * g[ch] * 1e12f;
  }
}

// dc of one row: conv c from x rows row-3 .. row, SiLU y = c sigmoid(c) and
// sigmoid(c) from one tanh.approx (the forward prologue's silu_fast on the
// same c), the L2-norm backward (q, k), dc = dy sigmoid(c) (1 + c (1 - sigmoid(c)));
// zero for rows past the sequence end.
__device__ __forceinline__ float4 post_dc_row(const bf16x4& x0, const bf16x4& x1, const bf16x4& x2,
                                              const bf16x4& x3, const float (&wt)[4][4], const bf16x4& gr,
                                              bool rowok, bool norm, float dscale) {
  float xa[4][4];
  unpack4(x0, xa[0]); unpack4(x1, xa[1]); unpack4(x2, xa[2]); unpack4(x3, xa[3]);
  float cv[4], y[4], sg[4], g[4], dyv[4];
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const float a = wt[ch][0] * xa[0][ch] + wt[ch][1] * xa[1][ch] + wt[ch][2] * xa[2][ch] + wt[ch][3] * xa[3][ch];
    const float hh = 0.5f * a, t = tanh_fast(hh);
    cv[ch] = a;
    y[ch] = fmaf(hh, t, hh);
    sg[ch] = fmaf(0.5f, t, 0.5f);
  }
  unpack4(gr, g);
  if (norm) {
    post_norm_bwd(y, g, dscale, dyv);
  } else {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dyv[ch] = g[ch];
  }
  float dc[4];
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) dc[ch] = rowok ? dyv[ch] * sg[ch] * (1.f + cv[ch] * (1.f - sg[ch])) : 0.f;
  return make_float4(dc[0], dc[1], dc[2], dc[3]);
}

template <bool CONV>
__global__ void __launch_bounds__(POST_THREADS, 2) kda_bwd_post_kernel(PostParams P) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int c = blockIdx.x, h = blockIdx.y, X = blockIdx.z, H = P.H;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int eos = seq_eos(P.seq, pos.seq);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const size_t rowH = (size_t)H * D;
  const bf16* x = X == 0 ? P.q : (X == 1 ? P.k : P.v);
  const bf16* gy = X == 0 ? P.dq_hat : (X == 1 ? P.dk_hat : P.dv_hat);
  bf16* dx = X == 0 ? P.dq : (X == 1 ? P.dk : P.dv);
  const float dscale = X == 0 ? P.scale : 1.f;
  const int r0 = 8 * warp;  // first row of this warp

  if (!CONV) {  // L2-norm backward only (q and k)
    bf16x4 xr[8], gr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = pos.t0 + r0 + j;
      xr[j] = post_ld(x, t, t < pos.t1, rowH, h, lane);
      gr[j] = post_ld(gy, t, t < pos.t1, rowH, h, lane);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float y[4], g[4], dyv[4];
      unpack4(xr[j], y);
      unpack4(gr[j], g);
      post_norm_bwd(y, g, dscale, dyv);
      const int t = pos.t0 + r0 + j;
      if (t < pos.t1) *reinterpret_cast<bf16x4*>(dx + (size_t)t * rowH + (size_t)h * D + 4 * lane) = pack4(dyv);
    }
    return;
  }

  float wt[4][4];
  {
    const float4* w = reinterpret_cast<const float4*>((X == 0 ? P.conv_q : (X == 1 ? P.conv_k : P.conv_v)) +
                                                      ((size_t)h * D + 4 * lane) * 4);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      const float4 t4 = __ldg(w + ch);
      wt[ch][0] = t4.x; wt[ch][1] = t4.y; wt[ch][2] = t4.z; wt[ch][3] = t4.w;
    }
  }
  const bool norm = X < 2;
  float4* dcs = reinterpret_cast<float4*>(smem);  // [67 rows][32 lanes]
  // x rows r0-3 .. r0+7 (zero before the sequence start and past its end)
  bf16x4 xr[11], gr[8];
#pragma unroll
  for (int j = 0; j < 11; ++j) {
    const int t = pos.t0 + r0 - 3 + j;
    xr[j] = post_ld(x, t, t >= pos.bos && t < eos, rowH, h, lane);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int t = pos.t0 + r0 + j;
    gr[j] = post_ld(gy, t, t < eos, rowH, h, lane);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    dcs[(r0 + j) * 32 + lane] =
        post_dc_row(xr[j], xr[j + 1], xr[j + 2], xr[j + 3], wt, gr[j], pos.t0 + r0 + j < eos, norm, dscale);
  if (warp == 7) {  // dc rows 64 .. 66: the next chunk's first rows (x rows 61 .. 66)
    bf16x4 xe[6], ge[3];
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      const int t = pos.t0 + 61 + j;
      xe[j] = post_ld(x, t, t < eos, rowH, h, lane);
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int t = pos.t0 + 64 + j;
      ge[j] = post_ld(gy, t, t < eos, rowH, h, lane);
    }
#pragma unroll
    for (int j = 0; j < 3; ++j)
      dcs[(64 + j) * 32 + lane] =
          post_dc_row(xe[j], xe[j + 1], xe[j + 2], xe[j + 3], wt, ge[j], pos.t0 + 64 + j < eos, norm, dscale);
  }
  __syncthreads();

  // conv backward: dx_t = sum_s w_s dc_(t+3-s), dw_s += dc_t x_(t-3+s)
  float acc[4][4];
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) acc[ch][0] = acc[ch][1] = acc[ch][2] = acc[ch][3] = 0.f;
  float4 win[4];  // dc rows t .. t+3 (ring)
#pragma unroll
  for (int i = 0; i < 3; ++i) win[i] = dcs[(r0 + i) * 32 + lane];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    win[(j + 3) & 3] = dcs[(r0 + j + 3) * 32 + lane];
    const float4 d0 = win[j & 3], d1 = win[(j + 1) & 3], d2 = win[(j + 2) & 3], d3 = win[(j + 3) & 3];
    const float e0[4] = {d0.x, d0.y, d0.z, d0.w}, e1[4] = {d1.x, d1.y, d1.z, d1.w};
    const float e2[4] = {d2.x, d2.y, d2.z, d2.w}, e3[4] = {d3.x, d3.y, d3.z, d3.w};
    float xs[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) unpack4(xr[j + i], xs[i]);
    float dxv[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      dxv[ch] = wt[ch][0] * e3[ch] + wt[ch][1] * e2[ch] + wt[ch][2] * e1[ch] + wt[ch][3] * e0[ch];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[ch][i] += e0[ch] * xs[i][ch];
    }
    const int t = pos.t0 + r0 + j;
    if (t < pos.t1) *reinterpret_cast<bf16x4*>(dx + (size_t)t * rowH + (size_t)h * D + 4 * lane) = pack4(dxv);
  }
  // tap-gradient partial of this chunk: the eight warps through shared memory
  // (reusing the dc tile), added in a fixed order
  __syncthreads();
  float4* red = dcs;  // [8 warps][128 channels] of 4 taps
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) red[warp * D + 4 * lane + ch] = make_float4(acc[ch][0], acc[ch][1], acc[ch][2], acc[ch][3]);
  __syncthreads();
  if (tid < D) {
    float4 s4 = red[tid];
#pragma unroll
    for (int w = 1; w < 8; ++w) {
      const float4 a = red[w * D + tid];
      s4.x += a.x; s4.y += a.y; s4.z += a.z; s4.w += a.w;
    }
    reinterpret_cast<float4*>(P.partW + (((size_t)c * 3 + X) * H + h) * D * 4)[tid] = s4;
  }
}

struct ReduceParams {
  SeqInfo seq;
  int H;
  bool conv;
  const float *partA, *partB, *partW;
  float *dA_log, *ddt_bias, *dconv_q, *dconv_k, *dconv_v;
};

// Deterministic sums over chunks of the per-chunk partials, 256 threads per
// block and 128 columns per block: warp w adds chunks w, w+8, ... (lane l owns
// four consecutive columns, float4 loads), then the eight warp partials are
// added in a fixed order.
//   blocks [0, H):        ddt_bias[h, :]   = sum_c partB[c, h, :]
//   blocks [H, 2H):       dA_log[h]        = sum_c sum_d partA[c, h, d]
//   blocks [2H, 2H+12H):  dconv (3 x H x 128 x 4 columns of partW)
__global__ void __launch_bounds__(256) kda_reduce_kernel(ReduceParams P) {
  __shared__ float4 red[8][32];
  const int H = P.H, b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nchunks = P.seq.cu_seqlens ? P.seq.chunk_offsets[P.seq.N] : P.seq.N * P.seq.nt;
  const float* src;
  size_t stride, col0;
  int kind;
  if (b < H) { kind = 0; src = P.partB; stride = (size_t)H * D; col0 = (size_t)b * D; }
  else if (b < 2 * H) { kind = 1; src = P.partA; stride = (size_t)H * D; col0 = (size_t)(b - H) * D; }
  else { kind = 2; src = P.partW; stride = (size_t)3 * H * D * 4; col0 = (size_t)(b - 2 * H) * 128; }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int c = warp; c < nchunks; c += 8) {
    float4 v = __ldg(reinterpret_cast<const float4*>(src + (size_t)c * stride + col0) + lane);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0) {
    float4 t = red[0][lane];
    for (int w = 1; w < 8; ++w) {
      float4 v = red[w][lane];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    if (kind == 0) {
      reinterpret_cast<float4*>(P.ddt_bias + col0)[lane] = t;
    } else if (kind == 1) {
      float sum = t.x + t.y + t.z + t.w;
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) P.dA_log[b - H] = sum;
    } else {
      // column index col0 + 4*lane within the [3][H][128][4] layout
      size_t col = col0 + 4 * (size_t)lane;
      size_t per = (size_t)H * D * 4;
      int X = (int)(col / per);
      float* out = X == 0 ? P.dconv_q : (X == 1 ? P.dconv_k : P.dconv_v);
      reinterpret_cast<float4*>(out + (col - (size_t)X * per))[0] = t;
    }
  }
}

// Builds the chunk table of packed sequences on the device (no host sync):
// chunk_offsets[n] = sum_{m<n} ceil(len_m / 64), chunk_seq[c] = sequence of
// chunk c.  cu_seqlens must start at 0, be non-decreasing and end at
// total_tokens; otherwise *error_flag = 1 and every offset is 0, so all
// kernels of the call see zero chunks and touch no token.  One CTA of 1024
// threads.
__global__ void __launch_bounds__(1024) kda_chunk_table_kernel(const int* cu, int N, long long total_tokens,
                                                               int* offsets, int* chunk_seq, int* error_flag) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  int bad = 0;
  for (int n = tid; n < N; n += 1024) bad |= (cu[n + 1] < cu[n]);
  if (tid == 0) bad |= (cu[0] != 0) || ((long long)cu[N] != total_tokens);
  bad = __syncthreads_or(bad);
  if (tid == 0) { carry = 0; *error_flag = bad; }
  if (bad) {
    for (int n = tid; n <= N; n += 1024) offsets[n] = 0;
    return;
  }
  __syncthreads();
  for (int base = 0; base < N; base += 1024) {
    int n = base + tid;
    int len = n < N ? cu[n + 1] - cu[n] : 0;
    int nc = (len + C - 1) / C;
    int x = nc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[wid] = x;
    __syncthreads();
    if (wid == 0) {
      int sv = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, sv, o);
        if (lane >= o) sv += y;
      }
      warp_sums[lane] = sv;
    }
    __syncthreads();
    int incl = x + (wid > 0 ? warp_sums[wid - 1] : 0) + carry;
    if (n < N) {
      offsets[n] = incl - nc;
      for (int i = 0; i < nc; ++i) chunk_seq[incl - nc + i] = n;
    }
    __syncthreads();
    if (tid == 1023) carry = incl;
    __syncthreads();
  }
  if (tid == 0) offsets[N] = carry;
}

}  // namespace kda
