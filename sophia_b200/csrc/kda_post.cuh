// Backward epilogue: L2-norm and ShortConv(+SiLU) backward, and the final
// deterministic reductions of the per-chunk partial sums.
//
//   kda_bwd_post_conv_kernel  (one warp per (chunk, head, tensor))
//     given dq_hat / dk_hat (gradients of the normalised inputs) and dv from
//     the chunk kernel, recomputes the conv output c = conv(x), y = silu(c)
//     and the norms, then
//       dy  = (dn - n (n . dn)) / max(|y|, eps)     (q: dn = scale dq_hat)
//       dc  = dy * silu'(c)
//       dx_t = sum_s w_s dc_(t+3-s),   dw_s += sum_t dc_t x_(t-3+s)
//   kda_bwd_post_norm_kernel: without the conv, only the L2-norm backward of
//     q and k (dv passes through).
//   kda_reduce_kernel: dA_log, dt_bias and conv-tap gradients, summed over
//     chunks in a fixed order.
#pragma once

#include "kda_common.cuh"
#include "kda_tc.cuh"  // g_kda_device_error

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

// Lane l of a warp owns channels 4l .. 4l+3 of a row, so a warp covers whole
// rows (the L2 norm of a row is a warp shuffle reduction) and each 8-byte
// load of a row is part of one 256-byte coalesced access.
constexpr int POST_THREADS = 256;

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
  if (ss > 1e-24f) {  // |y| > eps
    // dy = dscale g / |y| - y (dscale (y . g) / |y|^3); rsqrt.approx is within 2 ulp
    const float inv = rsqrtf(ss), gs = dscale * inv, ys = gs * dot * inv * inv;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dyv[ch] = fmaf(g[ch], gs, -y[ch] * ys);
  } else {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dyv[ch] = dscale * g[ch] * 1e12f;
  }
}

// Conv variant, one warp per (chunk, head, tensor), four chunks per CTA.  The
// warp walks rows r = 0 .. 66 of its chunk (rows 64 .. 66 are the next
// chunk's first rows, whose dc the conv backward of rows 61 .. 63 needs) with
// sliding four-row windows of x (conv inputs) and dc in registers; lane l owns
// channels 4l .. 4l+3, so the L2 norm of a row is a warp reduction.  Per row:
//   c = sum_s w_s x_(r-3+s), y = silu(c), dc_r = (norm backward of dy_r) silu'(c)
//   dw_s += dc_r x_(r-3+s)                       (own rows r < 64)
//   dx_(r-3) = sum_s w_s dc_(r-s)                (r >= 3)
// No shared memory and no barrier; the tap-gradient partial of the chunk
// leaves straight from the lanes.
constexpr int POST_CHUNKS_PER_CTA = 4;
constexpr int POST_GROUP = 4;  // rows per prefetch group

__global__ void __launch_bounds__(32 * POST_CHUNKS_PER_CTA) kda_bwd_post_conv_kernel(PostParams P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * POST_CHUNKS_PER_CTA + warp, h = blockIdx.y, X = blockIdx.z, H = P.H;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;  // warp-uniform
  const int eos = seq_eos(P.seq, pos.seq);
  const size_t rowH = (size_t)H * D;
  const bf16* x = X == 0 ? P.q : (X == 1 ? P.k : P.v);
  const bf16* gy = X == 0 ? P.dq_hat : (X == 1 ? P.dk_hat : P.dv_hat);
  bf16* dx = X == 0 ? P.dq : (X == 1 ? P.dk : P.dv);
  const float dscale = X == 0 ? P.scale : 1.f;
  const bool norm = X < 2;

  float wt[4][4];  // [channel][tap]
  {
    const float4* w = reinterpret_cast<const float4*>((X == 0 ? P.conv_q : (X == 1 ? P.conv_k : P.conv_v)) +
                                                      ((size_t)h * D + 4 * lane) * 4);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      const float4 t4 = __ldg(w + ch);
      wt[ch][0] = t4.x; wt[ch][1] = t4.y; wt[ch][2] = t4.z; wt[ch][3] = t4.w;
    }
  }
  float x0[4], x1[4], x2[4];  // x rows r-3, r-2, r-1
  float d0[4], d1[4], d2[4];  // dc rows r-3, r-2, r-1
  float acc[4][4];            // tap gradients [channel][tap]
  {
    const int t = pos.t0 - 3;
    unpack4(post_ld(x, t, t >= pos.bos, rowH, h, lane), x0);
    unpack4(post_ld(x, t + 1, t + 1 >= pos.bos, rowH, h, lane), x1);
    unpack4(post_ld(x, t + 2, t + 2 >= pos.bos, rowH, h, lane), x2);
  }
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    d0[ch] = d1[ch] = d2[ch] = 0.f;
    acc[ch][0] = acc[ch][1] = acc[ch][2] = acc[ch][3] = 0.f;
  }
  // rows go in groups of POST_GROUP; the next group's x and dy rows are loaded
  // before the current group is computed, so loads overlap a group of work
  constexpr int G = POST_GROUP, NG = (C + 3 + G - 1) / G;
  bf16x4 nx[G], ngy[G];
  auto load_group = [&](int grp) {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int r = grp * G + j, t = pos.t0 + r;
      const bool ok = r < C + 3 && t < eos;
      nx[j] = post_ld(x, t, ok, rowH, h, lane);
      ngy[j] = post_ld(gy, t, ok, rowH, h, lane);
    }
  };
  load_group(0);
#pragma unroll 1
  for (int grp = 0; grp < NG; ++grp) {
    bf16x4 cx[G], cgy[G];
#pragma unroll
    for (int j = 0; j < G; ++j) { cx[j] = nx[j]; cgy[j] = ngy[j]; }
    if (grp + 1 < NG) load_group(grp + 1);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int r = grp * G + j, t = pos.t0 + r;
      if (r >= C + 3) break;
      const bool rowok = t < eos;
      float xn[4], g[4];
      unpack4(cx[j], xn);
      unpack4(cgy[j], g);
      float cv[4], y[4], sg[4];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const float a = wt[ch][0] * x0[ch] + wt[ch][1] * x1[ch] + wt[ch][2] * x2[ch] + wt[ch][3] * xn[ch];
        const float hh = 0.5f * a, th = tanh_fast(hh);
        cv[ch] = a;
        y[ch] = fmaf(hh, th, hh);
        sg[ch] = fmaf(0.5f, th, 0.5f);
      }
      float dyv[4];
      if (norm) {
        post_norm_bwd(y, g, dscale, dyv);
      } else {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) dyv[ch] = g[ch];
      }
      float dn[4];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) dn[ch] = rowok ? dyv[ch] * sg[ch] * (1.f + cv[ch] * (1.f - sg[ch])) : 0.f;
      if (r < C) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          acc[ch][0] += dn[ch] * x0[ch];
          acc[ch][1] += dn[ch] * x1[ch];
          acc[ch][2] += dn[ch] * x2[ch];
          acc[ch][3] += dn[ch] * xn[ch];
        }
      }
      if (r >= 3 && t - 3 < pos.t1) {
        float dxv[4];
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
          dxv[ch] = wt[ch][0] * dn[ch] + wt[ch][1] * d2[ch] + wt[ch][2] * d1[ch] + wt[ch][3] * d0[ch];
        *reinterpret_cast<bf16x4*>(dx + (size_t)(t - 3) * rowH + (size_t)h * D + 4 * lane) = pack4(dxv);
      }
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        x0[ch] = x1[ch]; x1[ch] = x2[ch]; x2[ch] = xn[ch];
        d0[ch] = d1[ch]; d1[ch] = d2[ch]; d2[ch] = dn[ch];
      }
    }
  }
  float4* dst = reinterpret_cast<float4*>(P.partW + (((size_t)c * 3 + X) * H + h) * D * 4) + 4 * lane;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) dst[ch] = make_float4(acc[ch][0], acc[ch][1], acc[ch][2], acc[ch][3]);
}

// Without the conv: the L2-norm backward of q and k alone (dv passes
// through).  One CTA per (chunk, head, tensor); warp w takes rows 8w .. 8w+7.
__global__ void __launch_bounds__(POST_THREADS) kda_bwd_post_norm_kernel(PostParams P) {
  const int c = blockIdx.x, h = blockIdx.y, X = blockIdx.z, H = P.H;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const size_t rowH = (size_t)H * D;
  const bf16* x = X == 0 ? P.q : P.k;
  const bf16* gy = X == 0 ? P.dq_hat : P.dk_hat;
  bf16* dx = X == 0 ? P.dq : P.dk;
  const float dscale = X == 0 ? P.scale : 1.f;
  const int r0 = 8 * warp;
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
// total_tokens; otherwise *error_flag = 1, the device error flag
// (kda_b200_device_error) is set to 3, and every offset is 0, so all kernels of
// the call see zero chunks and touch no token.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) kda_chunk_table_kernel(const int* cu, int N, long long total_tokens,
                                                               int* offsets, int* chunk_seq, int* error_flag) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  int bad = 0;
  for (int n = tid; n < N; n += 1024) bad |= (cu[n + 1] < cu[n]);
  if (tid == 0) bad |= (cu[0] != 0) || ((long long)cu[N] != total_tokens);
  bad = __syncthreads_or(bad);
  if (tid == 0) {
    carry = 0;
    *error_flag = bad;
    if (bad) atomicExch(&g_kda_device_error, 3);
  }
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
