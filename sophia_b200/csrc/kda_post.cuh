// Backward epilogue: L2-norm and ShortConv(+SiLU) backward, and the final
// deterministic reductions of the per-chunk partial sums.
//
//   kda_bwd_post_kernel  (one CTA per (chunk, head))
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

struct PostSmem {
  static constexpr int XS = 0;                      // 70 x 128 bf16
  static constexpr int DS = XS + 70 * D * 2;        // 67 x 128 bf16
  static constexpr int DC = DS + 67 * D * 2;        // 67 x 128 fp32
  static constexpr int PW = DC + 67 * D * 4;        // 16 x 4 x 128 fp32 (row group, tap, channel)
  static constexpr int TAPS = PW + 16 * 4 * D * 4;  // 4 x 128 fp32, tap-major
  static constexpr int END = TAPS + 4 * D * 4;
};

__global__ void __launch_bounds__(256) kda_bwd_post_kernel(PostParams P) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int c = blockIdx.x, h = blockIdx.y, H = P.H;
  ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int eos = seq_eos(P.seq, pos.seq);
  const int nv = pos.t1 - pos.t0;
  const int tid = threadIdx.x, tg = tid >> 4, cg = tid & 15;
  bf16* xs = reinterpret_cast<bf16*>(smem + PostSmem::XS);
  bf16* ds = reinterpret_cast<bf16*>(smem + PostSmem::DS);
  float* dcs = reinterpret_cast<float*>(smem + PostSmem::DC);
  float* pw = reinterpret_cast<float*>(smem + PostSmem::PW);
  const size_t rowH = (size_t)H * D;

  for (int X = 0; X < 3; ++X) {
    if (!P.conv && X == 2) break;  // dv passes through unchanged
    const bf16* x = X == 0 ? P.q : (X == 1 ? P.k : P.v);
    const bf16* dy = X == 0 ? P.dq_hat : (X == 1 ? P.dk_hat : P.dv_hat);
    bf16* dx = X == 0 ? P.dq : (X == 1 ? P.dk : P.dv);
    const float* w = P.conv ? (X == 0 ? P.conv_q : (X == 1 ? P.conv_k : P.conv_v)) + (size_t)h * D * 4 : nullptr;
    const float dscale = X == 0 ? P.scale : 1.f;
    const int nrow = P.conv ? 67 : nv;  // rows of dc needed
    // loads: x rows t0-3 .. t0+66 (conv) or t0 .. t1-1, gradient rows t0 .. t0+nrow-1
    for (int i = tid; i < 70 * 16; i += blockDim.x) {
      int r = i >> 4, cc = i & 15;
      int t = P.conv ? pos.t0 - 3 + r : pos.t0 + r;
      bool ok = (t >= pos.bos) && (t < eos) && (P.conv ? r < 70 : r < nv);
      cp_async16(xs + r * D + cc * 8, x + (ok ? (size_t)t * rowH + (size_t)h * D + cc * 8 : 0), ok);
    }
    for (int i = tid; i < 67 * 16; i += blockDim.x) {
      int r = i >> 4, cc = i & 15;
      int t = pos.t0 + r;
      bool ok = (t < eos) && (r < nrow);
      cp_async16(ds + r * D + cc * 8, dy + (ok ? (size_t)t * rowH + (size_t)h * D + cc * 8 : 0), ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    float wt[8][4];
    if (P.conv) {
      float* taps = reinterpret_cast<float*>(smem + PostSmem::TAPS);
      for (int i = tid; i < D; i += blockDim.x) {
        float4 t4 = __ldg(reinterpret_cast<const float4*>(w) + i);
        taps[i] = t4.x; taps[D + i] = t4.y; taps[2 * D + i] = t4.z; taps[3 * D + i] = t4.w;
      }
      __syncthreads();
#pragma unroll
      for (int tap = 0; tap < 4; ++tap) {
        float4 a = *reinterpret_cast<const float4*>(taps + tap * D + 8 * cg);
        float4 b = *reinterpret_cast<const float4*>(taps + tap * D + 8 * cg + 4);
        wt[0][tap] = a.x; wt[1][tap] = a.y; wt[2][tap] = a.z; wt[3][tap] = a.w;
        wt[4][tap] = b.x; wt[5][tap] = b.y; wt[6][tap] = b.z; wt[7][tap] = b.w;
      }
    }
    // dc (or the norm backward alone) for rows tg, tg+16, ...; every lane runs
    // all five iterations so the full-warp shuffles stay uniform
    for (int it = 0; it < 5; ++it) {
      const int r = tg + 16 * it;
      const bool live = r < 67;
      const int rr = live ? r : 66;
      float cv[8], y[8], g[8];
      unpack8(*reinterpret_cast<const bf16x8*>(ds + rr * D + 8 * cg), g);
      if (P.conv) {
        float xr[4][8];
#pragma unroll
        for (int sidx = 0; sidx < 4; ++sidx) unpack8(*reinterpret_cast<const bf16x8*>(xs + (rr + sidx) * D + 8 * cg), xr[sidx]);
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) {
          float a = wt[cch][0] * xr[0][cch] + wt[cch][1] * xr[1][cch] + wt[cch][2] * xr[2][cch] + wt[cch][3] * xr[3][cch];
          cv[cch] = a;
          y[cch] = silu_fast(a);
        }
      } else {
        unpack8(*reinterpret_cast<const bf16x8*>(xs + rr * D + 8 * cg), y);
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) cv[cch] = 0.f;
      }
      float dyv[8];
      if (X < 2) {
        float ss = 0.f, dot = 0.f;
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) { ss += y[cch] * y[cch]; dot += y[cch] * g[cch]; }
#pragma unroll
        for (int m = 8; m >= 1; m >>= 1) {
          ss += __shfl_xor_sync(0xffffffffu, ss, m);
          dot += __shfl_xor_sync(0xffffffffu, dot, m);
        }
        float nrm = sqrtf(ss);
        if (nrm > 1e-12f) {
          float inv = 1.f / nrm;
          // n = y/nrm, dn = dscale*g: dy = (dn - n (n.dn)) / nrm
          float nd = dot * inv * dscale;
#pragma unroll
          for (int cch = 0; cch < 8; ++cch) dyv[cch] = (dscale * g[cch] - y[cch] * inv * nd) * inv;
        } else {
#pragma unroll
          for (int cch = 0; cch < 8; ++cch) dyv[cch] = dscale * g[cch] * 1e12f;
        }
      } else {
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) dyv[cch] = g[cch];
      }
      bool rowok = live && pos.t0 + r < eos;
      if (!live) continue;
      if (P.conv) {
        float dcv[8];
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) {
          float sg = sigmoid_fast(cv[cch]);
          dcv[cch] = rowok ? dyv[cch] * sg * (1.f + cv[cch] * (1.f - sg)) : 0.f;
        }
        float* dp = dcs + r * D + 8 * cg;
        *reinterpret_cast<float4*>(dp) = make_float4(dcv[0], dcv[1], dcv[2], dcv[3]);
        *reinterpret_cast<float4*>(dp + 4) = make_float4(dcv[4], dcv[5], dcv[6], dcv[7]);
      } else if (r < nv) {
        *reinterpret_cast<bf16x8*>(dx + (size_t)(pos.t0 + r) * rowH + (size_t)h * D + 8 * cg) = pack8(dyv);
      }
    }
    if (P.conv) {
      __syncthreads();
      float acc[8][4];
#pragma unroll
      for (int cch = 0; cch < 8; ++cch) acc[cch][0] = acc[cch][1] = acc[cch][2] = acc[cch][3] = 0.f;
      for (int r = tg; r < nv; r += 16) {
        float dcr[4][8];
#pragma unroll
        for (int sidx = 0; sidx < 4; ++sidx) {
          const float* dp = dcs + (r + sidx) * D + 8 * cg;
          float4 a = *reinterpret_cast<const float4*>(dp);
          float4 b = *reinterpret_cast<const float4*>(dp + 4);
          dcr[sidx][0] = a.x; dcr[sidx][1] = a.y; dcr[sidx][2] = a.z; dcr[sidx][3] = a.w;
          dcr[sidx][4] = b.x; dcr[sidx][5] = b.y; dcr[sidx][6] = b.z; dcr[sidx][7] = b.w;
        }
        float xr[4][8];
#pragma unroll
        for (int sidx = 0; sidx < 4; ++sidx) unpack8(*reinterpret_cast<const bf16x8*>(xs + (r + sidx) * D + 8 * cg), xr[sidx]);
        float dxv[8];
#pragma unroll
        for (int cch = 0; cch < 8; ++cch) {
          // dx_t = sum_s w_s dc_(t+3-s): dc row r+3-s
          dxv[cch] = wt[cch][0] * dcr[3][cch] + wt[cch][1] * dcr[2][cch] + wt[cch][2] * dcr[1][cch] +
                     wt[cch][3] * dcr[0][cch];
          // dw_s += dc_t x_(t-3+s): x row r+s
#pragma unroll
          for (int sidx = 0; sidx < 4; ++sidx) acc[cch][sidx] += dcr[0][cch] * xr[sidx][cch];
        }
        *reinterpret_cast<bf16x8*>(dx + (size_t)(pos.t0 + r) * rowH + (size_t)h * D + 8 * cg) = pack8(dxv);
      }
#pragma unroll
      for (int tap = 0; tap < 4; ++tap) {
        float* dst = pw + (tg * 4 + tap) * D + 8 * cg;
        *reinterpret_cast<float4*>(dst) = make_float4(acc[0][tap], acc[1][tap], acc[2][tap], acc[3][tap]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[4][tap], acc[5][tap], acc[6][tap], acc[7][tap]);
      }
      __syncthreads();
      for (int i = tid; i < D * 4; i += blockDim.x) {
        // output layout [channel][tap]: i = channel * 4 + tap
        const int ch = i >> 2, tap = i & 3;
        float sum = 0.f;
#pragma unroll
        for (int u = 0; u < 16; ++u) sum += pw[(u * 4 + tap) * D + ch];
        P.partW[(((size_t)c * 3 + X) * H + h) * D * 4 + i] = sum;
      }
    }
    __syncthreads();
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
