// fp32 mode of the KDA layer: fp32 inputs, fp32 state and fp32 arithmetic
// throughout, on CUDA-core FMAs (no tensor-core rounding), forward and
// backward.  This is the configuration the reference itself runs in
// (SophiaKDA._reference_kda, ml/runtime/model/attention.py:260-294, float32
// inside) and the one flash-linear-attention's chunk_kda accepts for fp32
// q/k/v/g.  The recurrence is evaluated token by token in the reference's own
// order, so the forward agrees with the reference to fp32 rounding.
//
// Kernels (one call = prep -> fwd; bwd -> dc -> conv -> reduce):
//   kda_f32_prep_kernel   one warp per (chunk, head): ShortConv(k=4)+SiLU (when
//                         taps are given), L2 norms (q times scale), decay
//                         alpha = exp(lb * sigmoid(exp(A_log) (g + dt_bias))),
//                         beta = sigmoid(b).  Lane l owns channels 4l..4l+3.
//   kda_f32_fwd_kernel    one warp per (sequence, head, 16-column group); lanes
//                         j and j + 16 keep rows 0-63 and 64-127 of column j of
//                         the 128x128 state in registers (the row sums of the
//                         two halves meet in one shuffle):
//                           S <- diag(alpha) S; r = v - k^T S; S <- S + k (beta r)^T;
//                           o = q^T S
//                         and saves r, plus the state at every chunk start
//                         (checkpoints for the backward).
//   kda_f32_bwd_kernel    persistent, one CTA of 128 threads per (sequence,
//                         head, 32-column group) item; thread i keeps row i of
//                         this group's columns of dS.  Chunks run last to first:
//                         the states at every 8th token are recomputed from the
//                         chunk's checkpoint into a per-CTA scratch, then per
//                         block of 8 tokens (last first) that block's states
//                         (bit-identical to the forward's, 256 KB of scratch
//                         per CTA, so it stays in L2), and the tokens run in
//                         reverse:
//                           dS += q dO^T;  de = k^T dS (CTA reduction over rows);
//                           dv = beta de;  dbeta = de . r;  dpred = -beta de;
//                           dq = alpha (S_prev dO) + k (e . dO)
//                           dk = dS e + U dpred,  U = diag(alpha) S_prev
//                           dU = dS + k dpred^T;  dalpha = rowsum(dU o S_prev)
//                           dS <- diag(alpha) dU
//                         Columns of dS evolve independently, so the four column
//                         groups run in parallel and dq/dk/dalpha/dbeta leave as
//                         per-group partials summed (in a fixed order) later.
//   kda_f32_dc_kernel     one warp per (chunk, head): sums the partials, gate and
//                         beta backward (per-chunk partials of dA_log and
//                         dt_bias), L2-norm backward and SiLU backward.
//   kda_f32_conv_bwd_kernel  one warp per (chunk, head, tensor): conv backward
//                         dx_t = sum_s w_s dc_(t+3-s) and per-chunk tap partials.
// The partial sums go through kda_reduce_kernel (kda_post.cuh).
#pragma once

#include "kda_common.cuh"
#include "kda_tc.cuh"  // g_kda_device_error

namespace kda {

constexpr int F32_COLS = 32;                  // state columns per backward recurrence item
constexpr int F32_FWD_COLS = 16;              // state columns per forward warp (two lanes per column)
constexpr int F32_FWD_GROUPS = D / F32_FWD_COLS;
constexpr int F32_GROUPS = D / F32_COLS;      // column groups per (sequence, head)
constexpr int F32_WARPS_PER_CTA = 4;          // chunks per CTA of the row kernels
constexpr int F32_BWD_THREADS = 128;          // one thread per state row
constexpr int F32_SUB = 8;                    // tokens per recompute block of the backward
// per backward CTA: the states at every F32_SUB-th token of a chunk, then the
// F32_SUB states of one block (each 32 columns x 128 rows)
constexpr size_t F32_SCRATCH_FLOATS = (size_t)(C / F32_SUB + F32_SUB) * F32_COLS * D;
constexpr float F32_NORM_EPS = 1e-12f;        // F.normalize's eps

struct F32Inputs {
  const float *q, *k, *v, *g, *beta;           // [TT][H][128], beta [TT][H]
  const float *A_log, *dt_bias;                // [H], [H*128]
  const float *conv_q, *conv_k, *conv_v;       // [H*128][4] or null
  int H;
  bool conv;
  float scale, lower_bound;
};

struct F32PrepParams {
  SeqInfo seq;
  F32Inputs in;
  float *qh, *kh, *vh, *alpha;  // [TT][H][128]
  float* bt;                    // [TT][H]
};

__device__ __forceinline__ float4 f32_row(const float* base, long long t, bool ok, size_t rowH, int h, int lane) {
  if (!ok) return make_float4(0.f, 0.f, 0.f, 0.f);
  return __ldg(reinterpret_cast<const float4*>(base + (size_t)t * rowH + (size_t)h * D) + lane);
}
__device__ __forceinline__ void f4_to(const float4& v, float (&f)[4]) { f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w; }
__device__ __forceinline__ float4 to_f4(const float (&f)[4]) { return make_float4(f[0], f[1], f[2], f[3]); }

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) x += __shfl_xor_sync(0xffffffffu, x, m);
  return x;
}

__device__ __forceinline__ float sigmoid_exact(float x) { return 1.f / (1.f + expf(-x)); }

// Conv output c (pre-activation) of one row's four channels: out_t =
// w0 x_(t-3) + w1 x_(t-2) + w2 x_(t-1) + w3 x_t with x = 0 before the document
// start (attention.py:40-60: a zero history of K-1 positions, then conv1d).
__device__ __forceinline__ void f32_conv_row(const float* x, const float* taps, long long t, long long bos,
                                             size_t rowH, int h, int lane, float (&c)[4]) {
  float xs[4][4];
#pragma unroll
  for (int s = 0; s < 4; ++s) f4_to(f32_row(x, t - 3 + s, t - 3 + s >= bos, rowH, h, lane), xs[s]);
  const float4* w = reinterpret_cast<const float4*>(taps + ((size_t)h * D + 4 * lane) * 4);
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const float4 wt = __ldg(w + ch);
    c[ch] = wt.x * xs[0][ch] + wt.y * xs[1][ch] + wt.z * xs[2][ch] + wt.w * xs[3][ch];
  }
}

// Post-activation (conv + SiLU, or the raw input) of one row.
__device__ __forceinline__ void f32_act_row(const float* x, const float* taps, bool conv, long long t, long long bos,
                                            size_t rowH, int h, int lane, float (&y)[4], float (&c)[4]) {
  if (conv) {
    f32_conv_row(x, taps, t, bos, rowH, h, lane, c);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) y[ch] = c[ch] * sigmoid_exact(c[ch]);
  } else {
    f4_to(f32_row(x, t, true, rowH, h, lane), y);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) c[ch] = y[ch];
  }
}

__global__ void __launch_bounds__(32 * F32_WARPS_PER_CTA) kda_f32_prep_kernel(F32PrepParams P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * F32_WARPS_PER_CTA + warp, h = blockIdx.y;
  const F32Inputs& in = P.in;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const size_t rowH = (size_t)in.H * D;
  const float eA = expf(in.A_log[h]);
  float bias[4];
  f4_to(__ldg(reinterpret_cast<const float4*>(in.dt_bias + (size_t)h * D) + lane), bias);
  for (int t = pos.t0; t < pos.t1; ++t) {
    float yq[4], yk[4], yv[4], cc[4];
    f32_act_row(in.q, in.conv_q, in.conv, t, pos.bos, rowH, h, lane, yq, cc);
    f32_act_row(in.k, in.conv_k, in.conv, t, pos.bos, rowH, h, lane, yk, cc);
    f32_act_row(in.v, in.conv_v, in.conv, t, pos.bos, rowH, h, lane, yv, cc);
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) { sq += yq[ch] * yq[ch]; sk += yk[ch] * yk[ch]; }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float nq = fmaxf(sqrtf(sq), F32_NORM_EPS), nk = fmaxf(sqrtf(sk), F32_NORM_EPS);
    float gl[4], qo[4], ko[4], al[4];
    f4_to(f32_row(in.g, t, true, rowH, h, lane), gl);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      qo[ch] = yq[ch] / nq * in.scale;
      ko[ch] = yk[ch] / nk;
      al[ch] = expf(in.lower_bound * sigmoid_exact(eA * (gl[ch] + bias[ch])));
    }
    const size_t off = (size_t)t * rowH + (size_t)h * D;
    reinterpret_cast<float4*>(P.qh + off)[lane] = to_f4(qo);
    reinterpret_cast<float4*>(P.kh + off)[lane] = to_f4(ko);
    reinterpret_cast<float4*>(P.vh + off)[lane] = to_f4(yv);
    reinterpret_cast<float4*>(P.alpha + off)[lane] = to_f4(al);
    if (lane == 0) P.bt[(size_t)t * in.H + h] = sigmoid_exact(in.beta[(size_t)t * in.H + h]);
  }
}

struct F32FwdParams {
  SeqInfo seq;
  int H;
  const float *qh, *kh, *vh, *alpha, *bt;  // from the prep kernel
  const float* h0;                         // [N][H][128][128] or null
  float* o;                                // [TT][H][128]
  float* r;                                // [TT][H][128]: v - k^T S (saved for the backward) or null
  float* ck;                               // [H][slots] x [128][128] chunk-start states, or null
  float* ht;                               // [N][H][128][128] or null
  long long total_tokens;
};

__global__ void __launch_bounds__(32) kda_f32_fwd_kernel(F32FwdParams P) {
  __shared__ float4 sq[2][32], sk[2][32], sa[2][32];
  const int n = blockIdx.x, h = blockIdx.y, lane = threadIdx.x, H = P.H;
  const int col = blockIdx.z * F32_FWD_COLS + (lane & 15), r0 = 64 * (lane >> 4);  // column, first row
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  if (bos < 0 || eos < bos || (long long)eos > P.total_tokens) {  // malformed cu_seqlens: touch nothing
    if (lane == 0) atomicExch(&g_kda_device_error, 3);
    return;
  }
  const size_t rowH = (size_t)H * D, stateoff = ((size_t)n * H + h) * D * D;
  float S[64];  // rows r0 .. r0 + 63 of column col
#pragma unroll
  for (int i = 0; i < 64; ++i) S[i] = P.h0 ? P.h0[stateoff + (size_t)(r0 + i) * D + col] : 0.f;
  const int cbase = seq_chunk_base(P.seq, n);
  // register prefetch of the next token's vectors
  float4 nq = make_float4(0.f, 0.f, 0.f, 0.f), nk = nq, na = nq;
  float nb = 0.f, nv = 0.f;
  auto fetch = [&](int t) {
    const size_t off = (size_t)t * rowH + (size_t)h * D;
    nq = __ldg(reinterpret_cast<const float4*>(P.qh + off) + lane);
    nk = __ldg(reinterpret_cast<const float4*>(P.kh + off) + lane);
    na = __ldg(reinterpret_cast<const float4*>(P.alpha + off) + lane);
    nb = __ldg(P.bt + (size_t)t * H + h);
    nv = __ldg(P.vh + off + col);
  };
  if (bos < eos) fetch(bos);
  for (int t = bos; t < eos; ++t) {
    const int m = t - bos, buf = t & 1;
    if (P.ck && (m & (C - 1)) == 0) {
      float* dst = P.ck + tile_index(P.seq, cbase + m / C, h) * (size_t)STATE_ELEMS + (size_t)r0 * D + col;
#pragma unroll
      for (int i = 0; i < 64; ++i) dst[(size_t)i * D] = S[i];
    }
    sq[buf][lane] = nq;
    sk[buf][lane] = nk;
    sa[buf][lane] = na;
    const float beta = nb, vx = nv;
    if (t + 1 < eos) fetch(t + 1);
    __syncwarp();
    const float* qv = reinterpret_cast<const float*>(sq[buf]) + r0;
    const float* kv = reinterpret_cast<const float*>(sk[buf]) + r0;
    const float* av = reinterpret_cast<const float*>(sa[buf]) + r0;
    float p0 = 0.f, p1 = 0.f, p2 = 0.f, p3 = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      S[i] *= av[i];
      S[i + 1] *= av[i + 1];
      S[i + 2] *= av[i + 2];
      S[i + 3] *= av[i + 3];
      p0 = fmaf(kv[i], S[i], p0);
      p1 = fmaf(kv[i + 1], S[i + 1], p1);
      p2 = fmaf(kv[i + 2], S[i + 2], p2);
      p3 = fmaf(kv[i + 3], S[i + 3], p3);
    }
    float pr = (p0 + p1) + (p2 + p3);
    pr += __shfl_xor_sync(0xffffffffu, pr, 16);  // the other row half of the column
    const float rr = vx - pr;
    const float e = rr * beta;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      S[i] = fmaf(kv[i], e, S[i]);
      S[i + 1] = fmaf(kv[i + 1], e, S[i + 1]);
      S[i + 2] = fmaf(kv[i + 2], e, S[i + 2]);
      S[i + 3] = fmaf(kv[i + 3], e, S[i + 3]);
      o0 = fmaf(qv[i], S[i], o0);
      o1 = fmaf(qv[i + 1], S[i + 1], o1);
      o2 = fmaf(qv[i + 2], S[i + 2], o2);
      o3 = fmaf(qv[i + 3], S[i + 3], o3);
    }
    float ov = (o0 + o1) + (o2 + o3);
    ov += __shfl_xor_sync(0xffffffffu, ov, 16);
    if (lane < 16) {
      const size_t off = (size_t)t * rowH + (size_t)h * D + col;
      P.o[off] = ov;
      if (P.r) P.r[off] = rr;
    }
    __syncwarp();  // buffer `buf` is rewritten two tokens later
  }
  if (P.ht) {
#pragma unroll
    for (int i = 0; i < 64; ++i) P.ht[stateoff + (size_t)(r0 + i) * D + col] = S[i];
  }
}

struct F32BwdParams {
  SeqInfo seq;
  int H;
  const float *qh, *kh, *alpha, *bt, *r, *ck;  // saved by the forward
  const float* dO;                             // [TT][H][128]
  const float* dht;                            // [N][H][128][128] or null
  float* scratch;                              // [gridDim.x][8 + 8][32][128]
  float *dqh_p, *dkh_p, *dal_p;                // [F32_GROUPS][TT][H][128] partials
  float* dbt_p;                                // [F32_GROUPS][TT][H]
  float* dvh;                                  // [TT][H][128]
  float* dh0;                                  // [N][H][128][128] or null
  long long total_tokens;
  int items;                                   // N * H * F32_GROUPS
};

// Sum over the 32 lanes of v[j], j = 0..31, ending with lane l holding the sum for
// j = l: five halving steps, each lane keeping the half of its values whose index
// bit matches its lane bit and adding its partner's copy of that half.
__device__ __forceinline__ float warp_reduce_scatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool up = lane & half;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float send = up ? v[j] : v[j + half];
      const float keep = up ? v[j + half] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
  return v[0];
}

struct F32BwdSmem {
  float rs[C][F32_COLS];           // r of this group's columns for the chunk's tokens
  float bs[C];                     // beta of the chunk's tokens
  float part[4][F32_COLS];         // per-warp partial sums of de
  float dov[2][F32_COLS];          // dO_t of this group's columns
  float rv[2][F32_COLS];           // r_t of this group's columns
  float de[2][F32_COLS];
  float ed[2];                     // e_t . dO_t over this group's columns
};

__global__ void __launch_bounds__(F32_BWD_THREADS, 4) kda_f32_bwd_kernel(F32BwdParams P) {
  __shared__ F32BwdSmem sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, H = P.H;
  const int i = tid;  // state row of this thread
  const size_t rowH = (size_t)H * D;
  float* scr = P.scratch + (size_t)blockIdx.x * F32_SCRATCH_FLOATS;
  for (int item = blockIdx.x; item < P.items; item += gridDim.x) {
    const int grp = item % F32_GROUPS, nh = item / F32_GROUPS, h = nh % H, n = nh / H;
    const int col0 = grp * F32_COLS;
    const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
    if (bos < 0 || eos < bos || (long long)eos > P.total_tokens) {  // block-uniform
      if (tid == 0) atomicExch(&g_kda_device_error, 3);
      continue;
    }
    const size_t stateoff = ((size_t)n * H + h) * D * D + (size_t)i * D + col0;
    float dS[F32_COLS];
#pragma unroll
    for (int j = 0; j < F32_COLS; j += 4) {
      const float4 v = P.dht ? *reinterpret_cast<const float4*>(P.dht + stateoff + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      dS[j] = v.x; dS[j + 1] = v.y; dS[j + 2] = v.z; dS[j + 3] = v.w;
    }
    const int nchunks = (eos - bos + C - 1) / C, cbase = seq_chunk_base(P.seq, n);
    for (int ci = nchunks - 1; ci >= 0; --ci) {
      const int t0 = bos + ci * C, t1 = min(t0 + C, eos), L = t1 - t0;
      // ---- states of row i, this group's columns, in [slot][j][i] order: the one
      //      before token t0 + 8 b in slot b of the block-start area, then the ones
      //      before the tokens of one block in the block area
      float* const sblk = scr + (size_t)(C / F32_SUB) * F32_COLS * D;
      // the chunk's r (this group's columns) and beta, staged once for the recompute
      for (int e = tid; e < L * (F32_COLS / 4); e += F32_BWD_THREADS) {
        const int m = e / (F32_COLS / 4), j4 = e % (F32_COLS / 4);
        reinterpret_cast<float4*>(sm.rs[m])[j4] =
            __ldg(reinterpret_cast<const float4*>(P.r + (size_t)(t0 + m) * rowH + (size_t)h * D + col0) + j4);
      }
      if (tid < L) sm.bs[tid] = P.bt[(size_t)(t0 + tid) * H + h];
      __syncthreads();
      // S <- the state after token t0 + m (the forward's update, bit for bit), with this
      // row's alpha and k of that token
      auto step = [&](float (&S)[F32_COLS], int m, float a, float kk) {
        const float beta = sm.bs[m];
        const float4* rr = reinterpret_cast<const float4*>(sm.rs[m]);
#pragma unroll
        for (int j = 0; j < F32_COLS; j += 4) {
          const float4 r4 = rr[j / 4];
          S[j] = fmaf(kk, r4.x * beta, a * S[j]);
          S[j + 1] = fmaf(kk, r4.y * beta, a * S[j + 1]);
          S[j + 2] = fmaf(kk, r4.z * beta, a * S[j + 2]);
          S[j + 3] = fmaf(kk, r4.w * beta, a * S[j + 3]);
        }
      };
      // row i's alpha and k of token t0 + m
      auto ak = [&](int m, float& a, float& kk) {
        const size_t off = (size_t)(t0 + m) * rowH + (size_t)h * D + i;
        a = P.alpha[off];
        kk = P.kh[off];
      };
      auto put = [&](float* area, int slot, const float (&S)[F32_COLS]) {
        float* dst = area + (size_t)slot * F32_COLS * D + i;
#pragma unroll
        for (int j = 0; j < F32_COLS; ++j) dst[(size_t)j * D] = S[j];
      };
      auto get = [&](const float* area, int slot, float (&S)[F32_COLS]) {
        const float* src = area + (size_t)slot * F32_COLS * D + i;
#pragma unroll
        for (int j = 0; j < F32_COLS; ++j) S[j] = src[(size_t)j * D];
      };
      {
        float S[F32_COLS];
        const float* src = P.ck + tile_index(P.seq, cbase + ci, h) * (size_t)STATE_ELEMS + (size_t)i * D + col0;
#pragma unroll
        for (int j = 0; j < F32_COLS; j += 4) {
          const float4 v = *reinterpret_cast<const float4*>(src + j);
          S[j] = v.x; S[j + 1] = v.y; S[j + 2] = v.z; S[j + 3] = v.w;
        }
        const int mlast = ((L - 1) / F32_SUB) * F32_SUB;  // the last block's first token
        float na = 0.f, nk = 0.f;  // the next step's alpha and k, loaded a step ahead
        if (mlast > 0) ak(0, na, nk);
        for (int m = 0; m < mlast; ++m) {
          if (m % F32_SUB == 0) put(scr, m / F32_SUB, S);
          const float a = na, kk = nk;
          if (m + 1 < mlast) ak(m + 1, na, nk);
          step(S, m, a, kk);
        }
        put(scr, mlast / F32_SUB, S);
      }
      for (int blk = (L - 1) / F32_SUB; blk >= 0; --blk) {
        const int mb0 = blk * F32_SUB, mb1 = min(mb0 + F32_SUB, L);
        {
          float S[F32_COLS];
          get(scr, blk, S);
          float na = 0.f, nk = 0.f;
          if (mb0 + 1 < mb1) ak(mb0, na, nk);
          for (int m = mb0; m < mb1; ++m) {
            put(sblk, m - mb0, S);
            if (m + 1 < mb1) {
              const float a = na, kk = nk;
              if (m + 2 < mb1) ak(m + 1, na, nk);
              step(S, m, a, kk);
            }
          }
        }
        __syncthreads();  // (each thread reads back only its own row; keeps the order simple)
        // ---- reverse over the block's tokens; each token's inputs are loaded while
        //      the token after it computes
        float nx = 0.f, nq, nk, na, nb;  // token m's dO / r column (threads < 64), q, k, alpha of row i, beta
        auto load_token = [&](int m) {
          const size_t off = (size_t)(t0 + m) * rowH + (size_t)h * D;
          if (tid < F32_COLS) nx = P.dO[off + col0 + tid];
          else if (tid < 2 * F32_COLS) nx = P.r[off + col0 + tid - F32_COLS];
          nq = P.qh[off + i];
          nk = P.kh[off + i];
          na = P.alpha[off + i];
          nb = P.bt[(size_t)(t0 + m) * H + h];
        };
        load_token(mb1 - 1);
        for (int m = mb1 - 1; m >= mb0; --m) {
          const int t = t0 + m, b = m & 1;
          const size_t off = (size_t)t * rowH + (size_t)h * D;
          if (tid < F32_COLS) sm.dov[b][tid] = nx;
          else if (tid < 2 * F32_COLS) sm.rv[b][tid - F32_COLS] = nx;
          const float qi = nq, ki = nk, ai = na, beta = nb;
          if (m > mb0) load_token(m - 1);
          __syncthreads();
          {
            // de_j = sum_i k_i dS[i][j]: warp w's rows 32w .. 32w+31 in registers (lane
            // `lane` ends with column `lane`), then the four warps' sums
            float kd[F32_COLS];
#pragma unroll
            for (int j = 0; j < F32_COLS; ++j) {
              dS[j] = fmaf(qi, sm.dov[b][j], dS[j]);
              kd[j] = ki * dS[j];
            }
            sm.part[warp][lane] = warp_reduce_scatter32(kd);
          }
          __syncthreads();
          if (warp == 0) {
            const float de = (sm.part[0][lane] + sm.part[1][lane]) + (sm.part[2][lane] + sm.part[3][lane]);
            const float rj = sm.rv[b][lane];
            P.dvh[off + col0 + lane] = beta * de;
            const float db = warp_sum(de * rj);
            const float ed = warp_sum(rj * beta * sm.dov[b][lane]);
            if (lane == 0) {
              P.dbt_p[((size_t)grp * P.total_tokens + t) * H + h] = db;
              sm.ed[b] = ed;
            }
            sm.de[b][lane] = de;
          }
          __syncthreads();
          const float* sp = sblk + (size_t)(m - mb0) * F32_COLS * D + i;
          float dq0 = 0.f, dq1 = 0.f, dk0 = 0.f, dk1 = 0.f, da0 = 0.f, da1 = 0.f;
#pragma unroll
          for (int j = 0; j < F32_COLS; j += 2) {
            const float sp0 = sp[(size_t)j * D], sp1 = sp[(size_t)(j + 1) * D];
            const float dp0 = -beta * sm.de[b][j], dp1 = -beta * sm.de[b][j + 1];
            const float e0 = sm.rv[b][j] * beta, e1 = sm.rv[b][j + 1] * beta;
            dq0 = fmaf(sp0, sm.dov[b][j], dq0);
            dq1 = fmaf(sp1, sm.dov[b][j + 1], dq1);
            dk0 = fmaf(dS[j], e0, fmaf(dp0, ai * sp0, dk0));
            dk1 = fmaf(dS[j + 1], e1, fmaf(dp1, ai * sp1, dk1));
            const float du0 = fmaf(ki, dp0, dS[j]), du1 = fmaf(ki, dp1, dS[j + 1]);
            da0 = fmaf(du0, sp0, da0);
            da1 = fmaf(du1, sp1, da1);
            dS[j] = ai * du0;
            dS[j + 1] = ai * du1;
          }
          const size_t poff = (size_t)grp * P.total_tokens * rowH + off + i;
          P.dqh_p[poff] = fmaf(ai, dq0 + dq1, ki * sm.ed[b]);
          P.dkh_p[poff] = dk0 + dk1;
          P.dal_p[poff] = da0 + da1;
        }
        __syncthreads();  // the block area is rewritten by the next block
      }
    }
    if (P.dh0) {
#pragma unroll
      for (int j = 0; j < F32_COLS; j += 4)
        *reinterpret_cast<float4*>(P.dh0 + stateoff + j) = make_float4(dS[j], dS[j + 1], dS[j + 2], dS[j + 3]);
    }
  }
}

struct F32DcParams {
  SeqInfo seq;
  F32Inputs in;
  long long total_tokens;
  const float *dqh_p, *dkh_p, *dal_p, *dbt_p, *dvh;
  const float *alpha, *bt;  // saved
  float *dq, *dk, *dv;      // without conv: the input gradients; with conv: dc (pre-SiLU) of q, k, v
  float *dg, *dbeta;        // gate-logit and beta-logit gradients
  float *partA, *partB;     // [chunks][H][128]
};

// Gradient of y / max(|y|, eps) * s with respect to y, given the output gradient dn (warp-wide rows).
__device__ __forceinline__ void f32_norm_bwd(const float (&y)[4], const float (&dn)[4], float s, float (&dy)[4]) {
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) { ss += y[ch] * y[ch]; dot += y[ch] * dn[ch]; }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float nrm = sqrtf(ss);
  if (nrm > F32_NORM_EPS) {
    const float inv = 1.f / nrm;
    const float proj = dot * inv * inv;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dy[ch] = s * inv * (dn[ch] - y[ch] * proj);
  } else {
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) dy[ch] = s * dn[ch] / F32_NORM_EPS;
  }
}

__device__ __forceinline__ float silu_grad(float c) {
  const float sg = sigmoid_exact(c);
  return sg * (1.f + c * (1.f - sg));
}

__global__ void __launch_bounds__(32 * F32_WARPS_PER_CTA) kda_f32_dc_kernel(F32DcParams P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * F32_WARPS_PER_CTA + warp, h = blockIdx.y;
  const F32Inputs& in = P.in;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int H = in.H;
  const size_t rowH = (size_t)H * D, gstride = (size_t)P.total_tokens * rowH;
  const float eA = expf(in.A_log[h]);
  float bias[4], pa[4] = {0.f, 0.f, 0.f, 0.f}, pb[4] = {0.f, 0.f, 0.f, 0.f};
  f4_to(__ldg(reinterpret_cast<const float4*>(in.dt_bias + (size_t)h * D) + lane), bias);
  for (int t = pos.t0; t < pos.t1; ++t) {
    const size_t off = (size_t)t * rowH + (size_t)h * D;
    float dqh[4] = {0.f, 0.f, 0.f, 0.f}, dkh[4] = {0.f, 0.f, 0.f, 0.f}, dal[4] = {0.f, 0.f, 0.f, 0.f};
    float dbt = 0.f;
#pragma unroll
    for (int gI = 0; gI < F32_GROUPS; ++gI) {  // fixed order
      float a4[4], b4[4], c4[4];
      f4_to(__ldg(reinterpret_cast<const float4*>(P.dqh_p + gI * gstride + off) + lane), a4);
      f4_to(__ldg(reinterpret_cast<const float4*>(P.dkh_p + gI * gstride + off) + lane), b4);
      f4_to(__ldg(reinterpret_cast<const float4*>(P.dal_p + gI * gstride + off) + lane), c4);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) { dqh[ch] += a4[ch]; dkh[ch] += b4[ch]; dal[ch] += c4[ch]; }
      dbt += __ldg(P.dbt_p + ((size_t)gI * P.total_tokens + t) * H + h);
    }
    // gate: alpha = exp(lb * sigmoid(z)), z = exp(A_log) (g + dt_bias)
    float gl[4], al[4], dgl[4];
    f4_to(f32_row(in.g, t, true, rowH, h, lane), gl);
    f4_to(f32_row(P.alpha, t, true, rowH, h, lane), al);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      const float z = eA * (gl[ch] + bias[ch]);
      const float sg = sigmoid_exact(z);
      const float dz = dal[ch] * al[ch] * in.lower_bound * sg * (1.f - sg);
      dgl[ch] = dz * eA;
      pb[ch] += dgl[ch];
      pa[ch] += dz * z;
    }
    reinterpret_cast<float4*>(P.dg + off)[lane] = to_f4(dgl);
    if (lane == 0) {
      const float bt = P.bt[(size_t)t * H + h];
      P.dbeta[(size_t)t * H + h] = dbt * bt * (1.f - bt);
    }
    // q and k: L2-norm backward, then SiLU backward when the conv is fused
    float y[4], cc[4], dy[4];
    f32_act_row(in.q, in.conv_q, in.conv, t, pos.bos, rowH, h, lane, y, cc);
    f32_norm_bwd(y, dqh, in.scale, dy);
    if (in.conv) {
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) dy[ch] *= silu_grad(cc[ch]);
    }
    reinterpret_cast<float4*>(P.dq + off)[lane] = to_f4(dy);
    f32_act_row(in.k, in.conv_k, in.conv, t, pos.bos, rowH, h, lane, y, cc);
    f32_norm_bwd(y, dkh, 1.f, dy);
    if (in.conv) {
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) dy[ch] *= silu_grad(cc[ch]);
    }
    reinterpret_cast<float4*>(P.dk + off)[lane] = to_f4(dy);
    f4_to(f32_row(P.dvh, t, true, rowH, h, lane), dy);
    if (in.conv) {
      f32_conv_row(in.v, in.conv_v, t, pos.bos, rowH, h, lane, cc);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) dy[ch] *= silu_grad(cc[ch]);
    }
    reinterpret_cast<float4*>(P.dv + off)[lane] = to_f4(dy);
  }
  const size_t poff = ((size_t)c * H + h) * D;
  reinterpret_cast<float4*>(P.partA + poff)[lane] = to_f4(pa);
  reinterpret_cast<float4*>(P.partB + poff)[lane] = to_f4(pb);
}

struct F32ConvParams {
  SeqInfo seq;
  F32Inputs in;
  const float *dcq, *dck, *dcv;  // pre-SiLU gradients
  float *dq, *dk, *dv;           // input gradients
  float* partW;                  // [chunks][3][H][128][4]
};

// Conv backward of one (chunk, head, tensor): dx_t = sum_s w_s dc_(t+3-s) over
// t+3-s inside the document, and the chunk's tap partials
// dw_s = sum_t dc_t x_(t-3+s) over its rows t (x = 0 before the document).
__global__ void __launch_bounds__(32 * F32_WARPS_PER_CTA) kda_f32_conv_bwd_kernel(F32ConvParams P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * F32_WARPS_PER_CTA + warp, h = blockIdx.y, X = blockIdx.z;
  const F32Inputs& in = P.in;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int H = in.H;
  const int eos = seq_eos(P.seq, pos.seq);
  const size_t rowH = (size_t)H * D;
  const float* x = X == 0 ? in.q : (X == 1 ? in.k : in.v);
  const float* dc = X == 0 ? P.dcq : (X == 1 ? P.dck : P.dcv);
  float* dx = X == 0 ? P.dq : (X == 1 ? P.dk : P.dv);
  const float* taps = X == 0 ? in.conv_q : (X == 1 ? in.conv_k : in.conv_v);
  float w[4][4];
  {
    const float4* wp = reinterpret_cast<const float4*>(taps + ((size_t)h * D + 4 * lane) * 4);
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      const float4 t4 = __ldg(wp + ch);
      w[ch][0] = t4.x; w[ch][1] = t4.y; w[ch][2] = t4.z; w[ch][3] = t4.w;
    }
  }
  float acc[4][4] = {};
  for (int t = pos.t0; t < pos.t1; ++t) {
    float d[4][4], xs[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      f4_to(f32_row(dc, t + s, t + s < eos, rowH, h, lane), d[s]);     // dc_(t+s)
      f4_to(f32_row(x, t - 3 + s, t - 3 + s >= pos.bos, rowH, h, lane), xs[s]);  // x_(t-3+s)
    }
    float o[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      // dx_t = w3 dc_t + w2 dc_(t+1) + w1 dc_(t+2) + w0 dc_(t+3)
      o[ch] = w[ch][3] * d[0][ch] + w[ch][2] * d[1][ch] + w[ch][1] * d[2][ch] + w[ch][0] * d[3][ch];
#pragma unroll
      for (int s = 0; s < 4; ++s) acc[ch][s] = fmaf(d[0][ch], xs[s][ch], acc[ch][s]);
    }
    reinterpret_cast<float4*>(dx + (size_t)t * rowH + (size_t)h * D)[lane] = to_f4(o);
  }
  float4* dst = reinterpret_cast<float4*>(P.partW + (((size_t)c * 3 + X) * H + h) * D * 4) + 4 * lane;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) dst[ch] = make_float4(acc[ch][0], acc[ch][1], acc[ch][2], acc[ch][3]);
}

}  // namespace kda
