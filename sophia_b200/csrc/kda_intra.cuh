// Intra-chunk stages shared by the forward and backward chunk kernels.
//
// One CTA of 256 threads owns one (chunk, head).  Elementwise work uses the
// "strip" mapping: thread tid owns tokens 4*tg .. 4*tg+3 (tg = tid / 16) and
// channels 8*cg .. 8*cg+7 (cg = tid % 16); the 16 threads of a half-warp share
// a token group, so a row reduction over 128 channels is a 16-lane shuffle.
//
// Overflow-safe factorisation of exp(Gam_i - Gam_j) (per channel, i >= j):
//   diagonal 16x16 block (I == J):   a_i * ia_j,   a = 2^(Gam - Gam_r(I)) <= 1,
//                                                  ia = 1/a >= 1 (<= 2^116),
//   off-diagonal block (I > J):      a_i * c_IJ * b_j,  c_IJ = 2^(Gam_r(I) - Gam_e(J)),
//                                                  b = 2^(Gam_e(J) - Gam) <= 1,
// with r(I) the first and e(J) the last token of a sub-chunk.  Every factor is
// bounded because the reference clamps the per-token log decay to [lb, 0) with
// lb >= -5 (sixteen tokens span at most 80 nats), and a factor that underflows
// only does so when the exact product underflows too.
#pragma once

#include "kda_common.cuh"

namespace kda {

// Per-channel ShortConv taps (fp32 [H*128][4]) of one tensor.
struct ConvTaps { const float* w; };

struct PrologueIn {
  const bf16* q; const bf16* k; const bf16* v;  // [T_total][H][128] (pre-conv if conv)
  const bf16* g; const bf16* beta;              // [T_total][H][128], [T_total][H]
  const float* A_log; const float* dt_bias;     // [H], [H*128]
  const float* conv_q; const float* conv_k; const float* conv_v;  // [H*128][4] or null
  int H;
  float scale, lower_bound;
};

// Shared-memory views used by the prologue.
struct PrologueSmem {
  bf16* xq; bf16* xk; bf16* xv;  // [67][128] raw rows t0-3 .. t0+63 (row stride 128)
  bf16* graw;                    // [64][128]
  bf16* braw;                    // [64]
  float* gam;                    // [64][128] log2 cumulative decay
  float* beta;                   // [64]
  float* tot;                    // [16][128] scratch for the cumsum
};

// Issue cp.async loads of the raw chunk inputs (zero fill outside [bos, t1)).
__device__ __forceinline__ void prologue_issue_loads(const PrologueIn& in, const PrologueSmem& sm,
                                                     const ChunkPos& p, int h, bool conv) {
  const int tid = threadIdx.x;
  const size_t rowH = (size_t)in.H * D;
  // q/k/v: 67 rows x 16 chunks of 16 bytes each
  for (int i = tid; i < 3 * 67 * 16; i += blockDim.x) {
    int tsel = i / (67 * 16);
    int rem = i - tsel * 67 * 16;
    int r = rem >> 4, cc = rem & 15;
    int t = p.t0 - 3 + r;
    bool ok = (t >= p.bos) && (t < p.t1) && (conv || r >= 3);
    const bf16* src = tsel == 0 ? in.q : (tsel == 1 ? in.k : in.v);
    bf16* dst = tsel == 0 ? sm.xq : (tsel == 1 ? sm.xk : sm.xv);
    const bf16* gp = src + (ok ? ((size_t)t * rowH + (size_t)h * D + cc * 8) : 0);
    cp_async16(dst + r * D + cc * 8, gp, ok);
  }
  for (int i = tid; i < 64 * 16; i += blockDim.x) {
    int r = i >> 4, cc = i & 15;
    int t = p.t0 + r;
    bool ok = t < p.t1;
    const bf16* gp = in.g + (ok ? ((size_t)t * rowH + (size_t)h * D + cc * 8) : 0);
    cp_async16(sm.graw + r * D + cc * 8, gp, ok);
  }
  if (tid < 64) {
    int t = p.t0 + tid;
    sm.braw[tid] = (t < p.t1) ? in.beta[(size_t)t * in.H + h] : __float2bfloat16(0.f);
  }
}

// Elementwise prologue.  On return (after the trailing __syncthreads) sm.gam
// and sm.beta are complete and the calling thread holds its strip of the
// normalised (q scaled) q, k, post-conv v and log2 decays.
struct Strip {
  float q[4][8], k[4][8], v[4][8], gam[4][8];
};

__device__ __forceinline__ void conv_strip(const bf16* x, const float* w, int tg, int cg, bool conv,
                                           float (&out)[4][8]) {
  if (conv) {
    float xs[7][8];
#pragma unroll
    for (int r = 0; r < 7; ++r) {
      bf16x8 v = *reinterpret_cast<const bf16x8*>(x + (4 * tg + r) * D + 8 * cg);
      unpack8(v, xs[r]);
    }
    float wt[8][4];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float4 t4 = __ldg(reinterpret_cast<const float4*>(w) + (8 * cg + c));
      wt[c][0] = t4.x; wt[c][1] = t4.y; wt[c][2] = t4.z; wt[c][3] = t4.w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float a = wt[c][0] * xs[r][c] + wt[c][1] * xs[r + 1][c] + wt[c][2] * xs[r + 2][c] +
                  wt[c][3] * xs[r + 3][c];
        out[r][c] = a * sigmoidf_(a);
      }
  } else {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      bf16x8 v = *reinterpret_cast<const bf16x8*>(x + (3 + 4 * tg + r) * D + 8 * cg);
      unpack8(v, out[r]);
    }
  }
}

__device__ __forceinline__ void prologue_compute(const PrologueIn& in, const PrologueSmem& sm,
                                                 const ChunkPos& p, int h, bool conv, Strip& s) {
  const int tid = threadIdx.x;
  const int tg = tid >> 4, cg = tid & 15;
  const int nvalid = p.t1 - p.t0;
  const float* wq = conv ? in.conv_q + (size_t)h * D * 4 : nullptr;
  const float* wk = conv ? in.conv_k + (size_t)h * D * 4 : nullptr;
  const float* wv = conv ? in.conv_v + (size_t)h * D * 4 : nullptr;
  conv_strip(sm.xq, wq, tg, cg, conv, s.q);
  conv_strip(sm.xk, wk, tg, cg, conv, s.k);
  conv_strip(sm.xv, wv, tg, cg, conv, s.v);
  // mask padded tokens, L2 normalise q and k per token (reduction over 16 lanes)
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    bool ok = 4 * tg + r < nvalid;
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (!ok) { s.q[r][c] = 0.f; s.k[r][c] = 0.f; s.v[r][c] = 0.f; }
      sq += s.q[r][c] * s.q[r][c];
      sk += s.k[r][c] * s.k[r][c];
    }
#pragma unroll
    for (int m = 8; m >= 1; m >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, m);
      sk += __shfl_xor_sync(0xffffffffu, sk, m);
    }
    float rq = in.scale / fmaxf(sqrtf(sq), 1e-12f);
    float rk = 1.f / fmaxf(sqrtf(sk), 1e-12f);
#pragma unroll
    for (int c = 0; c < 8; ++c) { s.q[r][c] *= rq; s.k[r][c] *= rk; }
  }
  // gate: g = lb * sigmoid(exp(A_log) * (x + dt_bias)), log2 units, prefix sum
  const float eA = __expf(__ldg(in.A_log + h));
  float bias[8];
  {
    float4 b0 = __ldg(reinterpret_cast<const float4*>(in.dt_bias + (size_t)h * D + 8 * cg));
    float4 b1 = __ldg(reinterpret_cast<const float4*>(in.dt_bias + (size_t)h * D + 8 * cg + 4));
    bias[0] = b0.x; bias[1] = b0.y; bias[2] = b0.z; bias[3] = b0.w;
    bias[4] = b1.x; bias[5] = b1.y; bias[6] = b1.z; bias[7] = b1.w;
  }
  float run[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) run[c] = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float gx[8];
    unpack8(*reinterpret_cast<const bf16x8*>(sm.graw + (4 * tg + r) * D + 8 * cg), gx);
    bool ok = 4 * tg + r < nvalid;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float z = eA * (gx[c] + bias[c]);
      float gv = ok ? in.lower_bound * sigmoidf_(z) * LOG2E : 0.f;
      run[c] += gv;
      s.gam[r][c] = run[c];
    }
  }
  *reinterpret_cast<float4*>(sm.tot + tg * D + 8 * cg) = make_float4(run[0], run[1], run[2], run[3]);
  *reinterpret_cast<float4*>(sm.tot + tg * D + 8 * cg + 4) = make_float4(run[4], run[5], run[6], run[7]);
  if (tid < 64) {
    float b = __bfloat162float(sm.braw[tid]);
    sm.beta[tid] = (tid < nvalid) ? sigmoidf_(b) : 0.f;
  }
  __syncthreads();
  float off[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) off[c] = 0.f;
  for (int u = 0; u < tg; ++u) {
    float4 a = *reinterpret_cast<const float4*>(sm.tot + u * D + 8 * cg);
    float4 b = *reinterpret_cast<const float4*>(sm.tot + u * D + 8 * cg + 4);
    off[0] += a.x; off[1] += a.y; off[2] += a.z; off[3] += a.w;
    off[4] += b.x; off[5] += b.y; off[6] += b.z; off[7] += b.w;
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
#pragma unroll
    for (int c = 0; c < 8; ++c) s.gam[r][c] += off[c];
    float* gp = sm.gam + (4 * tg + r) * D + 8 * cg;
    *reinterpret_cast<float4*>(gp) = make_float4(s.gam[r][0], s.gam[r][1], s.gam[r][2], s.gam[r][3]);
    *reinterpret_cast<float4*>(gp + 4) = make_float4(s.gam[r][4], s.gam[r][5], s.gam[r][6], s.gam[r][7]);
  }
  __syncthreads();
}

// Operand tiles (bf16, row stride LD128) built from the strip.
struct Operands {
  bf16* Qa;  // q * a        (row-side, reference r(I))
  bf16* Ka;  // k * a
  bf16* Kd;  // k / a        (column side of diagonal blocks)
  bf16* Kb;  // k * b        (column side of off-diagonal blocks, reference e(J))
  bf16* V;   // v
  bf16* Ke;  // k * 2^Gam
  float* cvec;  // [6][128] c_IJ = 2^(Gam_r(I) - Gam_e(J)), pair p = I(I-1)/2 + J
  float* er;    // [4][128] 2^Gam_r(J)           (may be null)
  float* ec;    // [4][128] 2^(Gam_C - Gam_e(J)) (may be null)
};

__device__ __forceinline__ int pair_index(int I, int J) { return I * (I - 1) / 2 + J; }

// Builds the operand tiles; optionally also returns the strip of q*2^Gam and
// k*2^(Gam_C - Gam) (the forward's Qt and Kbar) through qt/kbar.
template <bool WANT_QK_DECAYED>
__device__ __forceinline__ void build_operands(const Strip& s, const float* gam, const Operands& op,
                                               float (*qt)[8], float (*kbar)[8]) {
  const int tid = threadIdx.x;
  const int tg = tid >> 4, cg = tid & 15;
  const int J = tg >> 2;
  const float* grow = gam + (16 * J) * D + 8 * cg;       // row r(J)
  const float* gend = gam + (16 * J + 15) * D + 8 * cg;  // row e(J)
  const float* gC = gam + 63 * D + 8 * cg;               // row C-1
  float Gr[8], Ge[8], erv[8], ecv[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    Gr[c] = grow[c];
    Ge[c] = gend[c];
    erv[c] = ex2(Gr[c]);
    ecv[c] = ex2(gC[c] - Ge[c]);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float qa[8], ka[8], kd[8], kb[8], ke[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float G = s.gam[r][c];
      float a = ex2(G - Gr[c]);
      float ia = ex2(Gr[c] - G);
      float b = ex2(Ge[c] - G);
      qa[c] = s.q[r][c] * a;
      ka[c] = s.k[r][c] * a;
      kd[c] = s.k[r][c] * ia;
      kb[c] = s.k[r][c] * b;
      ke[c] = s.k[r][c] * (a * erv[c]);
      if (WANT_QK_DECAYED) {
        qt[r][c] = s.q[r][c] * (a * erv[c]);
        kbar[r][c] = s.k[r][c] * (b * ecv[c]);
      }
    }
    int row = (4 * tg + r) * LD128 + 8 * cg;
    *reinterpret_cast<bf16x8*>(op.Qa + row) = pack8(qa);
    *reinterpret_cast<bf16x8*>(op.Ka + row) = pack8(ka);
    *reinterpret_cast<bf16x8*>(op.Kd + row) = pack8(kd);
    *reinterpret_cast<bf16x8*>(op.Kb + row) = pack8(kb);
    *reinterpret_cast<bf16x8*>(op.V + row) = pack8(s.v[r]);
    *reinterpret_cast<bf16x8*>(op.Ke + row) = pack8(ke);
  }
  // per-pair and per-sub-chunk channel vectors
  for (int i = tid; i < 6 * D; i += blockDim.x) {
    int pidx = i / D, d = i - pidx * D;
    int I = pidx >= 3 ? 3 : (pidx >= 1 ? 2 : 1);
    int Jp = pidx - pair_index(I, 0);
    op.cvec[i] = ex2(gam[(16 * I) * D + d] - gam[(16 * Jp + 15) * D + d]);
  }
  if (op.er) {
    for (int i = tid; i < 4 * D; i += blockDim.x) {
      int Jp = i / D, d = i - Jp * D;
      op.er[i] = ex2(gam[(16 * Jp) * D + d]);
      op.ec[i] = ex2(gam[63 * D + d] - gam[(16 * Jp + 15) * D + d]);
    }
  }
}

// Scales the 8 bf16 elements of an A fragment (k columns k0+2t, +1, +8, +9) by
// per-channel factors.
__device__ __forceinline__ void scale_A_frag(uint32_t (&a)[4], const float* sv, int k0) {
  const int t = threadIdx.x & 3;
  float s0 = sv[k0 + 2 * t], s1 = sv[k0 + 2 * t + 1];
  float s2 = sv[k0 + 8 + 2 * t], s3 = sv[k0 + 9 + 2 * t];
  float2 x;
  x = unpack_bf16(a[0]); a[0] = pack_bf16(x.x * s0, x.y * s1);
  x = unpack_bf16(a[1]); a[1] = pack_bf16(x.x * s0, x.y * s1);
  x = unpack_bf16(a[2]); a[2] = pack_bf16(x.x * s2, x.y * s3);
  x = unpack_bf16(a[3]); a[3] = pack_bf16(x.x * s2, x.y * s3);
}

// One 16x16 block (I, J) of X = [A_i . (B_j * 2^(Gam_i - Gam_j))] with A = Qa or
// Ka rows of block I.  Result in acc[2][4] (two n8 tiles).
__device__ __forceinline__ void block_product(float (&acc)[2][4], const bf16* Arow, const Operands& op,
                                              int I, int J) {
  zero_acc<2>(acc);
  const bool diag = I == J;
  const bf16* Bt = diag ? op.Kd : op.Kb;
  const float* sv = diag ? nullptr : op.cvec + pair_index(I, J) * D;
#pragma unroll 2
  for (int kk = 0; kk < D; kk += 16) {
    uint32_t a[4], b[4];
    load_A(a, Arow, LD128, 16 * I, kk);
    if (!diag) scale_A_frag(a, sv, kk);
    load_B_nk(b, Bt, LD128, 16 * J, kk);
    mma16816(acc[0], a, b[0], b[1]);
    mma16816(acc[1], a, b[2], b[3]);
  }
}

// Computes the strictly-lower L' blocks (and the lower-inclusive M blocks when
// Msm != nullptr) into Lp (fp32 [64][LDF64], upper part zeroed) and Msm (bf16
// [64][LD64], upper part zeroed).  Caller syncs afterwards.
__device__ __forceinline__ void lm_blocks(const Operands& op, float* Lp, bf16* Msm) {
  const int warp = threadIdx.x >> 5;
  const int ntask = Msm ? 20 : 10;
  // zero the strictly-upper blocks
  for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
    int r = i >> 6, c = i & 63;
    if ((c >> 4) > (r >> 4)) {
      Lp[r * LDF64 + c] = 0.f;
      if (Msm) Msm[r * LD64 + c] = __float2bfloat16(0.f);
    }
  }
  for (int task = warp; task < ntask; task += 8) {
    bool isM = task >= 10;
    int bi = isM ? task - 10 : task;
    // block list in order (0,0),(1,0),(1,1),(2,0),(2,1),(2,2),(3,0),...
    int I = bi >= 6 ? 3 : (bi >= 3 ? 2 : (bi >= 1 ? 1 : 0));
    int J = bi - I * (I + 1) / 2;
    float acc[2][4];
    block_product(acc, isM ? op.Qa : op.Ka, op, I, J);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int r = acc_row(e), c = acc_col(j, e);
        int gi = 16 * I + r, gj = 16 * J + c;
        float x = acc[j][e];
        if (isM) {
          if (I == J && c > r) x = 0.f;
          Msm[gi * LD64 + gj] = __float2bfloat16(x);
        } else {
          if (I == J && c >= r) x = 0.f;
          Lp[gi * LDF64 + gj] = x;
        }
      }
  }
}

// A = (I + diag(beta) Lp)^-1 (unit lower triangular, fp32).  Uses xtmp
// ([3][16][16] fp32).  Ends with __syncthreads().
__device__ __forceinline__ void tri_inverse(const float* Lp, const float* beta, float* A, float* xtmp) {
  const int tid = threadIdx.x;
  // zero the strictly-upper blocks of A
  for (int i = tid; i < 64 * 64; i += blockDim.x) {
    int r = i >> 6, c = i & 63;
    if ((c >> 4) > (r >> 4)) A[r * LDF64 + c] = 0.f;
  }
  // diagonal blocks by forward substitution, one column per thread
  if (tid < 64) {
    int blk = tid >> 4, col = tid & 15;
    int o = 16 * blk;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float acc = (r == col) ? 1.f : 0.f;
      if (r > col) {
        float bi = beta[o + r];
        float sum = 0.f;
#pragma unroll
        for (int m = 0; m < 15; ++m)
          if (m < r && m >= col) sum += Lp[(o + r) * LDF64 + o + m] * x[m];
        acc = -bi * sum;
      }
      x[r] = acc;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) A[(o + r) * LDF64 + o + col] = x[r];
  }
  __syncthreads();
  // off-diagonal blocks, by distance I - J
  for (int dist = 1; dist <= 3; ++dist) {
    int npairs = 4 - dist;
    // xtmp_p = sum_{K=J}^{I-1} L_IK A_KJ
    for (int e = tid; e < npairs * 256; e += blockDim.x) {
      int pp = e >> 8, r = (e >> 4) & 15, c = e & 15;
      int J = pp, I = pp + dist;
      float bi = beta[16 * I + r];
      float sum = 0.f;
      for (int K = J; K < I; ++K)
#pragma unroll
        for (int m = 0; m < 16; ++m)
          sum += Lp[(16 * I + r) * LDF64 + 16 * K + m] * A[(16 * K + m) * LDF64 + 16 * J + c];
      xtmp[e] = bi * sum;
    }
    __syncthreads();
    for (int e = tid; e < npairs * 256; e += blockDim.x) {
      int pp = e >> 8, r = (e >> 4) & 15, c = e & 15;
      int J = pp, I = pp + dist;
      float sum = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) sum += A[(16 * I + r) * LDF64 + 16 * I + m] * xtmp[(pp << 8) + m * 16 + c];
      A[(16 * I + r) * LDF64 + 16 * J + c] = -sum;
    }
    __syncthreads();
  }
}

}  // namespace kda
