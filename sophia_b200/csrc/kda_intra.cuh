// Intra-chunk stages of the chunk kernels: the forward's prologue (conv, norms,
// gate, cumsum), its tcgen05 operand build and the UT inverse.
//
// One CTA of 512 threads (16 warps) owns one (chunk, head).  Elementwise work
// uses the "strip" mapping: thread tid owns tokens 2*tg, 2*tg+1 (tg = tid / 16)
// and channels 8*cg .. 8*cg+7 (cg = tid % 16); the 16 threads of a half-warp
// share a token pair, so a row reduction over 128 channels is a 16-lane shuffle.
//
// Overflow-safe factorisations of exp(Gam_i - Gam_j) (per channel, i >= j), with
// r(I) the first and e(J) the last token of a 16-token sub-chunk:
//   * the backward chunk kernel scales its block products in the epilogues:
//       diagonal 16x16 block (I == J):  a_i * ia_j,   a = 2^(Gam - Gam_r(I)) <= 1,
//                                                     ia = 1/a >= 1 (<= 2^116),
//       off-diagonal block (I > J):     a_i * c_IJ * b_j,  c_IJ = 2^(Gam_r(I) - Gam_e(J)),
//                                                     b = 2^(Gam_e(J) - Gam) <= 1;
//   * the forward chunk kernel folds the factors into its operands, one copy
//     of the decayed k per row block (Kc_I, build_tc_operands below).
// Every factor is bounded because the reference clamps the per-token log decay
// to [lb, 0) with lb >= -5 (sixteen tokens span at most 80 nats), and a factor
// that underflows only does so where the exact product is negligible.
#pragma once

#include "kda_common.cuh"
#include "kda_tc.cuh"

namespace kda {

constexpr int INTRA_THREADS = 512;
constexpr int INTRA_WARPS = INTRA_THREADS / 32;
constexpr int STRIP = 2;  // tokens per thread in the strip mapping

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
  float* gam;                    // [64][LDG] log2 cumulative decay
  float* beta;                   // [64]
  float* tot;                    // [16][128] scratch for the cumsum (one row per warp)
  float* taps;                   // [3][128] x 4 conv taps, channel-major 16-byte slots at tap_slot(ch)
  float* bias;                   // [128] dt_bias of the head, then A_log of the head
};

// Slot of channel ch's four taps: the eight channels a strip thread reads
// (8*cg .. 8*cg+7) land in eight different bank quads for any eight
// consecutive cg, so the 128-bit reads are conflict-free.
__device__ __forceinline__ int tap_slot(int ch) { return ch ^ ((ch >> 3) & 7); }

// The last two warps issue the next chunk's loads (the TMA issuer and the 64
// beta gatherers): they are the least loaded warps while the inverse runs.
constexpr int LOADER_T0 = INTRA_THREADS - 64;  // beta of token t0 + i goes to thread LOADER_T0 + i
constexpr int TMA_ISSUER = INTRA_THREADS - 32;

// Issues the loads of one (chunk, head)'s inputs.  One thread starts four
// tiled TMA loads -- the raw q/k/v rows t0-3 .. t0+63 and the gate-logit rows
// t0 .. t0+63 of head h, boxes of `maps` (q, k, v, g: [T_total][H][128] bf16,
// rows outside the tensor arrive as zeros) -- and a bulk copy of the head's
// dt_bias, all completing on `ready` (one arrival with the byte count).  Rows
// of another sequence in the conv halo (tokens bos-3 .. bos-1) are zeroed by
// zero_foreign_halo once `ready` has completed; rows at or past t1 are masked
// by the prologue.  The conv taps (16-byte slots at tap_slot) and A_log go by
// cp.async, which the caller commits.  beta is gathered with a plain load (one
// bf16 per token at a stride of H elements): the value of token t0 + i is
// returned to thread LOADER_T0 + i, which stores it into sm.braw once the
// previous chunk no longer reads it.  The gather is a predicated load into a
// zeroed register, so that nothing waits for it before that store.
constexpr uint32_t PROLOGUE_TMA_BYTES = (3 * 67 + 64) * D * 2 + D * 4;
__device__ __forceinline__ bf16 prologue_issue_loads(const PrologueIn& in, const PrologueSmem& sm,
                                                     const ChunkPos& p, int h, bool conv, uint64_t* ready,
                                                     const CUtensorMap* maps) {
  const int tid = threadIdx.x;
  if (tid == TMA_ISSUER) {
    tc::mbar_expect_tx(ready, PROLOGUE_TMA_BYTES);
    tc::tma_load_3d(sm.xq, maps + 0, 0, h, p.t0 - 3, ready);
    tc::tma_load_3d(sm.xk, maps + 1, 0, h, p.t0 - 3, ready);
    tc::tma_load_3d(sm.xv, maps + 2, 0, h, p.t0 - 3, ready);
    tc::tma_load_3d(sm.graw, maps + 3, 0, h, p.t0, ready);
    tc::bulk_g2s(sm.bias, in.dt_bias + (size_t)h * D, D * 4, ready);
  }
  if (conv) {
    for (int i = tid; i < 3 * D; i += blockDim.x) {
      int X = i >> 7, ch = i & 127;
      const float* src = (X == 0 ? in.conv_q : (X == 1 ? in.conv_k : in.conv_v)) + ((size_t)h * D + ch) * 4;
      cp_async16(sm.taps + (X * D + tap_slot(ch)) * 4, src, true);
    }
  }
  if (tid == 64) cp_async4(sm.bias + D, in.A_log + h);
  unsigned short b = 0;
  if (tid >= LOADER_T0) {
    const int t = p.t0 + (tid - LOADER_T0);
    const bf16* src = in.beta + (t < p.t1 ? (size_t)t * in.H + h : 0);
    asm volatile("{\n.reg .pred p;\nsetp.lt.s32 p, %2, %3;\n@p ld.global.nc.u16 %0, [%1];\n}\n"
                 : "+h"(b) : "l"(src), "r"(t), "r"(p.t1));
  }
  return __ushort_as_bfloat16(b);
}

// Zeroes the conv-halo rows (tokens t0-3 .. t0-1) that precede the sequence
// start: the tiled loads bring the previous sequence's rows there.  Run after
// the loads completed and before the barrier that publishes them.
__device__ __forceinline__ void zero_foreign_halo(const PrologueSmem& sm, const ChunkPos& p) {
  if (p.t0 - 3 >= p.bos) return;
  for (int i = threadIdx.x; i < 3 * 3 * 16; i += blockDim.x) {
    const int X = i / 48, r = (i >> 4) % 3, j = i & 15;
    if (p.t0 - 3 + r < p.bos)
      reinterpret_cast<uint4*>((X == 0 ? sm.xq : (X == 1 ? sm.xk : sm.xv)) + r * D)[j] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// Elementwise prologue, run once the loads of prologue_issue_loads have landed
// and sm.braw is filled (the caller waits and syncs).  On return (after the
// trailing __syncthreads) sm.gam and sm.beta are complete and the calling
// thread holds its strip of the normalised (q scaled) q, k, post-conv v and
// log2 decays.
struct Strip {
  float q[STRIP][8], k[STRIP][8], v[STRIP][8], gam[STRIP][8];
};

// w: this tensor's [128] x 4 taps in shared memory (slots at tap_slot(ch)).
__device__ __forceinline__ void conv_strip(const bf16* x, const float* w, int tg, int cg, bool conv,
                                           float (&out)[STRIP][8]) {
  if (conv) {
    float xs[STRIP + 3][8];
#pragma unroll
    for (int r = 0; r < STRIP + 3; ++r) {
      bf16x8 v = *reinterpret_cast<const bf16x8*>(x + (STRIP * tg + r) * D + 8 * cg);
      unpack8(v, xs[r]);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 t4 = *reinterpret_cast<const float4*>(w + 4 * tap_slot(8 * cg + c));
      const float wt[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
      for (int r = 0; r < STRIP; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int tap = 0; tap < 4; ++tap) acc = fmaf(wt[tap], xs[r + tap][c], acc);
        out[r][c] = acc;
      }
    }
#pragma unroll
    for (int r = 0; r < STRIP; ++r)
#pragma unroll
      for (int c = 0; c < 8; ++c) out[r][c] = silu_fast(out[r][c]);
  } else {
#pragma unroll
    for (int r = 0; r < STRIP; ++r) {
      bf16x8 v = *reinterpret_cast<const bf16x8*>(x + (3 + STRIP * tg + r) * D + 8 * cg);
      unpack8(v, out[r]);
    }
  }
}

__device__ __forceinline__ void prologue_compute(const PrologueIn& in, const PrologueSmem& sm,
                                                 const ChunkPos& p, bool conv, Strip& s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tg = tid >> 4, cg = tid & 15;
  const int nvalid = p.t1 - p.t0;
  const float* wq = sm.taps;
  const float* wk = sm.taps + 4 * D;
  const float* wv = sm.taps + 8 * D;
  conv_strip(sm.xq, wq, tg, cg, conv, s.q);
  conv_strip(sm.xk, wk, tg, cg, conv, s.k);
  conv_strip(sm.xv, wv, tg, cg, conv, s.v);
  // mask padded tokens, L2 normalise q and k per token (reduction over 16 lanes)
#pragma unroll
  for (int r = 0; r < STRIP; ++r) {
    bool ok = STRIP * tg + r < nvalid;
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
  const float eA = __expf(sm.bias[D]);
  float bias[8];
  {
    float4 b0 = *reinterpret_cast<const float4*>(sm.bias + 8 * cg);
    float4 b1 = *reinterpret_cast<const float4*>(sm.bias + 8 * cg + 4);
    bias[0] = b0.x; bias[1] = b0.y; bias[2] = b0.z; bias[3] = b0.w;
    bias[4] = b1.x; bias[5] = b1.y; bias[6] = b1.z; bias[7] = b1.w;
  }
  float run[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) run[c] = 0.f;
#pragma unroll
  for (int r = 0; r < STRIP; ++r) {
    float gx[8];
    unpack8(*reinterpret_cast<const bf16x8*>(sm.graw + (STRIP * tg + r) * D + 8 * cg), gx);
    bool ok = STRIP * tg + r < nvalid;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float z = eA * (gx[c] + bias[c]);
      float gv = ok ? in.lower_bound * sigmoidf_(z) * LOG2E : 0.f;
      run[c] += gv;
      s.gam[r][c] = run[c];
    }
  }
  // token-pair totals: the odd half-warp adds the even half-warp's, the warp
  // total (4 tokens) goes to tot[warp]
  float inw[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float up = __shfl_up_sync(0xffffffffu, run[c], 16);
    inw[c] = lane >= 16 ? up : 0.f;
  }
  if (lane >= 16) {
    float* tp = sm.tot + warp * D + 8 * cg;
    *reinterpret_cast<float4*>(tp) = make_float4(inw[0] + run[0], inw[1] + run[1], inw[2] + run[2], inw[3] + run[3]);
    *reinterpret_cast<float4*>(tp + 4) = make_float4(inw[4] + run[4], inw[5] + run[5], inw[6] + run[6], inw[7] + run[7]);
  }
  if (tid < 64) {
    float b = __bfloat162float(sm.braw[tid]);
    sm.beta[tid] = (tid < nvalid) ? sigmoidf_(b) : 0.f;
  }
  __syncthreads();
  // exclusive prefix of the 16 warp totals, per channel, in place: warp w
  // takes channels 8w .. 8w+7, four lanes per channel, four totals per lane,
  // then a two-step shuffle scan over the four lanes
  static_assert(INTRA_WARPS == 16 && INTRA_THREADS == 4 * D, "prefix layout");
  {
    const int ch = 8 * warp + (lane >> 2), part = lane & 3;
    float* col = sm.tot + 4 * part * D + ch;
    const float v0 = col[0], v1 = col[D], v2 = col[2 * D], v3 = col[3 * D];
    const float own = (v0 + v1) + (v2 + v3);
    float incl = own;
    float y = __shfl_up_sync(0xffffffffu, incl, 1);
    if (part >= 1) incl += y;
    y = __shfl_up_sync(0xffffffffu, incl, 2);
    if (part >= 2) incl += y;
    float ex = __shfl_up_sync(0xffffffffu, incl, 1);
    if (part == 0) ex = 0.f;
    col[0] = ex;
    col[D] = ex + v0;
    col[2 * D] = (ex + v0) + v1;
    col[3 * D] = ((ex + v0) + v1) + v2;
  }
  __syncthreads();
  float off[8];
  {
    float4 a = *reinterpret_cast<const float4*>(sm.tot + warp * D + 8 * cg);
    float4 b = *reinterpret_cast<const float4*>(sm.tot + warp * D + 8 * cg + 4);
    off[0] = inw[0] + a.x; off[1] = inw[1] + a.y; off[2] = inw[2] + a.z; off[3] = inw[3] + a.w;
    off[4] = inw[4] + b.x; off[5] = inw[5] + b.y; off[6] = inw[6] + b.z; off[7] = inw[7] + b.w;
  }
#pragma unroll
  for (int r = 0; r < STRIP; ++r) {
#pragma unroll
    for (int c = 0; c < 8; ++c) s.gam[r][c] += off[c];
    float* gp = sm.gam + (STRIP * tg + r) * LDG + 8 * cg;
    *reinterpret_cast<float4*>(gp) = make_float4(s.gam[r][0], s.gam[r][1], s.gam[r][2], s.gam[r][3]);
    *reinterpret_cast<float4*>(gp + 4) = make_float4(s.gam[r][4], s.gam[r][5], s.gam[r][6], s.gam[r][7]);
  }
  __syncthreads();
}

// Sub-chunk pair index p = I (I - 1) / 2 + J of an off-diagonal pair J < I
// (pairs (1,0), (2,0), (2,1), (3,0), (3,1), (3,2)).
__device__ __forceinline__ int pair_index(int I, int J) { return I * (I - 1) / 2 + J; }

// Byte offset of the 16-byte chunk c8 (columns 8 c8 .. 8 c8 + 7) of row r in a
// 128B-swizzled bf16 tile of `rows` rows: 64-column atoms of rows x 128 bytes
// one after the other, chunk position c8 ^ (r & 7) inside a row (the tcgen05
// operand layout of kda_tc.cuh; every atom starts on a 1 KB boundary).
__device__ __forceinline__ uint32_t sw_rows_byte(int rows, int r, int c8) {
  return (uint32_t)((c8 >> 3) * rows * 128 + r * 128 + (((c8 & 7) ^ (r & 7)) << 4));
}

// The forward's tcgen05 block products of L' and M.  With a = 2^(Gam - Gam_r(J))
// (J the token's own sub-chunk, r(J) its first token) and, per row block I,
//   Kc_I[j] = k_j 2^(Gam_r(I) - Gam_j)   for the tokens j < 16 (I + 1),
// every entry of row block I is one dot product over the 128 channels:
//   L'[i, j] = Ka_i . Kc_I[j],   M[i, j] = Qa_i . Kc_I[j]   (Ka = k a, Qa = q a),
// so with the four Kc_I stacked as the rows of one B operand (N = 160), every
// block is one M = 128 MMA chain ([Ka; Qa] against [Kc_0; ..; Kc_3]); row
// block I reads the 16 (I + 1) columns of Kc_I and the epilogue masks them to
// the strictly lower (L') or lower (M) part.  Bounds: a <= 1; for j in I the
// factor of Kc_I is 2^(Gam_r(I) - Gam_j) <= 2^108 (15 tokens of log2 decay
// >= -7.22 each); for j < r(I) it is at most 1 and is formed as
// (k_j 2^(Gam_r(J) - Gam_j)) 2^(Gam_r(I) - Gam_r(J)), a factor in [1, 2^108]
// times one in (0, 1]: the second flushes to zero only below 2^-126, where the
// exact product is below 2^-18 -- negligible against the bf16 operands.
//
// Tiles of the operand region (128B-swizzled bf16, K-major over the channels
// unless noted; every atom 1 KB aligned):
//   KQ  [Ka; Qa]: 128 rows;
//   KC  [Kc_0; Kc_1; Kc_2; Kc_3]: 160 rows, Kc_I from row kc_row(I) = 8 I (I + 1);
//   KE  Ke = k 2^Gam, then V: 64 rows each (the MN-major B operands of
//       W = T Ke and U = T V).
__host__ __device__ constexpr int kc_row(int I) { return 8 * I * (I + 1); }
constexpr int KC_ROWS = 160;             // kc_row(4)
constexpr int KC_BYTES = KC_ROWS * 256;  // two 64-channel atoms

// Builds KQ, KC and KE/V from the strip (shared-memory writes only; the caller
// fences and syncs) and stores the strip of q 2^Gam and k 2^(Gam_C - Gam) (the
// forward's Qt and Kbar, rows t0 .. t0 + nvalid - 1 of head h) to global memory.
__device__ __forceinline__ void build_tc_operands(const Strip& s, const float* gam, unsigned char* kq,
                                                  unsigned char* kc, unsigned char* kev, bf16* Qt, bf16* Kb,
                                                  int t0, int nvalid, int H, int h) {
  const int tid = threadIdx.x;
  const int tg = tid >> 4, cg = tid & 15;
  const int J = (STRIP * tg) >> 4;  // warp-uniform (a warp holds tokens 4w .. 4w + 3)
  const float* gch = gam + 8 * cg;
  float Gr[8], kd[STRIP][8];
  {
    float erv[8], gC[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      Gr[c] = gch[(16 * J) * LDG + c];
      erv[c] = ex2(Gr[c]);
      gC[c] = gch[63 * LDG + c];
    }
#pragma unroll
    for (int r = 0; r < STRIP; ++r) {
      const int t = STRIP * tg + r;
      float qa[8], ka[8], ke[8], qt[8], kbar[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float G = s.gam[r][c];
        const float a = ex2(G - Gr[c]);
        const float ia = ex2(Gr[c] - G);
        qa[c] = s.q[r][c] * a;
        ka[c] = s.k[r][c] * a;
        kd[r][c] = s.k[r][c] * ia;
        ke[c] = ka[c] * erv[c];
        qt[c] = qa[c] * erv[c];
        kbar[c] = s.k[r][c] * ex2(gC[c] - G);  // 2^(Gam_C - Gam) <= 1
      }
      *reinterpret_cast<bf16x8*>(kq + sw_rows_byte(128, t, cg)) = pack8(ka);
      *reinterpret_cast<bf16x8*>(kq + sw_rows_byte(128, 64 + t, cg)) = pack8(qa);
      *reinterpret_cast<bf16x8*>(kev + sw_rows_byte(64, t, cg)) = pack8(ke);
      *reinterpret_cast<bf16x8*>(kev + 16384 + sw_rows_byte(64, t, cg)) = pack8(s.v[r]);
      *reinterpret_cast<bf16x8*>(kc + sw_rows_byte(KC_ROWS, kc_row(J) + t, cg)) = pack8(kd[r]);
      if (t < nvalid) {
        const size_t off = ((size_t)(t0 + t) * H + h) * D + 8 * cg;
        *reinterpret_cast<bf16x8*>(Qt + off) = pack8(qt);
        *reinterpret_cast<bf16x8*>(Kb + off) = pack8(kbar);
      }
    }
  }
  // the later row blocks' copies: Kc_I = kd 2^(Gam_r(I) - Gam_r(J)), I > J
#pragma unroll
  for (int d = 1; d < 4; ++d) {
    const int I = J + d;
    if (I < 4) {
      float cp[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) cp[c] = ex2(gch[(16 * I) * LDG + c] - Gr[c]);
#pragma unroll
      for (int r = 0; r < STRIP; ++r) {
        float x[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) x[c] = kd[r][c] * cp[c];
        *reinterpret_cast<bf16x8*>(kc + sw_rows_byte(KC_ROWS, kc_row(I) + STRIP * tg + r, cg)) = pack8(x);
      }
    }
  }
}

// A = (I + diag(beta) Lp)^-1 (unit lower triangular, fp32; only the lower
// 16x16 blocks are written): tri_inverse_diag (forward substitution in fp32,
// one column per thread) for the diagonal blocks, then tri_inverse_offdiag
// (16x16x16 tensor-core products, tf32 in, fp32 accumulate) for the rest.
__device__ __forceinline__ void warp_tf32_16x16(float (&acc)[2][4], const float* Am, int lda, const float* rowscale,
                                                const float* Bm, int ldb) {
  // acc[16 x 16] += diag(rowscale) Am[16 x 16] * Bm[16 x 16] (row-major fp32 tiles)
  const int l = threadIdx.x & 31, g = l >> 2, t = l & 3;
  const float s0 = rowscale ? rowscale[g] : 1.f, s1 = rowscale ? rowscale[g + 8] : 1.f;
#pragma unroll
  for (int k0 = 0; k0 < 16; k0 += 8) {
    uint32_t a[4];
    a[0] = to_tf32(s0 * Am[g * lda + k0 + t]);
    a[1] = to_tf32(s1 * Am[(g + 8) * lda + k0 + t]);
    a[2] = to_tf32(s0 * Am[g * lda + k0 + t + 4]);
    a[3] = to_tf32(s1 * Am[(g + 8) * lda + k0 + t + 4]);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      uint32_t b0 = to_tf32(Bm[(k0 + t) * ldb + 8 * n + g]);
      uint32_t b1 = to_tf32(Bm[(k0 + t + 4) * ldb + 8 * n + g]);
      mma1688_tf32(acc[n], a, b0, b1);
    }
  }
}

// Diagonal 16x16 blocks of A, threads 0..63 (one column each); no sync.
// Column-oriented forward substitution: once x_m is final it updates every
// later row, x_r -= beta_r L'_rm x_m, so each step is 15 - m independent FMAs
// and the dependent chain is one FMA per step (rows above the column stay 0).
__device__ __forceinline__ void tri_inverse_diag(const float* Lp, const float* beta, float* A) {
  const int tid = threadIdx.x;
  // (strictly-upper blocks of A are never written; readers mask them)
  if (tid < 64) {
    const int blk = tid >> 4, col = tid & 15;
    const int o = 16 * blk;
    float x[16], nb[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      x[r] = (r == col) ? 1.f : 0.f;
      nb[r] = -beta[o + r];
    }
#pragma unroll
    for (int m = 0; m < 15; ++m) {
#pragma unroll
      for (int r = m + 1; r < 16; ++r) x[r] = fmaf(nb[r] * Lp[(o + r) * LDF64 + o + m], x[m], x[r]);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) A[(o + r) * LDF64 + o + col] = x[r];
  }
}

// Off-diagonal blocks of A by distance (the diagonal blocks must be complete
// and visible).  Ends with __syncthreads().
__device__ __forceinline__ void tri_inverse_offdiag(const float* Lp, const float* beta, float* A, float* xtmp) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  (void)tid;
  float* xs = xtmp + warp * 16 * 17;
  const int g = lane >> 2, t = lane & 3;
  for (int dist = 1; dist <= 3; ++dist) {
    if (warp < 4 - dist) {
      const int J = warp, I = warp + dist;
      float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int K = J; K < I; ++K)
        warp_tf32_16x16(acc, Lp + (16 * I) * LDF64 + 16 * K, LDF64, beta + 16 * I,
                        A + (16 * K) * LDF64 + 16 * J, LDF64);
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        xs[g * 17 + 8 * n + 2 * t] = acc[n][0];
        xs[g * 17 + 8 * n + 2 * t + 1] = acc[n][1];
        xs[(g + 8) * 17 + 8 * n + 2 * t] = acc[n][2];
        xs[(g + 8) * 17 + 8 * n + 2 * t + 1] = acc[n][3];
      }
      __syncwarp();
      float out[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      warp_tf32_16x16(out, A + (16 * I) * LDF64 + 16 * I, LDF64, nullptr, xs, 17);
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        float* dst = A + (16 * I + g) * LDF64 + 16 * J + 8 * n + 2 * t;
        dst[0] = -out[n][0];
        dst[1] = -out[n][1];
        dst[8 * LDF64] = -out[n][2];
        dst[8 * LDF64 + 1] = -out[n][3];
      }
    }
    __syncthreads();
  }
}


}  // namespace kda
