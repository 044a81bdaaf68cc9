// Chunk-parallel backward of the chunked KDA layer on the fifth-generation
// tensor cores (tcgen05 + TMEM).
//
// One CTA of 512 threads per (chunk, head).  The forward's saved products --
// normalised q and k, post-conv v (bf16, in the 128B-swizzled operand layout),
// the decay cumsum, beta, and A = (I + diag(beta) L')^-1 and L' as bf16
// operand tiles -- arrive by bulk copies, and so do the state pass's gradient
// tiles dE, dW and dM (stored in the swizzled operand layout).  With T =
// A diag(beta) and the decayed operands Qa = q a, Ka = k a, Kd = k / a,
// Ke = k 2^Gam built in shared memory, every block product is a tcgen05 MMA
// with M = 64 (a 64 x 128 result is two N = 64 halves at TMEM lane offsets
// 0 and 16, sharing 64 columns):
//   G1  dv = T^T dE,  dKe = T^T dW,  dT = dE V^T + dW Ke^T
//   G2  P_J = dM[:, J] Kd[J]          (row side of the gradient through M, J = 0..3)
//   G3  X = dA A^T                    (dA = dT diag(beta))
//   G4  R_I = dM[I, :]^T Qa[I]        (column side through M)
//   G5  -dL = A^T X                   (then dL' = diag(beta) tril(dL))
//   G6  P_J = dL'[:, J] Kd[J]         (row side through L')
//   G7  R_I = dL'[I, :]^T Ka[I]       (column side through L')
// One thread issues each group and commits it to its own mbarrier.  The
// epilogues on the chain G1 -> dA -> G3 -> X -> G5 -> dL' -> G6/G7 run first;
// the others (dv and dKe, the row and column sides through M) run while the
// chain's MMAs compute.  TMEM holds 512 columns in eight 64-column units: G1 in
// units 0-2, X in 3, dL in 0, the row side of L' in 0-3, the row side of M and
// both column sides in 4-7.  Accumulator slices a phase needs are loaded
// together and waited for once.
//
// Epilogues run in the TMEM row layout: warp w reads lane quarter w % 4 (rows
// 16 (w % 4) .. +15 = sub-chunk block I), lanes 0-15 the first half of the
// columns and lanes 16-31 the second, 16 columns per thread.  Each thread
// keeps its 16 elements of dq, dk, dGam and of the decay factor
//   af = 2^(Gam - Gam_r(I)) <= 1   (and bf = 2^(Gam_e(I) - Gam) = rev_I / af <= 1,
//                                   rev_I = 2^(Gam_e(I) - Gam_r(I)))
// in registers for the whole kernel.  The sub-chunk factorisation is that of
// the chunk kernels (kda_intra.cuh): the row side scales P_J (J < I) by
// 2^(Gam_r(I) - Gam_r(J)) and then by af, the column side scales R_Ib (Ib > I)
// by 2^(Gam_r(Ib) - Gam_e(I)) and then by bf, the diagonal blocks by af and
// 1/af; every factor is bounded, and one that underflows only does so where
// the exact product is negligible.
// Per element then:
//   dq  = dQt 2^Gam + af (row side through M)
//   dk  = dKe 2^Gam + dKbar 2^(Gam_C - Gam) + af (row side through L')
//         + 1/af (diagonal) + bf (off-diagonal column sides)
//   dGam collects q o dq - k o dk terms; dg = reverse cumsum of dGam inside
//   the chunk; the gate and beta sigmoids are differentiated last.
// Outputs: dq_hat, dk_hat (gradients of the normalised, scaled q and of the
// normalised k; the L2-norm and conv backward run in the post kernel), dv,
// dg_logits, dbeta_logits and per-chunk partial sums for dA_log and dt_bias.
// Every wait is bounded; on a timeout the CTA records an error, lets its
// copies and MMAs in flight finish (bounded), frees TMEM and leaves.
#pragma once

#include "kda_fwd.cuh"
#include "kda_tc.cuh"

namespace kda {

struct BwdIntraParams {
  PrologueIn in;
  SeqInfo seq;
  bool conv;
  const bf16 *dE, *dW, *dM;              // [chunks][H] 128B-swizzled operand tiles (dM: 64 x 64)
  const bf16 *dQt, *dKb;                 // [chunks][H] acc64 tiles
  const bf16 *A, *LP;                    // [chunks][H] bf16 64x64 swizzled tiles of A and L' from the forward
  const bf16 *QN, *KN, *VN;              // [chunks][H] bf16 64x128 swizzled prologue products of the forward
  const float *GM, *BT;                  // [chunks][H] [64][LDG] fp32 decay cumsum, [64] fp32 beta
  const float* dGC;
  bf16 *dq_hat, *dk_hat, *dv;  // [T_total][H][128]
  bf16 *dg, *dbeta;            // [T_total][H][128], [T_total][H]
  float *partA, *partB;        // [chunks][H][128]
};

struct BwdIntraSmem {
  static constexpr int T128 = 16384, T64 = 8192;  // swizzled bf16 tiles of 64 x 128 / 64 x 64
  static constexpr int QA = 0, KA = QA + T128, KD = KA + T128, KE = KD + T128, V = KE + T128;
  static constexpr int DE = V + T128, DW = DE + T128;
  static constexpr int QN = DW + T128, KN = QN + T128;
  static constexpr int AT = KN + T128, LPT = AT + T64, DM = LPT + T64, TT = DM + T64;
  static constexpr int GAM = TT + T64;  // 64 x LDG fp32; then the dQt | dKbar acc64 tiles; then dGam
  static constexpr int VEC = GAM + 64 * LDG * 4;
  static constexpr int CP = VEC;                    // [6][128] 2^(Gam_r(I) - Gam_r(J)), pair I(I-1)/2 + J
  static constexpr int CC = CP + 6 * D * 4;         // [6][128] 2^(Gam_r(I) - Gam_e(J))
  static constexpr int ER = CC + 6 * D * 4;         // [4][128] 2^Gam_r(J)
  static constexpr int EC = ER + 4 * D * 4;         // [4][128] 2^(Gam_C - Gam_e(J))
  static constexpr int REV = EC + 4 * D * 4;        // [4][128] 2^(Gam_e(J) - Gam_r(J))
  static constexpr int BETA = REV + 4 * D * 4;      // [64] fp32
  static constexpr int MISC = BETA + 64 * 4;        // 11 mbarriers, TMEM slot, issued mask
  static constexpr int END = MISC + 128;
  // aliases (regions dead by then)
  static constexpr int DA = QN, XS = QN + T64;      // dA, X tiles (after the operand build)
  static constexpr int DLP = KN;                    // dL' tile
  static constexpr int DBT = KN + T64;              // fp32 [4][64] dbeta from T
  static constexpr int DBL = DBT + 1024;            // fp32 [4][64] dbeta from L'
  static constexpr int COLS = DBL + 1024;           // fp32 [4][128] column sums of Kbar o dKbar
  static constexpr int GRE = DE;                    // bf16 [64][128] gate logits (after G1)
  static constexpr int GBV = DW;                    // fp32 dGam_C [128], dt_bias [128], A_log (after G1)
  static constexpr int PSUM = DW + 2048;            // fp32 [8][128] partial sums of the gate tail
  static constexpr int DQT = GAM, DKB = GAM + T128; // acc64 state-pass tiles (after the decay factors)
  static constexpr int DGAM = KE;                   // fp32 [64][128] dGam over Ke and V (after G1)
  static_assert(V == KE + T128, "dGam needs Ke and V adjacent");
  static_assert(COLS + 4 * D * 4 <= KN + T128, "small arrays overflow the dL' region");
  static_assert(PSUM + 8 * D * 4 <= DW + T128 && GBV + (2 * D + 4) * 4 <= PSUM, "gate-tail arrays overflow");
  static_assert(DKB + T128 <= VEC, "gradient tiles overflow the decay region");
  static_assert(END <= 232448, "shared memory");
  static_assert(GAM % 1024 == 0 && MISC % 8 == 0, "alignment");
};

// Bytes of the products arriving by bulk copy at the start.
constexpr uint32_t BWD_DECAY_BYTES = 64 * LDG * 4 + 64 * 4;                      // Gam, beta
constexpr uint32_t BWD_TILE_BYTES = 3 * BwdIntraSmem::T128 + 2 * BwdIntraSmem::T64;  // q, k, v, A, L'

__device__ __forceinline__ uint4 lds_chunk(const unsigned char* tile, int r, int c8) {
  return *reinterpret_cast<const uint4*>(tile + 2 * sw64_chunk(r, c8));
}
__device__ __forceinline__ void unpack16(const uint4& a, const uint4& b, float (&f)[16]) {
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 p = unpack_bf16(w[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}
// 16 consecutive columns of row r of a swizzled tile (two 16-byte chunks).
__device__ __forceinline__ void lds_row16(const unsigned char* tile, int r, int col0, float (&f)[16]) {
  unpack16(lds_chunk(tile, r, col0 >> 3), lds_chunk(tile, r, (col0 >> 3) + 1), f);
}
__device__ __forceinline__ void pack16(const float (&f)[16], uint4& a, uint4& b) {
  a.x = pack_bf16(f[0], f[1]); a.y = pack_bf16(f[2], f[3]); a.z = pack_bf16(f[4], f[5]); a.w = pack_bf16(f[6], f[7]);
  b.x = pack_bf16(f[8], f[9]); b.y = pack_bf16(f[10], f[11]); b.z = pack_bf16(f[12], f[13]);
  b.w = pack_bf16(f[14], f[15]);
}
__device__ __forceinline__ void sts_row16(unsigned char* tile, int r, int col0, const float (&f)[16]) {
  uint4 a, b;
  pack16(f, a, b);
  *reinterpret_cast<uint4*>(tile + 2 * sw64_chunk(r, col0 >> 3)) = a;
  *reinterpret_cast<uint4*>(tile + 2 * sw64_chunk(r, (col0 >> 3) + 1)) = b;
}
// 16 consecutive columns of row r of an acc64 tile (two 16-byte chunks).
__device__ __forceinline__ void lds_acc64_16(const bf16* tile, int r, int col0, float (&f)[16]) {
  unpack16(*reinterpret_cast<const uint4*>(tile + acc64_off(r, col0)),
           *reinterpret_cast<const uint4*>(tile + acc64_off(r, col0 + 8)), f);
}
__device__ __forceinline__ void ld_vec16(const float* v, float (&f)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 x = *reinterpret_cast<const float4*>(v + i);
    f[i] = x.x; f[i + 1] = x.y; f[i + 2] = x.z; f[i + 3] = x.w;
  }
}
__device__ __forceinline__ void st_global16(bf16* dst, const float (&f)[16]) {
  uint4 a, b;
  pack16(f, a, b);
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = b;
}
// Column sums over the 16 lanes of this lane half (the rows of one sub-chunk
// block): lane L of the half returns sum over the half's lanes of v[L].
// Recursive halving, 8 + 4 + 2 + 1 shuffles.
__device__ __forceinline__ float half_reduce_scatter(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 8, n = 8; m >= 1; m >>= 1, n >>= 1) {
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[i + n];
      const float keep = up ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
  return v[0];
}
// The same for 8 values: lanes L and L ^ 1 of the half both return the column
// sum of v[(L & 15) >> 1].
__device__ __forceinline__ float half_reduce_scatter8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int m = 8, n = 4; m >= 2; m >>= 1, n >>= 1) {
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < n; ++i) {
      const float send = up ? v[i] : v[i + n];
      const float keep = up ? v[i + n] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// 8 consecutive floats of a 16-byte-aligned shared vector (two LDS.128).
__device__ __forceinline__ void ld8f(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// dGam as fp32 [64][128] over the dead V and Ke tiles: 16-byte chunk k of row
// r at position k ^ (r & 7), so the 16 rows a warp half touches hit distinct banks.
__device__ __forceinline__ float4* dg_chunk(unsigned char* base, int r, int col) {
  return reinterpret_cast<float4*>(base + r * 512 + ((((col >> 2) ^ (r & 7))) << 4));
}
__device__ __forceinline__ void ld_dg16(unsigned char* base, int r, int col0, float (&f)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4) {
    const float4 x = *dg_chunk(base, r, col0 + i);
    f[i] = x.x; f[i + 1] = x.y; f[i + 2] = x.z; f[i + 3] = x.w;
  }
}
__device__ __forceinline__ void st_dg16(unsigned char* base, int r, int col0, const float (&f)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i += 4) *dg_chunk(base, r, col0 + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
}
__device__ __forceinline__ void st_dg8(unsigned char* base, int r, int col0, const float (&f)[8]) {
  *dg_chunk(base, r, col0) = make_float4(f[0], f[1], f[2], f[3]);
  *dg_chunk(base, r, col0 + 4) = make_float4(f[4], f[5], f[6], f[7]);
}

__global__ void __launch_bounds__(INTRA_THREADS, 1) kda_bwd_intra_kernel(BwdIntraParams P) {
  extern __shared__ __align__(1024) unsigned char bwi_smem[];  // 1 KB-aligned dynamic shared memory
  unsigned char* smem = bwi_smem;
  using S = BwdIntraSmem;
  const int c = blockIdx.x, h = blockIdx.y;
  const ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int H = P.in.H;
  const int nv = pos.t1 - pos.t0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t cidx = (size_t)c * H + h;
  const size_t tix = tile_index(P.seq, c, h);
  // mbarriers: 0 decay cumsum and beta, 1 dQt/dKbar, 2..8 MMA groups G1..G7, 9 product tiles
  uint64_t* mb = reinterpret_cast<uint64_t*>(smem + S::MISC);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mb + 11);
  volatile uint32_t* issued = tslot + 1;  // bit i: mbarrier i has work in flight
  float* gam = reinterpret_cast<float*>(smem + S::GAM);
  float* beta = reinterpret_cast<float*>(smem + S::BETA);
  if (smem_u32(smem) & 1023) {  // swizzled tiles need 1 KB alignment (block-uniform)
    if (tid == 0) atomicExch(&g_kda_device_error, 9);
    return;
  }
  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < 11; ++i) tc::mbar_init(mb + i, 1);
    tc::fence_mbar_init();
    *issued = 0u;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  if (tid == 0) {
    constexpr uint32_t TB = S::T128, GB = 64 * LDG * 4, BB = 64 * 4, AB = S::T64;
    // the decay cumsum first: the channel vectors and decay factors need only it
    tc::mbar_expect_tx(mb + 0, BWD_DECAY_BYTES);
    tc::bulk_g2s(gam, P.GM + tix * 64 * LDG, GB, mb + 0);
    tc::bulk_g2s(beta, P.BT + tix * 64, BB, mb + 0);
    tc::mbar_expect_tx(mb + 9, BWD_TILE_BYTES);
    tc::bulk_g2s(smem + S::QN, P.QN + tix * TILE64_ELEMS, TB, mb + 9);
    tc::bulk_g2s(smem + S::KN, P.KN + tix * TILE64_ELEMS, TB, mb + 9);
    tc::bulk_g2s(smem + S::V, P.VN + tix * TILE64_ELEMS, TB, mb + 9);
    tc::bulk_g2s(smem + S::AT, P.A + tix * TILE64N64_ELEMS, AB, mb + 9);
    tc::bulk_g2s(smem + S::LPT, P.LP + tix * TILE64N64_ELEMS, AB, mb + 9);
    // the state pass's gradient tiles dE, dW, dM, stored in the swizzled operand layout
    tc::mbar_expect_tx(mb + 10, 2 * TB + AB);
    tc::bulk_g2s(smem + S::DE, P.dE + tix * TILE64_ELEMS, TB, mb + 10);
    tc::bulk_g2s(smem + S::DW, P.dW + tix * TILE64_ELEMS, TB, mb + 10);
    tc::bulk_g2s(smem + S::DM, P.dM + tix * TILE64N64_ELEMS, AB, mb + 10);
    *issued = 0x601u;
  }

  // epilogue mapping: rows 16 s .. 16 s + 15 (block I = s), 16 columns from c0
  const int s = warp & 3, qd = warp >> 2, hh = lane >> 4;
  const int r = 16 * s + (lane & 15);
  const int c0 = 64 * hh + 16 * qd;
  const uint32_t trow = tbase + ((uint32_t)(32 * s) << 16);
  const uint32_t idMM = tc::idesc_bf16(64, 64, true, true);    // A MN-major, B MN-major
  const uint32_t idKM = tc::idesc_bf16(64, 64, false, true);   // A K-major,  B MN-major
  const uint32_t idKK = tc::idesc_bf16(64, 64, false, false);  // A K-major,  B K-major
  const uint32_t sb = smem_u32(smem);
  // Descriptors: the address field (bits 0-13, address / 16) of a base descriptor
  // plus the operand's offset / 16 (every address stays below 256 KB).
  const uint64_t kbase = tc::smem_desc(sb, 16, 1024), mbase = tc::smem_desc(sb, 8192, 1024);
  // K-major operand at byte offset `off`: K step ks (16 elements) of a tile of 64-element atoms
  auto kdesc = [&](int off, int ks) { return kbase + (uint64_t)((off + (ks >> 2) * 8192 + (ks & 3) * 32) >> 4); };
  // MN-major operand: K step ks (16 rows)
  auto mdesc = [&](int off, int ks) { return mbase + (uint64_t)((off + ks * 2048) >> 4); };

  // dq, dk and the decay factor stay in registers; dGam lives in shared memory
  // over the V and Ke tiles once G1 has read them (each thread owns its 16
  // elements there: no synchronisation needed).
  float dq[16], dk[16], af[16];
  unsigned char* dgb = smem + S::DGAM;
  bool ok = true;
  for (int once = 0; once < 1; ++once) {
    ok = tc::mbar_wait(mb + 0, 0);
    if (__syncthreads_or(!ok)) { ok = false; if (tid == 0) atomicExch(&g_kda_device_error, 7); break; }

    // ---- from the decay cumsum alone (the product tiles are still arriving)
    {
      // per-pair and per-sub-chunk channel vectors
      float* cpv = reinterpret_cast<float*>(smem + S::CP);
      float* ccv = reinterpret_cast<float*>(smem + S::CC);
      for (int i = tid; i < 6 * D; i += blockDim.x) {
        const int p = i / D, d = i - p * D;
        const int I = p >= 3 ? 3 : (p >= 1 ? 2 : 1);
        const int Jp = p - pair_index(I, 0);
        cpv[i] = ex2(gam[(16 * I) * LDG + d] - gam[(16 * Jp) * LDG + d]);
        ccv[i] = ex2(gam[(16 * I) * LDG + d] - gam[(16 * Jp + 15) * LDG + d]);
      }
      {
        float* erw = reinterpret_cast<float*>(smem + S::ER);
        float* ecw = reinterpret_cast<float*>(smem + S::EC);
        float* rvw = reinterpret_cast<float*>(smem + S::REV);
        const int Jp = tid >> 7, d = tid & 127;
        const float gr = gam[(16 * Jp) * LDG + d], ge = gam[(16 * Jp + 15) * LDG + d];
        erw[tid] = ex2(gr);
        ecw[tid] = ex2(gam[63 * LDG + d] - ge);
        rvw[tid] = ex2(ge - gr);
      }
      // the decay factor of this thread's epilogue elements
#pragma unroll
      for (int u = 0; u < 16; u += 4) {
        const float4 g = *reinterpret_cast<const float4*>(gam + r * LDG + c0 + u);
        const float4 g0 = *reinterpret_cast<const float4*>(gam + (16 * s) * LDG + c0 + u);
        af[u] = ex2(g.x - g0.x);
        af[u + 1] = ex2(g.y - g0.y);
        af[u + 2] = ex2(g.z - g0.z);
        af[u + 3] = ex2(g.w - g0.w);
      }
    }
    ok = tc::mbar_wait(mb + 9, 0);
    if (__syncthreads_or(!ok)) { ok = false; if (tid == 0) atomicExch(&g_kda_device_error, 7); break; }

    // ---- operands (strip mapping: tokens 2 tg, 2 tg + 1, channels 8 cg .. +7)
    {
      const int tg = tid >> 4, cg = tid & 15;
      const int J = (STRIP * tg) >> 4;
      float Gr[8], erv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        Gr[u] = gam[(16 * J) * LDG + 8 * cg + u];
        erv[u] = ex2(Gr[u]);
      }
#pragma unroll
      for (int rr = 0; rr < STRIP; ++rr) {
        const int t = STRIP * tg + rr;
        float qv[8], kv[8], qa[8], ka[8], kd[8], ke[8];
        {
          const uint4 qx = lds_chunk(smem + S::QN, t, cg), kx = lds_chunk(smem + S::KN, t, cg);
          const uint32_t qw[4] = {qx.x, qx.y, qx.z, qx.w}, kw[4] = {kx.x, kx.y, kx.z, kx.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = unpack_bf16(qw[i]), b = unpack_bf16(kw[i]);
            qv[2 * i] = a.x; qv[2 * i + 1] = a.y; kv[2 * i] = b.x; kv[2 * i + 1] = b.y;
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float G = gam[t * LDG + 8 * cg + u];
          const float a = ex2(G - Gr[u]), ia = ex2(Gr[u] - G);
          qa[u] = qv[u] * a;
          ka[u] = kv[u] * a;
          kd[u] = kv[u] * ia;
          ke[u] = ka[u] * erv[u];
        }
        const uint32_t so = 2 * sw64_chunk(t, cg);
        *reinterpret_cast<bf16x8*>(smem + S::QA + so) = pack8(qa);
        *reinterpret_cast<bf16x8*>(smem + S::KA + so) = pack8(ka);
        *reinterpret_cast<bf16x8*>(smem + S::KD + so) = pack8(kd);
        *reinterpret_cast<bf16x8*>(smem + S::KE + so) = pack8(ke);
      }
      // T = A diag(beta): row k, columns i
      {
        const int k = tid >> 3, c8 = tid & 7;
        float tv[8];
        const uint4 ax = lds_chunk(smem + S::AT, k, c8);
        const uint32_t aw[4] = {ax.x, ax.y, ax.z, ax.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 p = unpack_bf16(aw[i]);
          tv[2 * i] = p.x * beta[8 * c8 + 2 * i];
          tv[2 * i + 1] = p.y * beta[8 * c8 + 2 * i + 1];
        }
        *reinterpret_cast<bf16x8*>(smem + S::TT + 2 * sw64_chunk(k, c8)) = pack8(tv);
      }
    }
    ok = tc::mbar_wait(mb + 10, 0);  // dE, dW, dM
    if (__syncthreads_or(!ok)) { ok = false; if (tid == 0) atomicExch(&g_kda_device_error, 7); break; }
    tc::fence_async_smem();  // operand tiles -> tensor cores; the decay region -> the bulk copy below
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 64) {
      // dQt and dKbar (acc64) land over the dead decay region while the MMAs run
      tc::mbar_expect_tx(mb + 1, 2 * S::T128);
      tc::bulk_g2s(smem + S::DQT, P.dQt + tix * TILE64_ELEMS, S::T128, mb + 1);
      tc::bulk_g2s(smem + S::DKB, P.dKb + tix * TILE64_ELEMS, S::T128, mb + 1);
    } else if (tid == 32) {
      tc::fence_after_sync();
      // G2: row side through M, P_J = dM[:, J] Kd[J] (units 4 + J)
      for (int J = 0; J < 4; ++J)
        for (int hf = 0; hf < 2; ++hf)
          tc::mma_bf16(tbase + ((uint32_t)(16 * hf) << 16) + 256 + 64 * J, kdesc(S::DM, J),
                       mdesc(S::KD + hf * 8192, J), idKM, false);
      tc::mma_commit(mb + 3);
    } else if (tid == 0) {
      tc::fence_after_sync();
      // G1: dv = T^T dE (unit 0), dKe = T^T dW (unit 1), dT = dE V^T + dW Ke^T (unit 2)
      for (int hf = 0; hf < 2; ++hf) {
        const uint32_t lo = (uint32_t)(16 * hf) << 16;
        for (int ks = 0; ks < 4; ++ks) {
          tc::mma_bf16(tbase + lo + 0, mdesc(S::TT, ks), mdesc(S::DE + hf * 8192, ks), idMM, ks > 0);
          tc::mma_bf16(tbase + lo + 64, mdesc(S::TT, ks), mdesc(S::DW + hf * 8192, ks), idMM, ks > 0);
        }
      }
      for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(tbase + 128, kdesc(S::DE, ks), kdesc(S::V, ks), idKK, ks > 0);
      for (int ks = 0; ks < 8; ++ks) tc::mma_bf16(tbase + 128, kdesc(S::DW, ks), kdesc(S::KE, ks), idKK, true);
      tc::mma_commit(mb + 2);
      *issued = 0x20Fu;
    }

    // Order of the epilogues: the chain G1 -> dA -> G3 -> X -> G5 -> dL' -> G6/G7 first,
    // the other epilogues while its MMAs run.
    auto fail_if = [&](bool bad) {
      if (__syncthreads_or(bad)) {
        if (tid == 0) atomicExch(&g_kda_device_error, 5);
        return true;
      }
      return false;
    };

    // ---- E1a: dT (64 x 64, lanes 0-15): dbeta_T[j] = sum_i dT_ij A_ij, dA = dT diag(beta)
    ok = tc::mbar_wait(mb + 2, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    {
      float a0[8], a1[8];
      tc::tmem_ld8_async(trow + 128 + 16 * qd, a0);
      tc::tmem_ld8_async(trow + 128 + 16 * qd + 8, a1);
      tc::tmem_wait8(a0);
      tc::tmem_wait8(a1);
      auto pass = [&](float (&acc)[8], int hb) {
        float av[8], cs[8], bv[8];
        const int c8 = (16 * qd + hb) >> 3;
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::AT + 2 * sw64_chunk(r, c8)), av);
        ld8f(beta + 16 * qd + hb, bv);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          cs[v] = acc[v] * av[v];
          acc[v] *= bv[v];
        }
        if (hh == 0) *reinterpret_cast<bf16x8*>(smem + S::DA + 2 * sw64_chunk(r, c8)) = pack8(acc);
        const float dbt = half_reduce_scatter8(cs);
        if (hh == 0 && (lane & 1) == 0) reinterpret_cast<float*>(smem + S::DBT)[s * 64 + 16 * qd + hb + (lane >> 1)] = dbt;
      };
      pass(a0, 0);
      pass(a1, 8);
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // G3: X = dA A^T (unit 3)
      tc::fence_after_sync();
      for (int ks = 0; ks < 4; ++ks) tc::mma_bf16(tbase + 192, kdesc(S::DA, ks), kdesc(S::AT, ks), idKK, ks > 0);
      tc::mma_commit(mb + 4);
      *issued = 0x21Fu;
    }

    // ---- E1b (while G3 runs): dv out; dk and dGam from dKe and the state-pass tiles
    // the gate logits and the gate backward's vectors, for the tail (dE / dW are dead)
    {
      bf16* gre = reinterpret_cast<bf16*>(smem + S::GRE);
      for (int i = tid; i < 64 * 16; i += blockDim.x) {
        const int rr = i >> 4, cc = i & 15;
        const bool okr = rr < nv;
        cp_async16(gre + sw64_chunk(rr, cc), P.in.g + (okr ? ((size_t)(pos.t0 + rr) * H + h) * D + cc * 8 : 0), okr);
      }
      float* gbv = reinterpret_cast<float*>(smem + S::GBV);
      if (tid < 32)
        cp_async16(gbv + 4 * tid, P.dGC + cidx * D + 4 * tid, true);
      else if (tid < 64)
        cp_async16(gbv + D + 4 * (tid - 32), P.in.dt_bias + (size_t)h * D + 4 * (tid - 32), true);
      else if (tid == 64)
        cp_async4(gbv + 2 * D, P.in.A_log + h);
      cp_async_commit();
    }
    ok = tc::mbar_wait(mb + 1, 0);
    if (fail_if(!ok)) { ok = false; break; }
    {
      bf16* dvrow = P.dv + ((size_t)(pos.t0 + r) * H + h) * D + c0;
      const bf16* tq = reinterpret_cast<const bf16*>(smem + S::DQT);
      const bf16* tk = reinterpret_cast<const bf16*>(smem + S::DKB);
      const float* erp = reinterpret_cast<const float*>(smem + S::ER) + s * D + c0;
      const float* ecp = reinterpret_cast<const float*>(smem + S::EC) + s * D + c0;
      const float* rvp = reinterpret_cast<const float*>(smem + S::REV) + s * D + c0;
#pragma unroll
      for (int hb = 0; hb < 16; hb += 8) {  // two 8-column passes
        float dv8[8], acc[8];
        tc::tmem_ld8_async(trow + 0 + 16 * qd + hb, dv8);   // dv
        tc::tmem_ld8_async(trow + 64 + 16 * qd + hb, acc);  // dKe
        float gq[8], gk[8], qa[8], ka[8], kd[8], colsum[8], g8[8];
        const int c8 = (c0 + hb) >> 3;
        unpack8(*reinterpret_cast<const bf16x8*>(tq + acc64_off(r, c0 + hb)), gq);
        unpack8(*reinterpret_cast<const bf16x8*>(tk + acc64_off(r, c0 + hb)), gk);
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::QA + 2 * sw64_chunk(r, c8)), qa);
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::KA + 2 * sw64_chunk(r, c8)), ka);
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::KD + 2 * sw64_chunk(r, c8)), kd);
        float erv[8], ecv[8], rvv[8];
        ld8f(erp + hb, erv);
        ld8f(ecp + hb, ecv);
        ld8f(rvp + hb, rvv);
        tc::tmem_wait8(dv8);
        tc::tmem_wait8(acc);
        if (r < nv) *reinterpret_cast<bf16x8*>(dvrow + hb) = pack8(dv8);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const int u = hb + v;
          const float er = erv[v], ec = ecv[v], rv = rvv[v];
          const float eg = af[u] * er, egc = rv * rcp(af[u]) * ec;
          const float kbar = kd[v] * rv * ec;
          dk[u] = acc[v] * eg + gk[v] * egc;
          g8[v] = ka[v] * er * acc[v] + qa[v] * er * gq[v] - kbar * gk[v];
          colsum[v] = kbar * gk[v];
        }
        st_dg8(dgb, r, c0 + hb, g8);
        // column sums over the 16 rows of this lane half
        const float cs = half_reduce_scatter8(colsum);
        if ((lane & 1) == 0) reinterpret_cast<float*>(smem + S::COLS)[s * D + c0 + hb + ((lane & 15) >> 1)] = cs;
      }
    }

    // row sides: dX += af (P_I + sum_J<I c'_IJ P_J), dGam += rowop o (...); the block's
    // accumulator slices load together (one wait)
    auto row_side = [&](uint32_t unit0, int rowop, float (&dx)[16]) {
      const float* cpb = reinterpret_cast<const float*>(smem + S::CP) + c0;
#pragma unroll
      for (int hb = 0; hb < 16; hb += 8) {
        float out[8], p0[8], p1[8], p2[8];
        const uint32_t col = trow + unit0 + 16 * qd + hb;
        tc::tmem_ld8_async(col + 64 * s, out);
        if (s > 0) tc::tmem_ld8_async(col + 0, p0);
        if (s > 1) tc::tmem_ld8_async(col + 64, p1);
        if (s > 2) tc::tmem_ld8_async(col + 128, p2);
        float ro[8], g8[8], cp[8];
        unpack8(*reinterpret_cast<const bf16x8*>(smem + rowop + 2 * sw64_chunk(r, (c0 + hb) >> 3)), ro);
        {
          const float4 a = *dg_chunk(dgb, r, c0 + hb), b = *dg_chunk(dgb, r, c0 + hb + 4);
          g8[0] = a.x; g8[1] = a.y; g8[2] = a.z; g8[3] = a.w; g8[4] = b.x; g8[5] = b.y; g8[6] = b.z; g8[7] = b.w;
        }
        tc::tmem_wait8(out);
        if (s > 0) {
          tc::tmem_wait8(p0);
          ld8f(cpb + pair_index(s, 0) * D + hb, cp);
#pragma unroll
          for (int v = 0; v < 8; ++v) out[v] = fmaf(cp[v], p0[v], out[v]);
        }
        if (s > 1) {
          tc::tmem_wait8(p1);
          ld8f(cpb + pair_index(s, 1) * D + hb, cp);
#pragma unroll
          for (int v = 0; v < 8; ++v) out[v] = fmaf(cp[v], p1[v], out[v]);
        }
        if (s > 2) {
          tc::tmem_wait8(p2);
          ld8f(cpb + pair_index(s, 2) * D + hb, cp);
#pragma unroll
          for (int v = 0; v < 8; ++v) out[v] = fmaf(cp[v], p2[v], out[v]);
        }
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          dx[hb + v] = fmaf(af[hb + v], out[v], dx[hb + v]);
          g8[v] = fmaf(ro[v], out[v], g8[v]);
        }
        st_dg8(dgb, r, c0 + hb, g8);
      }
    };
    // column sides: tot = R_I + rev_I sum_{Ib > I} c_{Ib,I} R_Ib; then dk += tot / af
    // (the diagonal's 1/af and the off-diagonal bf = rev_I / af at once), dGam -= Kd o tot
    auto column_side = [&](uint32_t unit0) {
      const float* rvp = reinterpret_cast<const float*>(smem + S::REV) + s * D + c0;
      const float* ccb = reinterpret_cast<const float*>(smem + S::CC) + c0;
#pragma unroll
      for (int hb = 0; hb < 16; hb += 8) {
        float tot[8], r1[8], r2[8], r3[8];
        const uint32_t col = trow + unit0 + 16 * qd + hb;
        tc::tmem_ld8_async(col + 64 * s, tot);  // diagonal block: R_I
        if (s < 3) tc::tmem_ld8_async(col + 192, r3);
        if (s < 2) tc::tmem_ld8_async(col + 128, r2);
        if (s < 1) tc::tmem_ld8_async(col + 64, r1);
        float kd[8], g8[8], cc[8], off[8];
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::KD + 2 * sw64_chunk(r, (c0 + hb) >> 3)), kd);
        {
          const float4 a = *dg_chunk(dgb, r, c0 + hb), b = *dg_chunk(dgb, r, c0 + hb + 4);
          g8[0] = a.x; g8[1] = a.y; g8[2] = a.z; g8[3] = a.w; g8[4] = b.x; g8[5] = b.y; g8[6] = b.z; g8[7] = b.w;
        }
        tc::tmem_wait8(tot);
        if (s < 3) {
          tc::tmem_wait8(r3);
          ld8f(ccb + pair_index(3, s) * D + hb, cc);
#pragma unroll
          for (int v = 0; v < 8; ++v) off[v] = cc[v] * r3[v];
          if (s < 2) {
            tc::tmem_wait8(r2);
            ld8f(ccb + pair_index(2, s) * D + hb, cc);
#pragma unroll
            for (int v = 0; v < 8; ++v) off[v] = fmaf(cc[v], r2[v], off[v]);
          }
          if (s < 1) {
            tc::tmem_wait8(r1);
            ld8f(ccb + pair_index(1, s) * D + hb, cc);
#pragma unroll
            for (int v = 0; v < 8; ++v) off[v] = fmaf(cc[v], r1[v], off[v]);
          }
          ld8f(rvp + hb, cc);
#pragma unroll
          for (int v = 0; v < 8; ++v) tot[v] = fmaf(cc[v], off[v], tot[v]);
        }
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          dk[hb + v] = fmaf(rcp(af[hb + v]), tot[v], dk[hb + v]);
          g8[v] = fmaf(-kd[v], tot[v], g8[v]);
        }
        st_dg8(dgb, r, c0 + hb, g8);
      }
    };

    // ---- E3: X -> bf16 tile
    ok = tc::mbar_wait(mb + 4, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    {
      float x0[8], x1[8];
      tc::tmem_ld8_async(trow + 192 + 16 * qd, x0);
      tc::tmem_ld8_async(trow + 192 + 16 * qd + 8, x1);
      tc::tmem_wait8(x0);
      tc::tmem_wait8(x1);
      if (hh == 0) {
        *reinterpret_cast<bf16x8*>(smem + S::XS + 2 * sw64_chunk(r, (16 * qd) >> 3)) = pack8(x0);
        *reinterpret_cast<bf16x8*>(smem + S::XS + 2 * sw64_chunk(r, (16 * qd + 8) >> 3)) = pack8(x1);
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // G5: -dL = A^T X (unit 0; dv was read in E1b)
      tc::fence_after_sync();
      for (int ks = 0; ks < 4; ++ks) tc::mma_bf16(tbase + 0, mdesc(S::AT, ks), mdesc(S::XS, ks), idMM, ks > 0);
      tc::mma_commit(mb + 6);
      *issued = 0x25Fu;
    }

    // ---- E2 (while G5 runs): dq = dQt 2^Gam + row side through M; dq out
    ok = tc::mbar_wait(mb + 3, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    {
      const bf16* tq = reinterpret_cast<const bf16*>(smem + S::DQT);
      const float* erp = reinterpret_cast<const float*>(smem + S::ER) + s * D + c0;
#pragma unroll
      for (int hb = 0; hb < 16; hb += 8) {
        float gq[8], er[8];
        unpack8(*reinterpret_cast<const bf16x8*>(tq + acc64_off(r, c0 + hb)), gq);
        ld8f(erp + hb, er);
#pragma unroll
        for (int v = 0; v < 8; ++v) dq[hb + v] = gq[v] * af[hb + v] * er[v];
      }
    }
    row_side(256, S::QA, dq);
    if (r < nv) st_global16(P.dq_hat + ((size_t)(pos.t0 + r) * H + h) * D + c0, dq);
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // G4: column side through M, R_I = dM[I, :]^T Qa[I] (units 4 + I)
      tc::fence_after_sync();
      for (int I = 0; I < 4; ++I)
        for (int hf = 0; hf < 2; ++hf)
          tc::mma_bf16(tbase + ((uint32_t)(16 * hf) << 16) + 256 + 64 * I, mdesc(S::DM, I),
                       mdesc(S::QA + hf * 8192, I), idMM, false);
      tc::mma_commit(mb + 5);
      *issued = 0x27Fu;
    }

    // ---- E4: dL = -(A^T X), strictly lower: dbeta_L = rowsum(dL o L'), dL' = diag(beta) dL
    ok = tc::mbar_wait(mb + 6, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    {
      float rs = 0.f;
      const float br = beta[r];
      float l0[8], l1[8];
      tc::tmem_ld8_async(trow + 0 + 16 * qd, l0);
      tc::tmem_ld8_async(trow + 0 + 16 * qd + 8, l1);
      tc::tmem_wait8(l0);
      tc::tmem_wait8(l1);
      auto pass = [&](float (&acc)[8], int hb) {
        float lp[8];
        const int c8 = (16 * qd + hb) >> 3;
        unpack8(*reinterpret_cast<const bf16x8*>(smem + S::LPT + 2 * sw64_chunk(r, c8)), lp);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float x = (16 * qd + hb + v < r) ? -acc[v] : 0.f;
          rs = fmaf(x, lp[v], rs);
          acc[v] = x * br;
        }
        if (hh == 0) *reinterpret_cast<bf16x8*>(smem + S::DLP + 2 * sw64_chunk(r, c8)) = pack8(acc);
      };
      pass(l0, 0);
      pass(l1, 8);
      if (hh == 0) reinterpret_cast<float*>(smem + S::DBL)[qd * 64 + r] = rs;
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // G6: row side through L', P_J = dL'[:, J] Kd[J] (units J)
      tc::fence_after_sync();
      for (int J = 0; J < 4; ++J)
        for (int hf = 0; hf < 2; ++hf)
          tc::mma_bf16(tbase + ((uint32_t)(16 * hf) << 16) + 64 * J, kdesc(S::DLP, J), mdesc(S::KD + hf * 8192, J),
                       idKM, false);
      tc::mma_commit(mb + 7);
      *issued = 0x2FFu;
    }

    // ---- E5 (while G6 runs): column side through M
    ok = tc::mbar_wait(mb + 5, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    column_side(256);
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {  // G7: column side through L', R_I = dL'[I, :]^T Ka[I] (units 4 + I)
      tc::fence_after_sync();
      for (int I = 0; I < 4; ++I)
        for (int hf = 0; hf < 2; ++hf)
          tc::mma_bf16(tbase + ((uint32_t)(16 * hf) << 16) + 256 + 64 * I, mdesc(S::DLP, I),
                       mdesc(S::KA + hf * 8192, I), idMM, false);
      tc::mma_commit(mb + 8);
      *issued = 0x3FFu;
    }

    // ---- E6: row side through L'; E7: column side through L'
    ok = tc::mbar_wait(mb + 7, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    row_side(0, S::KA, dk);
    ok = tc::mbar_wait(mb + 8, 0);
    if (fail_if(!ok)) { ok = false; break; }
    tc::fence_after_sync();
    column_side(256);
  }

  if (!ok) {
    // let what is in flight finish (bounded), then release TMEM and leave
    const uint32_t iss = *issued;
    for (int i = 0; i < 11; ++i)
      if (iss & (1u << i)) tc::mbar_wait(mb + i, 0, 1u << 22);
    cp_async_wait<0>();
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tbase, 512);
    return;
  }

  // ---- outputs: dk_hat (dq_hat left after the row side through M)
  if (r < nv) st_global16(P.dk_hat + ((size_t)(pos.t0 + r) * H + h) * D + c0, dk);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);

  // ---- the gate backward, in the same row layout.  dg_r = f(r) (C + sum_{r' >= r} dGam_r'),
  // C = dGam_C + sum over the chunk of Kbar o dKbar: a suffix scan over the 16 rows of
  // this lane half, plus the totals of the later sub-chunk blocks.
  float* qtot = reinterpret_cast<float*>(smem + S::PSUM);  // [4][128] block totals, then [2][4][128] sums
  {
    // the scan runs down the columns of dGam in shared memory, in place: thread
    // t takes channel t & 127 of block t >> 7 (a warp's 32 channels are one
    // 128-byte span of a row, so the accesses are conflict-free)
    const int cc = tid & 127, sb = tid >> 7;
    float run = 0.f;
#pragma unroll
    for (int i = 15; i >= 0; --i) {
      float* p = reinterpret_cast<float*>(dg_chunk(dgb, 16 * sb + i, cc)) + (cc & 3);
      run += *p;
      *p = run;
    }
    qtot[sb * D + cc] = run;  // the block total
  }
  __syncthreads();
  float dG[16];
  ld_dg16(dgb, r, c0, dG);  // this thread's suffix sums
  cp_async_wait<0>();  // gate logits and vectors
  __syncthreads();
  float* coff = qtot + 4 * D;  // [4][128]: what the rows of block s add to their suffix sums
  {
    const int sb2 = tid >> 7, cc = tid & 127;
    const float* gbv = reinterpret_cast<const float*>(smem + S::GBV);
    const float* cols = reinterpret_cast<const float*>(smem + S::COLS);
    float o = gbv[cc] + ((cols[cc] + cols[D + cc]) + (cols[2 * D + cc] + cols[3 * D + cc]));
    for (int s2 = sb2 + 1; s2 < 4; ++s2) o += qtot[s2 * D + cc];
    coff[sb2 * D + cc] = o;
  }
  __syncthreads();
  {
    const float* gbv = reinterpret_cast<const float*>(smem + S::GBV);
    const float eA = __expf(gbv[2 * D]);
    const bool okr = r < nv;
    bf16* dgrow = P.dg + ((size_t)(pos.t0 + r) * H + h) * D + c0;
    float a2[2], b2[2];
#pragma unroll
    for (int hb = 0; hb < 16; hb += 8) {
      float gl[8], ofs[8], bias[8], sA[8], sB[8];
      unpack8(*reinterpret_cast<const bf16x8*>(smem + S::GRE + 2 * sw64_chunk(r, (c0 + hb) >> 3)), gl);
      ld8f(coff + s * D + c0 + hb, ofs);
      ld8f(gbv + D + c0 + hb, bias);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float run = dG[hb + v] + ofs[v];
        const float z = eA * (gl[v] + bias[v]);
        const float sg = sigmoidf_(z);
        const float dz = run * P.in.lower_bound * sg * (1.f - sg);
        const float dx = dz * eA;
        gl[v] = dx;
        sA[v] = okr ? dz * z : 0.f;
        sB[v] = okr ? dx : 0.f;
      }
      if (okr) *reinterpret_cast<bf16x8*>(dgrow + hb) = pack8(gl);
      a2[hb >> 3] = half_reduce_scatter8(sA);
      b2[hb >> 3] = half_reduce_scatter8(sB);
    }
    __syncthreads();  // the block totals and offsets are read
    if ((lane & 1) == 0) {
      const int cc = c0 + ((lane & 15) >> 1);
      qtot[s * D + cc] = a2[0];
      qtot[s * D + cc + 8] = a2[1];
      qtot[4 * D + s * D + cc] = b2[0];
      qtot[4 * D + s * D + cc + 8] = b2[1];
    }
    __syncthreads();
    if (tid < D) {
      P.partA[cidx * D + tid] = (qtot[tid] + qtot[D + tid]) + (qtot[2 * D + tid] + qtot[3 * D + tid]);
    } else if (tid < 2 * D) {
      const int cc = tid - D;
      const float* q2 = qtot + 4 * D;
      P.partB[cidx * D + cc] = (q2[cc] + q2[D + cc]) + (q2[2 * D + cc] + q2[3 * D + cc]);
    }
  }
  if (tid >= 2 * D && tid < 2 * D + 64) {
    const int rr = tid - 2 * D;
    if (rr < nv) {
      const float* dbt = reinterpret_cast<const float*>(smem + S::DBT);
      const float* dbl = reinterpret_cast<const float*>(smem + S::DBL);
      const float db = dbt[rr] + dbt[64 + rr] + dbt[128 + rr] + dbt[192 + rr] + dbl[rr] + dbl[64 + rr] +
                       dbl[128 + rr] + dbl[192 + rr];
      const float bt = beta[rr];
      P.dbeta[(size_t)(pos.t0 + rr) * H + h] = __float2bfloat16(db * bt * (1.f - bt));
    }
  }
}

}  // namespace kda
