// Reverse state pass of the chunked KDA backward.
//
// One CTA per (sequence, head) walks the chunks last to first, carrying the
// gradient of the chunk-end state dS (128x128 fp32, registers).  Per chunk,
// with S0 the chunk-start state saved by the forward (bf16):
//   dE   = M^T dO + Kbar dS
//   dGC  = 2^Gam_C * rowsum(dS o S0)          (extra gradient of Gam_C)
//   dQt  = dO S0^T,  dW = -dE S0^T,  dKbar = E dS^T,  dM = tril(dO E^T)
//   dS  <- diag(2^Gam_C) dS + Qt^T dO - W^T dE
// and finally dh0 = dS.  Everything after dE only needs the chunk's own data,
// but is computed here because S0 and dS are already on chip.
#pragma once

#include "kda_fwd.cuh"

namespace kda {

template <int NT, bool TA, bool TB>
__device__ __forceinline__ void warp_mma_neg(float (&acc)[NT][4], const bf16* A, int lda, int m0,
                                             const bf16* B, int ldb, int n0, int k0, int K) {
#pragma unroll 2
  for (int kk = 0; kk < K; kk += 16) {
    uint32_t a[4];
    if (TA) load_AT(a, A, lda, m0, k0 + kk); else load_A(a, A, lda, m0, k0 + kk);
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] ^= 0x80008000u;
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      if (TB) load_B_kn(b, B, ldb, n0 + 8 * j, k0 + kk); else load_B_nk(b, B, ldb, n0 + 8 * j, k0 + kk);
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}

struct BwdStateParams {
  SeqInfo seq;
  int H;
  const bf16 *W, *Qt, *Kb, *M, *E, *hs, *dO;
  const float* dC;
  const float* dht;  // [N][H][128][128] or null
  bf16 *dE, *dQt, *dW, *dKb, *dM;
  float* dGC;        // [chunks][H][128]
  float* dh0;        // [N][H][128][128] or null
};

// Loads come in two cp.async groups per chunk:
//   A = M, Kbar, dO, 2^Gam_C  -- everything dE needs; double-buffered and
//       prefetched one chunk ahead, so dE starts as soon as a chunk begins;
//   B = W, Qt, E, S0          -- issued at the chunk start, first used after dE.
struct BwdStateSmem {
  static constexpr int TILE = 64 * LD128 * 2;
  static constexpr int A_M = 0, A_KB = 64 * LD64 * 2, A_DO = A_KB + TILE, A_DC = A_DO + TILE;
  static constexpr int A_STAGE = A_DC + D * 4;              // 44544
  static constexpr int W = 2 * A_STAGE, QT = W + TILE, E = QT + TILE;
  static constexpr int S0 = E + TILE;                       // 128 x LD128
  static constexpr int DS = S0 + 128 * LD128 * 2;           // 128 x LD128
  static constexpr int DE = DS + 128 * LD128 * 2;           // 64 x LD128
  static constexpr int END = DE + 64 * LD128 * 2;
};
static_assert(BwdStateSmem::END <= 232448, "bwd state shared memory");

__device__ __forceinline__ void store_frag_rows(bf16* g, const float (&acc)[8][4], int m0, int n0, int nv, int t0,
                                                int H, int h, bool neg) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
      if (r < nv) {
        float x0 = acc[j][e], x1 = acc[j][e + 1];
        if (neg) { x0 = -x0; x1 = -x1; }
        *reinterpret_cast<uint32_t*>(g + ((size_t)(t0 + r) * H + h) * D + cc) = pack_bf16(x0, x1);
      }
    }
}

__global__ void __launch_bounds__(256, 1) kda_bwd_state_kernel(BwdStateParams P) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int n = blockIdx.x, h = blockIdx.y, H = P.H;
  const int warp = threadIdx.x >> 5;
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  const int nchunks = seq_nchunks(P.seq, n);
  const int cbase = seq_chunk_base(P.seq, n);
  bf16* Wt = reinterpret_cast<bf16*>(smem + BwdStateSmem::W);
  bf16* Qt = reinterpret_cast<bf16*>(smem + BwdStateSmem::QT);
  bf16* Et = reinterpret_cast<bf16*>(smem + BwdStateSmem::E);
  bf16* S0 = reinterpret_cast<bf16*>(smem + BwdStateSmem::S0);
  bf16* dSs = reinterpret_cast<bf16*>(smem + BwdStateSmem::DS);
  bf16* dEs = reinterpret_cast<bf16*>(smem + BwdStateSmem::DE);
  auto stage = [&](int b) { return smem + b * BwdStateSmem::A_STAGE; };
  auto issue_A = [&](int ci, int b) {
    const int t0 = bos + ci * C, nv = min(C, eos - t0);
    unsigned char* st = stage(b);
    load_tile64(reinterpret_cast<bf16*>(st + BwdStateSmem::A_M), P.M, t0, nv, H, h);
    load_tile128(reinterpret_cast<bf16*>(st + BwdStateSmem::A_KB), P.Kb, t0, nv, H, h);
    load_tile128(reinterpret_cast<bf16*>(st + BwdStateSmem::A_DO), P.dO, t0, nv, H, h);
    load_vec128(reinterpret_cast<float*>(st + BwdStateSmem::A_DC), P.dC + ((size_t)(cbase + ci) * H + h) * D);
  };

  if (nchunks > 0) issue_A(nchunks - 1, (nchunks - 1) & 1);
  cp_async_commit();

  float dS[16][4];
  const float* dht = P.dht ? P.dht + ((size_t)n * H + h) * D * D : nullptr;
#pragma unroll
  for (int j = 0; j < 16; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int r = 16 * warp + acc_row(e), cc = acc_col(j, e);
      dS[j][e] = dht ? dht[r * D + cc] : 0.f;
    }

  const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
  for (int ci = nchunks - 1; ci >= 0; --ci) {
    const int t0 = bos + ci * C;
    const int nv = min(C, eos - t0);
    const size_t cidx = (size_t)(cbase + ci) * H + h;
    unsigned char* st = stage(ci & 1);
    const bf16* Mt = reinterpret_cast<const bf16*>(st + BwdStateSmem::A_M);
    const bf16* Kb = reinterpret_cast<const bf16*>(st + BwdStateSmem::A_KB);
    const bf16* dO = reinterpret_cast<const bf16*>(st + BwdStateSmem::A_DO);
    const float* dC = reinterpret_cast<const float*>(st + BwdStateSmem::A_DC);
    // group B of this chunk, then group A of the next one (an empty group at
    // the last step keeps the group count uniform)
    load_tile128(Wt, P.W, t0, nv, H, h);
    load_tile128(Qt, P.Qt, t0, nv, H, h);
    load_tile128(Et, P.E, t0, nv, H, h);
    {
      const bf16* src = P.hs + cidx * D * D;
      for (int i = threadIdx.x; i < 128 * 16; i += blockDim.x) {
        int r = i >> 4, cc = i & 15;
        cp_async16(S0 + r * LD128 + cc * 8, src + r * D + cc * 8, true);
      }
    }
    cp_async_commit();
    if (ci > 0) issue_A(ci - 1, (ci - 1) & 1);
    cp_async_commit();
    // dS -> bf16 tile
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = 16 * warp + acc_row(e), cc = acc_col(j, e);
        *reinterpret_cast<uint32_t*>(dSs + r * LD128 + cc) = pack_bf16(dS[j][e], dS[j][e + 1]);
      }
    cp_async_wait<2>();  // group A of this chunk
    __syncthreads();
    // dE = M^T dO + Kbar dS
    {
      float acc[8][4];
      zero_acc<8>(acc);
      warp_mma<8, true, true>(acc, Mt, LD64, m0, dO, LD128, n0, 0, 64);
      warp_mma<8, false, true>(acc, Kb, LD128, m0, dSs, LD128, n0, 0, 128);
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
          uint32_t pk = pack_bf16(acc[j][e], acc[j][e + 1]);
          *reinterpret_cast<uint32_t*>(dEs + r * LD128 + cc) = pk;
          if (r < nv) *reinterpret_cast<uint32_t*>(P.dE + ((size_t)(t0 + r) * H + h) * D + cc) = pk;
        }
    }
    cp_async_wait<1>();  // group B
    __syncthreads();
    // dGC = 2^Gam_C * rowsum(dS o S0)
    {
      float part[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int r = 16 * warp + acc_row(e), cc = acc_col(j, e);
          float2 s = unpack_bf16(*reinterpret_cast<const uint32_t*>(S0 + r * LD128 + cc));
          part[e >> 1] += dS[j][e] * s.x + dS[j][e + 1] * s.y;
        }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        part[i] += __shfl_xor_sync(0xffffffffu, part[i], 1);
        part[i] += __shfl_xor_sync(0xffffffffu, part[i], 2);
      }
      if ((threadIdx.x & 3) == 0) {
        int r0 = 16 * warp + acc_row(0);
        P.dGC[cidx * D + r0] = dC[r0] * part[0];
        P.dGC[cidx * D + r0 + 8] = dC[r0 + 8] * part[1];
      }
    }
    // dS <- diag(dC) dS + Qt^T dO - W^T dE
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) dS[j][e] *= dC[16 * warp + acc_row(e)];
    warp_mma<16, true, true>(dS, Qt, LD128, 16 * warp, dO, LD128, 0, 0, 64);
    warp_mma_neg<16, true, true>(dS, Wt, LD128, 16 * warp, dEs, LD128, 0, 0, 64);
    // chunk-local gradient pieces
    {
      float acc[8][4];
      zero_acc<8>(acc);
      warp_mma<8, false, false>(acc, dO, LD128, m0, S0, LD128, n0, 0, 128);
      store_frag_rows(P.dQt, acc, m0, n0, nv, t0, H, h, false);
      zero_acc<8>(acc);
      warp_mma<8, false, false>(acc, dEs, LD128, m0, S0, LD128, n0, 0, 128);
      store_frag_rows(P.dW, acc, m0, n0, nv, t0, H, h, true);
      zero_acc<8>(acc);
      warp_mma<8, false, false>(acc, Et, LD128, m0, dSs, LD128, n0, 0, 128);
      store_frag_rows(P.dKb, acc, m0, n0, nv, t0, H, h, false);
    }
    {
      float acc[4][4];
      zero_acc<4>(acc);
      const int n1 = 32 * (warp >> 2);
      warp_mma<4, false, false>(acc, dO, LD128, m0, Et, LD128, n1, 0, 128);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int r = m0 + acc_row(e), cc = n1 + acc_col(j, e);
          if (r < nv) {
            float x0 = cc <= r ? acc[j][e] : 0.f;
            float x1 = cc + 1 <= r ? acc[j][e + 1] : 0.f;
            *reinterpret_cast<uint32_t*>(P.dM + ((size_t)(t0 + r) * H + h) * 64 + cc) = pack_bf16(x0, x1);
          }
        }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (P.dh0) {
    float* dst = P.dh0 + ((size_t)n * H + h) * D * D;
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = 16 * warp + acc_row(e), cc = acc_col(j, e);
        *reinterpret_cast<float2*>(dst + r * D + cc) = make_float2(dS[j][e], dS[j][e + 1]);
      }
  }
}

}  // namespace kda
