// Parameters of the reverse state pass (kda_bwd_state_tc.cuh) and the
// negated-A warp MMA used by the chunk kernels.
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
  const bf16 *W, *Qt, *Kb, *M, *dO;  // [T_total][H][128] (M: [T_total][H][64])
  const bf16 *E, *hs;                // [chunks][H] acc64 / st128 tiles
  const float* dC;
  const float* dht;  // [N][H][128][128] or null
  bf16 *dE, *dQt, *dW, *dKb, *dM;  // [chunks][H] acc64 tiles (dM: acc64n64)
  float* dGC;        // [chunks][H][128]
  float* dh0;        // [N][H][128][128] or null
};

}  // namespace kda
