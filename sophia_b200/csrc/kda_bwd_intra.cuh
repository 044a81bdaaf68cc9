// Chunk-parallel backward of the chunked KDA layer.
//
// One CTA per (chunk, head).  Loads the forward's saved prologue products
// (normalised q and k, post-conv v, the decay cumsum, beta) and its A =
// (I + diag(beta) L')^-1, rebuilds the decayed operand tiles and L' from them
// (T = A diag(beta)),
// then, from the state-pass gradient pieces (dE, dW, dQt, dKbar, dM, dGC):
//   dv  = T^T dE                      (written out as the value gradient)
//   dKe = T^T dW,  dT = dE v^T + dW Ke^T,  dbeta += colsum(dT o A)
//   dA  = dT diag(beta),  dL = -A^T dA A^T (strictly lower)
//   dbeta += rowsum(dL o L'),  dL' = diag(beta) dL
//   block products of dM and dL' against the decayed q/k operands give the
//   gradients through M (Aqk) and L'
//   dGam collects q o dq + k o dk terms; dg = reverse cumsum of dGam inside
//   the chunk; the gate and beta sigmoids are differentiated last.
// Outputs: dq_hat, dk_hat (gradients of the normalised, scaled q and of the
// normalised k; the L2-norm and conv backward run in the post kernel), dv,
// dg_logits, dbeta_logits and per-chunk partial sums for dA_log and dt_bias.
//
// 512 threads.  Accumulator layout "F": warp w owns rows 16*(w&3) .. +15 and
// columns 32*(w>>2) .. +31 of every 64x128 per-chunk gradient; the per-element
// decay factors of that tile stay in registers for the whole kernel.
#pragma once

#include "kda_fwd.cuh"
#include "kda_tc.cuh"

namespace kda {

struct BwdIntraParams {
  PrologueIn in;
  SeqInfo seq;
  bool conv;
  const bf16 *dE, *dW, *dQt, *dKb, *dM;  // [chunks][H] acc64 tiles (dM: acc64n64)
  const float* A;                        // [chunks][H] fp32 [64][LDF64] tiles saved by the forward
  const bf16 *QN, *KN, *VN;              // [chunks][H] [64][128] bf16 prologue products of the forward
  const float *GM, *BT;                  // [chunks][H] [64][LDG] fp32 decay cumsum, [64] fp32 beta
  const float* dGC;
  bf16 *dq_hat, *dk_hat, *dv;  // [T_total][H][128]
  bf16 *dg, *dbeta;            // [T_total][H][128], [T_total][H]
  float *partA, *partB;        // [chunks][H][128]
};

struct BwdIntraSmem {
  static constexpr int OPSZ = 64 * LD128 * 2;                // 17408
  static constexpr int OPS = 0;                              // 6 operand tiles
  static constexpr int GAM = OPS + 6 * OPSZ;                 // 64 x LDG fp32 (later dQt, dKbar, dGam)
  static constexpr int DEW = GAM + 64 * LDG * 4;             // dE, dW tiles
  static constexpr int RAW = DEW + 2 * OPSZ;                 // raw q/k/v, later small tiles
  static constexpr int RAWSZ = 51712;
  static constexpr int CVEC = RAW + RAWSZ;                   // 6 x 128 fp32
  static constexpr int ER = CVEC + 6 * D * 4;                // 4 x 128 fp32
  static constexpr int EC = ER + 4 * D * 4;                  // 4 x 128 fp32
  static constexpr int BETA = EC + 4 * D * 4;                // 64 fp32
  static constexpr int BRAW = BETA + 64 * 4;                 // 64 bf16
  static constexpr int MISC = BRAW + 64 * 2;                 // mbarriers: gradient tiles, prologue products
  static constexpr int END = MISC + 16;
  // RAW aliases after the operands are built
  static constexpr int AINV = RAW + 16640;                   // fp32 [64][LDF64] A from the forward (until the T build;
                                                             // DMS reuses part of it afterwards)
  static constexpr int LPB = RAW + 33280;                    // bf16 64 x LD64 (after inverse)
  static constexpr int ABF = RAW;                            // bf16 64 x LD64
  static constexpr int TBF = RAW + 42496;                    // bf16 64 x LD64
  static constexpr int DMS = RAW + 9216;                     // bf16 64 x LD64
  static constexpr int DLS = RAW + 18432;                    // bf16 64 x LD64
  static constexpr int DBT = RAW + 27648;                    // fp32 4 x 64   (dbeta from T)
  static constexpr int DBL = DBT + 1024;                     // fp32 4 x 64   (dbeta from L)
  static constexpr int COLS = DBL + 1024;                    // fp32 4 x 128  (sum Kbar o dKbar)
  static_assert(COLS + 2048 <= LPB, "small tiles overlap Lp bf16");
  static constexpr int GB = COLS + 2048;                     // fp32 dGam_C [128], dt_bias [128], A_log
                                                             // (over the dead A tile, after the T build)
  static_assert(GB + (2 * D + 4) * 4 <= LPB && GB % 16 == 0, "gate-backward vectors overlap Lp bf16");
  static_assert(TBF + 64 * LD64 * 2 <= RAWSZ + RAW, "T tile overflows");
  static_assert(AINV + A_TILE_ELEMS * 4 <= LPB && AINV % 16 == 0, "A tile overlaps Lp bf16 or is misaligned");
  // DEW aliases after the WY backward
  static constexpr int DAS = DEW;                            // bf16 64 x LD64
  static constexpr int XS = DEW + 9216;                      // bf16 64 x LD64
  static constexpr int GRE = DEW + 18432;                    // bf16 64 x 128 gate logits (reloaded)
  static_assert(GRE + 64 * D * 2 <= RAW, "gate reload overflows");
  static_assert(MISC % 8 == 0 && DEW % 16 == 0 && GAM % 16 == 0, "bulk-copy targets and mbarrier alignment");
};

__global__ void __launch_bounds__(INTRA_THREADS, 1) kda_bwd_intra_kernel(BwdIntraParams P) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int c = blockIdx.x, h = blockIdx.y;
  ChunkPos pos = chunk_pos(P.seq, c);
  if (!pos.valid) return;
  const int H = P.in.H;
  const int nv = pos.t1 - pos.t0;
  const int tid = threadIdx.x, warp = tid >> 5;
  const size_t cidx = (size_t)c * H + h;
  const size_t tix = tile_index(P.seq, c, h);

  PrologueSmem ps;
  ps.xq = reinterpret_cast<bf16*>(smem + BwdIntraSmem::RAW);
  ps.xk = ps.xq + 64 * D;
  ps.xv = ps.xk + 64 * D;
  ps.braw = reinterpret_cast<bf16*>(smem + BwdIntraSmem::BRAW);
  ps.gam = reinterpret_cast<float*>(smem + BwdIntraSmem::GAM);
  ps.beta = reinterpret_cast<float*>(smem + BwdIntraSmem::BETA);

  // The forward's prologue products (scaled normalised q, normalised k,
  // post-conv v, the log2 decay cumsum in its padded layout, beta) arrive by
  // five bulk copies; each thread then takes its strip.
  uint64_t* pro_ready = reinterpret_cast<uint64_t*>(smem + BwdIntraSmem::MISC) + 1;
  if (tid == 0) {
    tc::mbar_init(reinterpret_cast<uint64_t*>(smem + BwdIntraSmem::MISC), 2);  // dE/dW, then the rest
    tc::mbar_init(pro_ready, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    constexpr uint32_t TB = TILE64_ELEMS * 2, GB = 64 * LDG * 4, BB = 64 * 4;
    tc::mbar_expect_tx(pro_ready, 3 * TB + GB + BB);
    tc::bulk_g2s(ps.xq, P.QN + tix * TILE64_ELEMS, TB, pro_ready);
    tc::bulk_g2s(ps.xk, P.KN + tix * TILE64_ELEMS, TB, pro_ready);
    tc::bulk_g2s(ps.xv, P.VN + tix * TILE64_ELEMS, TB, pro_ready);
    tc::bulk_g2s(ps.gam, P.GM + tix * 64 * LDG, GB, pro_ready);
    tc::bulk_g2s(ps.beta, P.BT + tix * 64, BB, pro_ready);
  }
  if (__syncthreads_or(!tc::mbar_wait(pro_ready, 0))) {
    // the products did not arrive in time: record it, let the copies land
    // (bounded) so none writes into a finished CTA's shared memory, and leave
    if (tid == 0) atomicExch(&g_kda_device_error, 7);
    tc::mbar_wait(pro_ready, 0);
    return;
  }
  // dE and dW land in their own region while the operands are built; dQt,
  // dKbar and A follow once the decay and raw regions are free
  if (tid == 0) {
    constexpr uint32_t TB = TILE64_ELEMS * 2;
    uint64_t* tr = reinterpret_cast<uint64_t*>(smem + BwdIntraSmem::MISC);
    bf16* de = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DEW);
    tc::mbar_expect_tx(tr, 2 * TB);
    tc::bulk_g2s(de, P.dE + tix * TILE64_ELEMS, TB, tr);
    tc::bulk_g2s(de + 64 * LD128, P.dW + tix * TILE64_ELEMS, TB, tr);
  }
  Strip s;
  {
    const int tg = tid >> 4, cg = tid & 15;
#pragma unroll
    for (int r = 0; r < STRIP; ++r) {
      const int t = STRIP * tg + r;
      unpack8(*reinterpret_cast<const bf16x8*>(ps.xq + t * D + 8 * cg), s.q[r]);
      unpack8(*reinterpret_cast<const bf16x8*>(ps.xk + t * D + 8 * cg), s.k[r]);
      unpack8(*reinterpret_cast<const bf16x8*>(ps.xv + t * D + 8 * cg), s.v[r]);
#pragma unroll
      for (int c = 0; c < 8; ++c) s.gam[r][c] = ps.gam[t * LDG + 8 * cg + c];
    }
  }
  __syncthreads();

  Operands op;
  op.Qa = reinterpret_cast<bf16*>(smem + BwdIntraSmem::OPS);
  op.Ka = op.Qa + 64 * LD128;
  op.Kd = op.Ka + 64 * LD128;
  op.Kb = op.Kd + 64 * LD128;
  op.V = op.Kb + 64 * LD128;
  op.Ke = op.V + 64 * LD128;
  op.cvec = reinterpret_cast<float*>(smem + BwdIntraSmem::CVEC);
  op.er = reinterpret_cast<float*>(smem + BwdIntraSmem::ER);
  op.ec = reinterpret_cast<float*>(smem + BwdIntraSmem::EC);
  build_operands<false>(s, ps.gam, op, nullptr, nullptr);

  // F layout of this warp and its per-element decay factors
  const int I = warp & 3;             // row block
  const int m0 = 16 * I, n0 = 32 * (warp >> 2);
  float af[4][4], bfv[4][4];          // a = 2^(Gam - Gam_r(I)), b = 2^(Gam_e(I) - Gam)
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int r = m0 + acc_row(e), col = n0 + acc_col(j, e);
      float G = ps.gam[r * LDG + col];
      af[j][e] = ex2(G - ps.gam[m0 * LDG + col]);
      bfv[j][e] = ex2(ps.gam[(m0 + 15) * LDG + col] - G);
    }
  tc::fence_async_smem();  // the regions below are rewritten by the bulk copies
  __syncthreads();

  // The state-pass gradient tiles (acc64 order, rows past the end zero) and
  // A = (I + diag(beta) L')^-1 as the forward computed it arrive by bulk copies
  // issued by one thread (dE and dW since the products landed, the rest now),
  // so the warps go on with L' meanwhile; the tiles stay in their global order
  // (Acc64Tile addressing).  dQt and dKbar land in the dead decay region, A in
  // the dead raw region (clear of L', which l_blocks writes below).
  bf16* dEs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DEW);
  bf16* dWs = dEs + 64 * LD128;
  bf16* dQs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::GAM);
  bf16* dKs = dQs + 64 * D;
  float* Asm = reinterpret_cast<float*>(smem + BwdIntraSmem::AINV);
  uint64_t* tiles_ready = reinterpret_cast<uint64_t*>(smem + BwdIntraSmem::MISC);
  if (tid == 0) {
    constexpr uint32_t TB = TILE64_ELEMS * 2, AB = A_TILE_ELEMS * 4;
    tc::mbar_expect_tx(tiles_ready, 2 * TB + AB);
    tc::bulk_g2s(dQs, P.dQt + tix * TILE64_ELEMS, TB, tiles_ready);
    tc::bulk_g2s(dKs, P.dKb + tix * TILE64_ELEMS, TB, tiles_ready);
    tc::bulk_g2s(Asm, P.A + tix * A_TILE_ELEMS, AB, tiles_ready);
  }
  const Acc64Tile dEt{dEs}, dWt{dWs};

  bf16* Lpb = reinterpret_cast<bf16*>(smem + BwdIntraSmem::LPB);
  l_blocks_bf16(op, Lpb);  // only the dbeta row sums read L', in bf16
  if (__syncthreads_or(!tc::mbar_wait(tiles_ready, 0))) {
    if (tid == 0) atomicExch(&g_kda_device_error, 5);
    tc::mbar_wait(tiles_ready, 0);
    return;
  }
  bf16* Abf = reinterpret_cast<bf16*>(smem + BwdIntraSmem::ABF);
  bf16* Tbf = reinterpret_cast<bf16*>(smem + BwdIntraSmem::TBF);
  {
    // A (fp32, [16640, 33280) of the raw region) -> Abf ([0, 9216)) and Tbf ([42496, 51712)): no overlap
    float av[8];
    const int r = tid >> 3, c0 = (tid & 7) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) av[i] = (c0 + i <= r) ? Asm[r * LDF64 + c0 + i] : 0.f;
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      *reinterpret_cast<uint32_t*>(Abf + r * LD64 + c0 + i) = pack_bf16(av[i], av[i + 1]);
      *reinterpret_cast<uint32_t*>(Tbf + r * LD64 + c0 + i) =
          pack_bf16(av[i] * ps.beta[c0 + i], av[i + 1] * ps.beta[c0 + i + 1]);
    }
  }
  bf16* dMs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DMS);
  __syncthreads();
  for (int idx = tid; idx < 64 * 8; idx += blockDim.x) {
    int r, cc;
    acc64n64_chunk(idx, r, cc);
    cp_async16(dMs + r * LD64 + cc * 8, P.dM + tix * TILE64N64_ELEMS + idx * 8, r < nv);
  }
  // the gate backward's per-channel vectors, so that the tail waits on no global load
  float* gbv = reinterpret_cast<float*>(smem + BwdIntraSmem::GB);
  if (tid < 32)
    cp_async16(gbv + 4 * tid, P.dGC + cidx * D + 4 * tid, true);
  else if (tid < 64)
    cp_async16(gbv + D + 4 * (tid - 32), P.in.dt_bias + (size_t)h * D + 4 * (tid - 32), true);
  else if (tid == 64)
    cp_async4(gbv + 2 * D, P.in.A_log + h);
  cp_async_commit();
  __syncthreads();

  float dq[4][4], dk[4][4], dG[4][4];
  // ---- WY backward and the state-side pieces --------------------------------
  {
    float acc[4][4];
    zero_acc<4>(acc);
    warp_mma_t<4, true, true>(acc, PadTile{Tbf, LD64}, m0, dEt, n0, 0, 64);  // dv = T^T dE
    // 16-byte runs per lane (quad transpose) instead of scattered 4-byte stores
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = pack_bf16(acc[j][e], acc[j][e + 1]);
      quad_transpose4(w);
      const int r = m0 + acc_row(e);
      if (r < nv)
        *reinterpret_cast<uint4*>(P.dv + ((size_t)(pos.t0 + r) * H + h) * D + n0 + 8 * (tid & 3)) =
            make_uint4(w[0], w[1], w[2], w[3]);
    }
    zero_acc<4>(acc);
    warp_mma_t<4, true, true>(acc, PadTile{Tbf, LD64}, m0, dWt, n0, 0, 64);  // dKe = T^T dW
    float colsum[4][2];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
        const int sw = (int)acc64_off(r, cc);
        float2 gq = unpack_bf16(*reinterpret_cast<const uint32_t*>(dQs + sw));
        float2 gk = unpack_bf16(*reinterpret_cast<const uint32_t*>(dKs + sw));
        float2 qa = unpack_bf16(*reinterpret_cast<const uint32_t*>(op.Qa + r * LD128 + cc));
        float2 kb = unpack_bf16(*reinterpret_cast<const uint32_t*>(op.Kb + r * LD128 + cc));
        float2 ke = unpack_bf16(*reinterpret_cast<const uint32_t*>(op.Ke + r * LD128 + cc));
        float2 er = *reinterpret_cast<const float2*>(op.er + I * D + cc);
        float2 ec = *reinterpret_cast<const float2*>(op.ec + I * D + cc);
        float qav[2] = {qa.x, qa.y}, kbv[2] = {kb.x, kb.y}, kev[2] = {ke.x, ke.y};
        float gqv[2] = {gq.x, gq.y}, gkv[2] = {gk.x, gk.y}, erv[2] = {er.x, er.y}, ecv[2] = {ec.x, ec.y};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float eg = af[j][e + u] * erv[u];
          float egc = bfv[j][e + u] * ecv[u];
          float dke = acc[j][e + u];
          dq[j][e + u] = gqv[u] * eg;
          dk[j][e + u] = dke * eg + gkv[u] * egc;
          float kbar = kbv[u] * ecv[u];
          float qt = qav[u] * erv[u];
          dG[j][e + u] = kev[u] * dke + qt * gqv[u] - kbar * gkv[u];
          if (e == 0) colsum[j][u] = kbar * gkv[u]; else colsum[j][u] += kbar * gkv[u];
        }
      }
    }
    // column sums of Kbar o dKbar over the chunk (lanes sharing a column differ in bits 2..4)
    float* cols = reinterpret_cast<float*>(smem + BwdIntraSmem::COLS);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float x = colsum[j][u];
        x += __shfl_xor_sync(0xffffffffu, x, 4);
        x += __shfl_xor_sync(0xffffffffu, x, 8);
        x += __shfl_xor_sync(0xffffffffu, x, 16);
        colsum[j][u] = x;
      }
    if ((tid & 31) < 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int u = 0; u < 2; ++u) cols[I * D + n0 + acc_col(j, u)] = colsum[j][u];
    }
  }
  // dT = dE V^T + dW Ke^T (64x64), warp tile rows m0, cols n1 (two n8 tiles)
  const int n1 = 16 * (warp >> 2);
  {
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma_t<2, false, false>(acc, dEt, m0, PadTile{op.V, LD128}, n1, 0, 128);
    warp_mma_t<2, false, false>(acc, dWt, m0, PadTile{op.Ke, LD128}, n1, 0, 128);
    // dbeta_T[j] = sum_i dT_ij A_ij ; dA = dT diag(beta)
    float cs[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float sum = 0.f;
#pragma unroll
        for (int e = u; e < 4; e += 2) {
          int r = m0 + acc_row(e), cc = n1 + acc_col(j, e);
          sum += acc[j][e] * __bfloat162float(Abf[r * LD64 + cc]);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        sum += __shfl_xor_sync(0xffffffffu, sum, 8);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        cs[j][u] = sum;
      }
    float* dbt = reinterpret_cast<float*>(smem + BwdIntraSmem::DBT);
    if ((tid & 31) < 4) {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int u = 0; u < 2; ++u) dbt[I * 64 + n1 + acc_col(j, u)] = cs[j][u];
    }
    __syncthreads();  // all reads of dE / dW are done
    bf16* dAs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DAS);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n1 + acc_col(j, e);
        *reinterpret_cast<uint32_t*>(dAs + r * LD64 + cc) =
            pack_bf16(acc[j][e] * ps.beta[cc], acc[j][e + 1] * ps.beta[cc + 1]);
      }
  }
  __syncthreads();
  // X = dA A^T ; dL = -A^T X (strictly lower)
  {
    bf16* dAs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DAS);
    bf16* Xs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::XS);
    float acc[2][4];
    zero_acc<2>(acc);
    warp_mma<2, false, false>(acc, dAs, LD64, m0, Abf, LD64, n1, 0, 64);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n1 + acc_col(j, e);
        *reinterpret_cast<uint32_t*>(Xs + r * LD64 + cc) = pack_bf16(acc[j][e], acc[j][e + 1]);
      }
    __syncthreads();
    zero_acc<2>(acc);
    warp_mma_neg<2, true, true>(acc, Abf, LD64, m0, Xs, LD64, n1, 0, 64);
    bf16* dLs = reinterpret_cast<bf16*>(smem + BwdIntraSmem::DLS);
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n1 + acc_col(j, e);
        float x0 = cc < r ? acc[j][e] : 0.f;
        float x1 = cc + 1 < r ? acc[j][e + 1] : 0.f;
        float2 lp = unpack_bf16(*reinterpret_cast<const uint32_t*>(Lpb + r * LD64 + cc));
        rs[e >> 1] += x0 * lp.x + x1 * lp.y;
        float br = ps.beta[r];
        *reinterpret_cast<uint32_t*>(dLs + r * LD64 + cc) = pack_bf16(x0 * br, x1 * br);
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
    }
    float* dbl = reinterpret_cast<float*>(smem + BwdIntraSmem::DBL);
    if ((tid & 3) == 0) {
      dbl[(warp >> 2) * 64 + m0 + acc_row(0)] = rs[0];
      dbl[(warp >> 2) * 64 + m0 + acc_row(2)] = rs[1];
    }
  }
  // the gate logits are needed again at the end: fetch them now (region free)
  bf16* gre = reinterpret_cast<bf16*>(smem + BwdIntraSmem::GRE);
  for (int i = tid; i < 64 * 16; i += blockDim.x) {
    int r = i >> 4, cc = i & 15;
    bool ok = r < nv;
    cp_async16(gre + r * D + cc * 8,
               P.in.g + (ok ? ((size_t)(pos.t0 + r) * H + h) * D + cc * 8 : 0), ok);
  }
  cp_async_commit();
  cp_async_wait<0>();  // dM and the gate logits
  __syncthreads();

  const bf16* dLs = reinterpret_cast<const bf16*>(smem + BwdIntraSmem::DLS);
  // ---- gradients through M (Aqk) and L' -------------------------------------
  // row side: rows of block I, reduction over j <= i
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    const bf16* dX = which == 0 ? dMs : dLs;
    const bf16* rowop = which == 0 ? op.Qa : op.Ka;
    float acc[4][4];
    zero_acc<4>(acc);
    {
      uint32_t a[4];
      load_A(a, dX, LD64, m0, 16 * I);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b[4];
        load_B_kn(b, op.Kd, LD128, n0 + 8 * j, 16 * I);
        mma16816(acc[j], a, b[0], b[1]);
        mma16816(acc[j + 1], a, b[2], b[3]);
      }
    }
    for (int J = 0; J < I; ++J) {
      float tmp[4][4];
      zero_acc<4>(tmp);
      uint32_t a[4];
      load_A(a, dX, LD64, m0, 16 * J);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b[4];
        load_B_kn(b, op.Kb, LD128, n0 + 8 * j, 16 * J);
        mma16816(tmp[j], a, b[0], b[1]);
        mma16816(tmp[j + 1], a, b[2], b[3]);
      }
      const float* cv = op.cvec + pair_index(I, J) * D;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 c2 = *reinterpret_cast<const float2*>(cv + n0 + acc_col(j, 0));
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] += ((e & 1) ? c2.y : c2.x) * tmp[j][e];
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
        float2 ro = unpack_bf16(*reinterpret_cast<const uint32_t*>(rowop + r * LD128 + cc));
        float rov[2] = {ro.x, ro.y};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float gval = acc[j][e + u];
          if (which == 0) dq[j][e + u] += af[j][e + u] * gval; else dk[j][e + u] += af[j][e + u] * gval;
          dG[j][e + u] += rov[u] * gval;
        }
      }
  }
  // column side: rows j of block I (as the column block), reduction over i >= j
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    const bf16* dX = which == 0 ? dMs : dLs;
    const bf16* rowop = which == 0 ? op.Qa : op.Ka;
    float acc[4][4];
    zero_acc<4>(acc);
    {
      uint32_t a[4];
      load_AT(a, dX, LD64, m0, 16 * I);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        uint32_t b[4];
        load_B_kn(b, rowop, LD128, n0 + 8 * j, 16 * I);
        mma16816(acc[j], a, b[0], b[1]);
        mma16816(acc[j + 1], a, b[2], b[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
        float2 kd = unpack_bf16(*reinterpret_cast<const uint32_t*>(op.Kd + r * LD128 + cc));
        float kdv[2] = {kd.x, kd.y};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          float ia = rcp(af[j][e + u]);
          dk[j][e + u] += ia * acc[j][e + u];
          dG[j][e + u] -= kdv[u] * acc[j][e + u];
        }
      }
    if (I < 3) {
      zero_acc<4>(acc);
      for (int Ib = I + 1; Ib < 4; ++Ib) {
        float tmp[4][4];
        zero_acc<4>(tmp);
        uint32_t a[4];
        load_AT(a, dX, LD64, m0, 16 * Ib);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
          uint32_t b[4];
          load_B_kn(b, rowop, LD128, n0 + 8 * j, 16 * Ib);
          mma16816(tmp[j], a, b[0], b[1]);
          mma16816(tmp[j + 1], a, b[2], b[3]);
        }
        const float* cv = op.cvec + pair_index(Ib, I) * D;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 c2 = *reinterpret_cast<const float2*>(cv + n0 + acc_col(j, 0));
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][e] += ((e & 1) ? c2.y : c2.x) * tmp[j][e];
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
          float2 kb = unpack_bf16(*reinterpret_cast<const uint32_t*>(op.Kb + r * LD128 + cc));
          float kbv[2] = {kb.x, kb.y};
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            dk[j][e + u] += bfv[j][e + u] * acc[j][e + u];
            dG[j][e + u] -= kbv[u] * acc[j][e + u];
          }
        }
    }
  }
  // ---- outputs ---------------------------------------------------------------
#pragma unroll
  for (int e = 0; e < 4; e += 2) {
    uint32_t wq[4], wk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wq[j] = pack_bf16(dq[j][e], dq[j][e + 1]);
      wk[j] = pack_bf16(dk[j][e], dk[j][e + 1]);
    }
    quad_transpose4(wq);
    quad_transpose4(wk);
    const int r = m0 + acc_row(e);
    if (r < nv) {
      const size_t off = ((size_t)(pos.t0 + r) * H + h) * D + n0 + 8 * (tid & 3);
      *reinterpret_cast<uint4*>(P.dq_hat + off) = make_uint4(wq[0], wq[1], wq[2], wq[3]);
      *reinterpret_cast<uint4*>(P.dk_hat + off) = make_uint4(wk[0], wk[1], wk[2], wk[3]);
    }
  }
  const float* cols = reinterpret_cast<const float*>(smem + BwdIntraSmem::COLS);
  float* dGs = ps.gam;  // Gam is dead: every decay factor is in registers
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      int r = m0 + acc_row(e), cc = n0 + acc_col(j, e);
      *reinterpret_cast<float2*>(dGs + r * LDG + cc) = make_float2(dG[j][e], dG[j][e + 1]);
    }
  __syncthreads();
  // reverse cumsum over the chunk and the gate backward: thread (part, col)
  // with col = tid % 128 owns rows 16*part .. 16*part+15 of one channel
  {
    const int col = tid & 127, part = tid >> 7;
    float own = 0.f;
#pragma unroll 4
    for (int r = 16 * part; r < 16 * part + 16; ++r) own += dGs[r * LDG + col];
    float* partsum = reinterpret_cast<float*>(smem + BwdIntraSmem::DAS);  // 4 x 128 fp32 (dA is dead)
    partsum[part * D + col] = own;
    __syncthreads();
    float run = gbv[col] + cols[col] + cols[D + col] + cols[2 * D + col] + cols[3 * D + col];
    for (int p2 = part + 1; p2 < 4; ++p2) run += partsum[p2 * D + col];
    const float eA = __expf(gbv[2 * D]);
    const float bias = gbv[D + col];
    float sA = 0.f, sB = 0.f;
    for (int r = 16 * part + 15; r >= 16 * part; --r) {
      run += dGs[r * LDG + col];
      if (r < nv) {
        size_t off = ((size_t)(pos.t0 + r) * H + h) * D + col;
        float x = __bfloat162float(gre[r * D + col]) + bias;
        float z = eA * x;
        float sg = sigmoidf_(z);
        float dz = run * P.in.lower_bound * sg * (1.f - sg);
        float dx = dz * eA;
        P.dg[off] = __float2bfloat16(dx);
        sA += dz * z;
        sB += dx;
      }
    }
    __syncthreads();
    partsum[part * D + col] = sA;
    partsum[4 * D + part * D + col] = sB;
    __syncthreads();
    if (part == 0) {
      P.partA[cidx * D + col] = partsum[col] + partsum[D + col] + partsum[2 * D + col] + partsum[3 * D + col];
      P.partB[cidx * D + col] = partsum[4 * D + col] + partsum[5 * D + col] + partsum[6 * D + col] +
                                partsum[7 * D + col];
    }
  }
  if (tid < 64) {
    int r = tid;
    if (r < nv) {
      const float* dbt = reinterpret_cast<const float*>(smem + BwdIntraSmem::DBT);
      const float* dbl = reinterpret_cast<const float*>(smem + BwdIntraSmem::DBL);
      float db = dbt[r] + dbt[64 + r] + dbt[128 + r] + dbt[192 + r] + dbl[r] + dbl[64 + r] + dbl[128 + r] +
                 dbl[192 + r];
      float bt = ps.beta[r];
      P.dbeta[(size_t)(pos.t0 + r) * H + h] = __float2bfloat16(db * bt * (1.f - bt));
    }
  }
}

}  // namespace kda
