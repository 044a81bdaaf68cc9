// Forward kernels of the chunked KDA layer.
//
//   kda_fwd_intra_kernel  (persistent: one CTA per SM walks the (chunk slot, head)
//                          items, slot fastest: item b first, then items from a
//                          shared counter; the next item's inputs are prefetched)
//       raw q/k/v (pre- or post-conv), gate and beta logits
//       -> W = T (k*2^Gam), U = T v, Qt = q*2^Gam, Kbar = k*2^(Gam_C-Gam),
//          M = Aqk (lower incl. diag), dC = 2^Gam_C
//       with T = (I + diag(beta) L')^-1 diag(beta).
// The state pass that consumes these (E = U - W S, O = Qt S + M E,
// S <- diag(dC) S + Kbar^T E) runs on the tensor cores: kda_fwd_state_tc.cuh.
#pragma once

#include "kda_intra.cuh"
#include "kda_tc.cuh"

namespace kda {

struct FwdIntraParams {
  PrologueIn in;
  SeqInfo seq;
  bool conv;
  bf16 *W, *U, *Qt, *Kb, *M;  // [T_total][H][128] (M: [T_total][H][64])
  float* dC;                  // [chunks][H][128]
  bf16* A;                    // [slots x H] 64x64 bf16 tiles of A = (I + diag(beta) L')^-1 (swizzled), or null
  bf16* LP;                   // [slots x H] 64x64 bf16 tiles of L' (swizzled), with A
  bf16 *QN, *KN, *VN;         // [slots x H] prologue products for the backward, or null
  float *GM, *BT;
  int grid_chunks;            // chunk slots per head: items are (slot, head), slot fastest
  int* item_counter;          // zero at launch: items from gridDim.x on are handed out by it
  CUtensorMap maps[4];        // q, k, v, g as [T_total][H][128] bf16; boxes of 67 (q/k/v) and 64 (g) rows
  uint32_t wait_polls;        // poll limit of the wait for an item's prefetched inputs
};

// Shared-memory layout of the forward intra kernel (bytes).  The raw inputs,
// taps and biases have regions of their own, so that the next item's loads can
// land while the current item's products and inverse are computed.  The
// tcgen05 operand tiles come first (1 KB aligned, 128B-swizzled).
struct IntraSmem {
  static constexpr int KQ = 0;                          // [Ka; Qa] 128 x 128 bf16 (cumsum scratch before)
  static constexpr int KC = KQ + 32768;                 // [Kc_0; ..; Kc_3] 160 x 128 bf16
  static constexpr int KE = KC + KC_BYTES;              // Ke, then V: 64 x 128 bf16 each
  static constexpr int RAW = KE + 32768;                // 3 x 67 x 128 bf16 (then the saved q/k/v tiles)
  static constexpr int GRAW = RAW + 3 * 67 * D * 2;     // 64 x 128 bf16
  static constexpr int GAM = GRAW + 64 * D * 2;         // 64 x LDG fp32
  static constexpr int BETA = GAM + 64 * LDG * 4;       // 64 fp32
  static constexpr int BRAW = BETA + 64 * 4;            // 64 bf16
  static constexpr int TAPS = BRAW + 64 * 2;            // 3 x 128 x 4 fp32
  static constexpr int BIAS = TAPS + 3 * D * 16;        // dt_bias [128], A_log, padding
  static constexpr int NXT = BIAS + (D + 4) * 4;        // next item: index, bos, t0, t1; then the mbarriers
                                                        // of the raw rows, the L'/M and the W/U products
                                                        // (offsets 16, 24, 32) and the TMEM slot (40)
  static constexpr int XTMP = NXT + 64;                 // 3 warps x 16 x 17 fp32
  static constexpr int END = XTMP + 3 * 16 * 17 * 4;
  // aliases valid once the operands are built and the product stores completed
  static constexpr int LP = GAM;                        // 64 x LDF64 fp32
  static constexpr int AINV = LP + 64 * LDF64 * 4;      // 64 x LDF64 fp32
  // aliases valid once the L'/M products completed (the Kc tiles are dead)
  static constexpr int TT = KC;                         // T = A diag(beta), 64 x 64 bf16 swizzled
  static constexpr int ASW = KC + 8192;                 // A for the backward, 64 x 64 bf16 swizzled
  static constexpr int LSW = KC + 16384;                // L' for the backward, 64 x 64 bf16 swizzled
  static_assert(AINV + 64 * LDF64 * 4 <= BETA, "the inverse tiles overflow the decay tile");
  static_assert(LSW + 8192 <= KE, "T, A and L' overflow the Kc tiles");
  static_assert(KC % 1024 == 0 && KE % 1024 == 0 && (KC_BYTES / 2) % 1024 == 0, "swizzled operand atoms");
  static_assert(RAW % 16 == 0 && GAM % 16 == 0 && BETA % 16 == 0 && AINV % 16 == 0 && TAPS % 16 == 0 &&
                    BIAS % 16 == 0 && NXT % 8 == 0 && 3 * 64 * D * 2 <= GRAW - RAW,
                "bulk-copy, cp.async and mbarrier targets");
  static_assert(16 * D * 4 <= KC - KQ, "cumsum scratch overflows the operand tile");
  static_assert((RAW + 67 * D * 2) % 128 == 0 && (RAW + 2 * 67 * D * 2) % 128 == 0 && GRAW % 128 == 0 &&
                    RAW % 128 == 0,
                "tiled TMA destinations");
  static_assert(END <= 232448, "shared memory");
};

// TMEM columns of the forward chunk kernel: the L'/M accumulator (M = 128,
// N = 160; row block I reads columns kc_row(I) .. kc_row(I) + 16 I + 15) at 0;
// W and U (M = 64, N = 128, at lane offsets 0 and 16) at WU_COL.
constexpr uint32_t WU_COL = 256;

// The CTA's next valid item from the shared counter (items below gridDim.x belong to
// the CTA of that index), or n_items when none is left.  Dynamic: a CTA that starts
// late (its SM busy with another kernel, e.g. a collective) simply takes fewer items.
__device__ __forceinline__ int grab_item(const FwdIntraParams& P, int n_items, int G, ChunkPos& pos) {
  for (;;) {
    const int it = (int)gridDim.x + atomicAdd(P.item_counter, 1);
    if (it >= n_items) return n_items;
    pos = chunk_pos(P.seq, it % G);
    if (pos.valid) return it;
  }
}

__global__ void __launch_bounds__(INTRA_THREADS, 1) kda_fwd_intra_kernel(const __grid_constant__ FwdIntraParams P) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const int H = P.in.H, G = P.grid_chunks, n_items = G * H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int* nxt = reinterpret_cast<int*>(smem + IntraSmem::NXT);
  ChunkPos pos = chunk_pos(P.seq, blockIdx.x % G);
  int item = blockIdx.x;
  if (!pos.valid) {  // block-uniform: one thread grabs, all read
    if (tid == 0) {
      ChunkPos p0;
      nxt[0] = grab_item(P, n_items, G, p0);
    }
    __syncthreads();
    item = nxt[0];
    if (item >= n_items) return;
    pos = chunk_pos(P.seq, item % G);
    __syncthreads();  // nxt is rewritten below
  }
  if (smem_u32(smem) & 1023) {  // swizzled operand tiles need 1 KB alignment (block-uniform)
    if (tid == 0) atomicExch(&g_kda_device_error, 9);
    return;
  }

  PrologueSmem ps;
  ps.xq = reinterpret_cast<bf16*>(smem + IntraSmem::RAW);
  ps.xk = ps.xq + 67 * D;
  ps.xv = ps.xk + 67 * D;
  ps.graw = reinterpret_cast<bf16*>(smem + IntraSmem::GRAW);
  ps.braw = reinterpret_cast<bf16*>(smem + IntraSmem::BRAW);
  ps.gam = reinterpret_cast<float*>(smem + IntraSmem::GAM);
  ps.beta = reinterpret_cast<float*>(smem + IntraSmem::BETA);
  ps.tot = reinterpret_cast<float*>(smem + IntraSmem::KQ);  // scratch, before the operands
  ps.taps = reinterpret_cast<float*>(smem + IntraSmem::TAPS);
  ps.bias = reinterpret_cast<float*>(smem + IntraSmem::BIAS);
  uint64_t* raw_ready = reinterpret_cast<uint64_t*>(smem + IntraSmem::NXT + 16);
  uint64_t* mb_lm = raw_ready + 1;
  uint64_t* mb_wu = raw_ready + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(raw_ready + 3);
  const bool save_products = P.QN != nullptr;
  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    tc::mbar_init(raw_ready, 1);
    tc::mbar_init(mb_lm, 1);
    tc::mbar_init(mb_wu, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t sb = smem_u32(smem);
  // K-major and MN-major descriptors from a base: the address field (bits 0-13,
  // address / 16) plus the operand's byte offset / 16
  const uint64_t kbase = tc::smem_desc(sb, 16, 1024), mbase = tc::smem_desc(sb, 8192, 1024);
  const uint32_t idLM = tc::idesc_bf16(128, KC_ROWS, false, false);  // [Ka; Qa] x Kc^T, both K-major
  const uint32_t idWU = tc::idesc_bf16(64, 128, false, true);        // A = T K-major, B = Ke / V MN-major

  bf16 braw = prologue_issue_loads(P.in, ps, pos, item / G, P.conv, raw_ready, P.maps);
  cp_async_commit();
  uint32_t raw_phase = 0, mma_phase = 0;
  for (;;) {
    const int c = item % G, h = item / G;
    const int nvalid = pos.t1 - pos.t0;
    if (tid == 0) {
      // the next item (its table lookups overlap this item's loads)
      ChunkPos np;
      nxt[0] = grab_item(P, n_items, G, np);
      nxt[1] = np.bos; nxt[2] = np.t0; nxt[3] = np.t1;
      // the previous item's A / L' stores read the Kc region the operands are rebuilt in
      if (P.A) tc::bulk_wait_read_all();
    }
    const bool arrived = tc::mbar_wait(raw_ready, raw_phase, P.wait_polls);
    if (P.conv) zero_foreign_halo(ps, pos);
    cp_async_wait<0>();
    if (tid >= LOADER_T0) ps.braw[tid - LOADER_T0] = braw;
    if (__syncthreads_or(!arrived)) {
      // this item's inputs did not arrive in time: record it, let the copies in
      // flight land (bounded wait) and leave without touching another item
      if (tid == 0) atomicExch(&g_kda_device_error, 8);
      tc::mbar_wait(raw_ready, raw_phase);
      break;
    }
    raw_phase ^= 1u;

    Strip s;
    prologue_compute(P.in, ps, pos, P.conv, s);
    // the prologue's products, so that the backward need not redo it: q, k, v
    // strips into [64][128] tiles over the dead raw inputs, then (with the decay
    // cumsum tile and beta, already in shared memory) five bulk stores issued by
    // one thread; they complete while the operands are built
    if (save_products) {
      const int tg = tid >> 4, cg = tid & 15;
      bf16* tq = reinterpret_cast<bf16*>(smem + IntraSmem::RAW);
#pragma unroll
      for (int r = 0; r < STRIP; ++r) {
        const int t = STRIP * tg + r;
        const uint32_t so = sw64_chunk(t, cg);  // the backward's tcgen05 operand layout
        *reinterpret_cast<bf16x8*>(tq + so) = pack8(s.q[r]);
        *reinterpret_cast<bf16x8*>(tq + TILE64_ELEMS + so) = pack8(s.k[r]);
        *reinterpret_cast<bf16x8*>(tq + 2 * TILE64_ELEMS + so) = pack8(s.v[r]);
      }
      tc::fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        const size_t tix = tile_index(P.seq, c, h);
        constexpr uint32_t TB = TILE64_ELEMS * 2;
        tc::bulk_s2g(P.QN + tix * TILE64_ELEMS, tq, TB);
        tc::bulk_s2g(P.KN + tix * TILE64_ELEMS, tq + TILE64_ELEMS, TB);
        tc::bulk_s2g(P.VN + tix * TILE64_ELEMS, tq + 2 * TILE64_ELEMS, TB);
        tc::bulk_s2g(P.GM + tix * 64 * LDG, ps.gam, 64 * LDG * 4);
        tc::bulk_s2g(P.BT + tix * 64, ps.beta, 64 * 4);
        tc::bulk_commit();
      }
    }

    build_tc_operands(s, ps.gam, smem + IntraSmem::KQ, smem + IntraSmem::KC, smem + IntraSmem::KE, P.Qt, P.Kb,
                      pos.t0, nvalid, H, h);
    if (tid < D) P.dC[((size_t)c * H + h) * D + tid] = ex2(ps.gam[63 * LDG + tid]);
    if (save_products && tid == 0) tc::bulk_wait_read_all();  // the raw region is reused from here on
    tc::fence_async_smem();  // operand tiles -> tensor cores; raw rows -> the next item's bulk copies
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 32) {
      // L' and M: [Ka; Qa] (M = 128) x [Kc_0; ..; Kc_3] (N = 160)
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a = kbase + (uint64_t)((IntraSmem::KQ + (ks >> 2) * 16384 + (ks & 3) * 32) >> 4);
        const uint64_t b = kbase + (uint64_t)((IntraSmem::KC + (ks >> 2) * (KC_BYTES / 2) + (ks & 3) * 32) >> 4);
        tc::mma_bf16(tbase, a, b, idLM, ks > 0);
      }
      tc::mma_commit(mb_lm);
    }
    // the next item's inputs stream in while this one's products are computed
    const int next = nxt[0];
    ChunkPos npos;
    npos.valid = next < n_items;
    npos.bos = nxt[1]; npos.t0 = nxt[2]; npos.t1 = nxt[3];
    if (npos.valid) braw = prologue_issue_loads(P.in, ps, npos, next / G, P.conv, raw_ready, P.maps);
    cp_async_commit();

    float* Lp = reinterpret_cast<float*>(smem + IntraSmem::LP);
    float* Ainv = reinterpret_cast<float*>(smem + IntraSmem::AINV);
    float* xtmp = reinterpret_cast<float*>(smem + IntraSmem::XTMP);
    if (__syncthreads_or(!tc::mbar_wait(mb_lm, mma_phase))) {
      // the products did not complete in time: record it, let them (and the
      // next item's copies) land, bounded, and leave
      if (tid == 0) atomicExch(&g_kda_device_error, 10);
      tc::mbar_wait(mb_lm, mma_phase);
      if (npos.valid) tc::mbar_wait(raw_ready, raw_phase);
      break;
    }
    tc::fence_after_sync();
    // L' and M out of TMEM (row i of [Ka; Qa] in lane i): warp quarter q holds
    // rows 32 q .. 32 q + 31 (L' for q < 2, M for q >= 2), warp w / 4 = kb the
    // columns 16 kb .. 16 kb + 15 of those rows (zero above the row's block)
    {
      const int q = warp & 3, kb = warp >> 2;
      const int Ia = 2 * (q & 1), Ib = Ia + 1, I = lane < 16 ? Ia : Ib;
      const int i = 32 * (q & 1) + lane;
      const uint32_t trow = tbase + ((uint32_t)(32 * q) << 16);
      const bool has = kb <= I, lower = q < 2;
      float x[16], t16[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = 0.f;
      if (kb <= Ia) {  // warp-uniform: the block of lanes 0-15
        tc::tmem_ld16(trow + kc_row(Ia) + 16 * kb, t16);
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = lane < 16 ? t16[e] : x[e];
      }
      if (kb <= Ib) {  // the block of lanes 16-31
        tc::tmem_ld16(trow + kc_row(Ib) + 16 * kb, t16);
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = lane < 16 ? x[e] : t16[e];
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = 16 * kb + e;
        if (!(has && (lower ? j < i : j <= i))) x[e] = 0.f;
      }
      if (lower) {
#pragma unroll
        for (int e = 0; e < 16; ++e) Lp[i * LDF64 + 16 * kb + e] = x[e];
        if (P.A) {
          float x0[8], x1[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) { x0[e] = x[e]; x1[e] = x[8 + e]; }
          bf16* lsw = reinterpret_cast<bf16*>(smem + IntraSmem::LSW);
          *reinterpret_cast<bf16x8*>(lsw + sw64_chunk(i, 2 * kb)) = pack8(x0);
          *reinterpret_cast<bf16x8*>(lsw + sw64_chunk(i, 2 * kb + 1)) = pack8(x1);
        }
      } else if (i < nvalid) {
        uint4* dst = reinterpret_cast<uint4*>(P.M + ((size_t)(pos.t0 + i) * H + h) * 64 + 16 * kb);
        dst[0] = make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]),
                            pack_bf16(x[6], x[7]));
        dst[1] = make_uint4(pack_bf16(x[8], x[9]), pack_bf16(x[10], x[11]), pack_bf16(x[12], x[13]),
                            pack_bf16(x[14], x[15]));
      }
    }
    __syncthreads();
    if (warp < 2) tri_inverse_diag(Lp, ps.beta, Ainv);
    __syncthreads();
    tri_inverse_offdiag(Lp, ps.beta, Ainv, xtmp);
    // T = A diag(beta) (the W/U operand) and A for the backward, as bf16 tiles in
    // the tcgen05 operand layout (A's strictly-upper part is not stored: zeros)
    {
      bf16* tsw = reinterpret_cast<bf16*>(smem + IntraSmem::TT);
      bf16* asw = reinterpret_cast<bf16*>(smem + IntraSmem::ASW);
      for (int i2 = tid; i2 < 64 * 8; i2 += blockDim.x) {
        const int r = i2 >> 3, c8 = i2 & 7;
        float av[8], tv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int cc = 8 * c8 + u;
          av[u] = cc <= r ? Ainv[r * LDF64 + cc] : 0.f;
          tv[u] = av[u] * ps.beta[cc];
        }
        *reinterpret_cast<bf16x8*>(tsw + sw64_chunk(r, c8)) = pack8(tv);
        if (P.A) *reinterpret_cast<bf16x8*>(asw + sw64_chunk(r, c8)) = pack8(av);
      }
    }
    tc::fence_async_smem();  // T -> tensor cores; A and L' -> the bulk stores
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 32) {
      // W = T Ke (lanes 0-15 of each quarter), U = T V (lanes 16-31): M = 64, N = 128
      tc::fence_after_sync();
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint64_t a = kbase + (uint64_t)((IntraSmem::TT + 32 * ks) >> 4);
        tc::mma_bf16(tbase + WU_COL, a, mbase + (uint64_t)((IntraSmem::KE + ks * 2048) >> 4), idWU, ks > 0);
        tc::mma_bf16(tbase + (16u << 16) + WU_COL, a, mbase + (uint64_t)((IntraSmem::KE + 16384 + ks * 2048) >> 4),
                     idWU, ks > 0);
      }
      tc::mma_commit(mb_wu);
    }
    // A and L' for the backward: one bulk store each, completed before the
    // operand tiles are rebuilt
    if (P.A && tid == 0) {
      const size_t tix = tile_index(P.seq, c, h);
      tc::bulk_s2g(P.A + tix * TILE64N64_ELEMS, smem + IntraSmem::ASW, TILE64N64_ELEMS * 2);
      tc::bulk_s2g(P.LP + tix * TILE64N64_ELEMS, smem + IntraSmem::LSW, TILE64N64_ELEMS * 2);
      tc::bulk_commit();
    }
    if (__syncthreads_or(!tc::mbar_wait(mb_wu, mma_phase))) {
      if (tid == 0) atomicExch(&g_kda_device_error, 10);
      tc::mbar_wait(mb_wu, mma_phase);
      if (npos.valid) tc::mbar_wait(raw_ready, raw_phase);
      break;
    }
    tc::fence_after_sync();
    mma_phase ^= 1u;
    // W and U out of TMEM: warp quarter s holds rows 16 s .. 16 s + 15 (lane & 15)
    // of W (lanes 0-15) and U (lanes 16-31); warp w / 4 = qd the channels 32 qd ..
    {
      const int sq = warp & 3, qd = warp >> 2;
      const int r = 16 * sq + (lane & 15);
      float acc[32];
      tc::tmem_ld32(tbase + ((uint32_t)(32 * sq) << 16) + WU_COL + 32 * qd, acc);
      if (r < nvalid) {
        bf16* dst = (lane < 16 ? P.W : P.U) + ((size_t)(pos.t0 + r) * H + h) * D + 32 * qd;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
          *reinterpret_cast<uint4*>(dst + 8 * c4) =
              make_uint4(pack_bf16(acc[8 * c4 + 0], acc[8 * c4 + 1]), pack_bf16(acc[8 * c4 + 2], acc[8 * c4 + 3]),
                         pack_bf16(acc[8 * c4 + 4], acc[8 * c4 + 5]), pack_bf16(acc[8 * c4 + 6], acc[8 * c4 + 7]));
      }
    }
    tc::fence_before_sync();
    if (next >= n_items) break;
    item = next;
    pos = npos;
  }
  cp_async_wait<0>();
  if (tid == 0) tc::bulk_wait_all();  // the bulk stores read shared memory
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------- state pass
struct FwdStateParams {
  SeqInfo seq;
  int H;
  const bf16 *W, *U, *Qt, *Kb, *M;
  const float* dC;
  const float* h0;       // [N][H][128][128] or null
  bf16* o;               // [T_total][H][128]
  bf16* hs;              // [chunks][H] chunk-start states (128B-swizzled bf16 operand tiles), or null
  bf16* E;               // [chunks][H] v_new (128B-swizzled bf16 operand tiles, rows past the end zero), or null
  float* ht;             // [N][H][128][128] or null
  // W, Qt, Kbar, U as [T_total][H][128] and M as [T_total][H][64] bf16, for
  // 128B-swizzled TMA boxes of 64 channels x 64 rows (one operand atom each)
  CUtensorMap maps[5];
  uint32_t wait_polls;   // poll limit of the consumers' wait for a chunk's operands
  int withhold_loads;    // test hook: the producer issues nothing (that wait runs out)
};

__device__ __forceinline__ void load_vec128(float* dst, const float* src) {
  for (int i = threadIdx.x; i < 32; i += blockDim.x) cp_async16(dst + 4 * i, src + 4 * i, true);
}

}  // namespace kda
