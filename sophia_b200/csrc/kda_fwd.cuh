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
// land while the current item's blocks and inverse are computed.
struct IntraSmem {
  static constexpr int RAW = 0;                         // 3 x 67 x 128 bf16 (then the q/k/v product tiles)
  static constexpr int GRAW = RAW + 3 * 67 * D * 2;     // 64 x 128 bf16
  static constexpr int GAM = GRAW + 64 * D * 2;         // 64 x LDG fp32
  static constexpr int OPS = GAM + 64 * LDG * 4;        // 6 x 64 x LD128 bf16 (cumsum scratch before)
  static constexpr int OPSZ = 64 * LD128 * 2;
  static constexpr int CVEC = OPS + 6 * OPSZ;           // 6 x 128 fp32
  static constexpr int BETA = CVEC + 6 * D * 4;         // 64 fp32
  static constexpr int BRAW = BETA + 64 * 4;            // 64 bf16
  static constexpr int TAPS = BRAW + 64 * 2;            // 3 x 128 x 4 fp32
  static constexpr int BIAS = TAPS + 3 * D * 16;        // dt_bias [128], A_log, padding
  static constexpr int NXT = BIAS + (D + 4) * 4;        // next item: index, bos, t0, t1; then the
                                                        // mbarrier of the raw rows (offset 16)
  static constexpr int XTMP = NXT + 32;                 // 3 warps x 16 x 17 fp32
  static constexpr int TBF = XTMP + 3 * 16 * 17 * 4;    // 64 x LD64 bf16
  static constexpr int END = TBF + 64 * LD64 * 2;
  // aliases valid once the operands are built and the product stores completed
  static constexpr int LP = GAM;                        // 64 x LDF64 fp32
  static constexpr int AINV = LP + 64 * LDF64 * 4;      // 64 x LDF64 fp32
  static constexpr int MSM = OPS + OPSZ;                // 64 x LD64 bf16 over Ka (dead once L' is formed)
  static_assert(AINV + 64 * LDF64 * 4 <= OPS, "the inverse tiles overflow the decay tile");
  static_assert(RAW % 16 == 0 && GAM % 16 == 0 && BETA % 16 == 0 && AINV % 16 == 0 && TAPS % 16 == 0 &&
                    BIAS % 16 == 0 && 3 * 64 * D * 2 <= GRAW,
                "bulk-copy and cp.async targets");
  static_assert(64 * LD64 * 2 <= OPSZ && 16 * D * 4 <= OPSZ, "M staging or cumsum scratch overflows a tile");
  static_assert((RAW + 67 * D * 2) % 128 == 0 && (RAW + 2 * 67 * D * 2) % 128 == 0 && GRAW % 128 == 0,
                "tiled TMA destinations");
  static_assert(END <= 232448, "shared memory");
};

__device__ __forceinline__ void store_rows64(bf16* gdst, const bf16* s, int ld, int nrows, int H, int h, int t0) {
  for (int i = threadIdx.x; i < nrows * 8; i += blockDim.x) {
    int r = i >> 3, cc = i & 7;
    bf16x8 v = *reinterpret_cast<const bf16x8*>(s + r * ld + cc * 8);
    *reinterpret_cast<bf16x8*>(gdst + ((size_t)(t0 + r) * H + h) * 64 + cc * 8) = v;
  }
}

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
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = P.in.H, G = P.grid_chunks, n_items = G * H;
  int* nxt = reinterpret_cast<int*>(smem + IntraSmem::NXT);
  ChunkPos pos = chunk_pos(P.seq, blockIdx.x % G);
  int item = blockIdx.x;
  if (!pos.valid) {  // block-uniform: one thread grabs, all read
    if (threadIdx.x == 0) {
      ChunkPos p0;
      nxt[0] = grab_item(P, n_items, G, p0);
    }
    __syncthreads();
    item = nxt[0];
    if (item >= n_items) return;
    pos = chunk_pos(P.seq, item % G);
    __syncthreads();  // nxt is rewritten below
  }

  PrologueSmem ps;
  ps.xq = reinterpret_cast<bf16*>(smem + IntraSmem::RAW);
  ps.xk = ps.xq + 67 * D;
  ps.xv = ps.xk + 67 * D;
  ps.graw = reinterpret_cast<bf16*>(smem + IntraSmem::GRAW);
  ps.braw = reinterpret_cast<bf16*>(smem + IntraSmem::BRAW);
  ps.gam = reinterpret_cast<float*>(smem + IntraSmem::GAM);
  ps.beta = reinterpret_cast<float*>(smem + IntraSmem::BETA);
  ps.tot = reinterpret_cast<float*>(smem + IntraSmem::OPS);  // scratch, before operands
  ps.taps = reinterpret_cast<float*>(smem + IntraSmem::TAPS);
  ps.bias = reinterpret_cast<float*>(smem + IntraSmem::BIAS);
  uint64_t* raw_ready = reinterpret_cast<uint64_t*>(smem + IntraSmem::NXT + 16);
  const bool save_products = P.QN != nullptr;
  if (threadIdx.x == 0) {
    tc::mbar_init(raw_ready, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();

  bf16 braw = prologue_issue_loads(P.in, ps, pos, item / G, P.conv, raw_ready, P.maps);
  cp_async_commit();
  uint32_t raw_phase = 0;
  for (;;) {
    const int c = item % G, h = item / G;
    const int nvalid = pos.t1 - pos.t0;
    if (threadIdx.x == 0) {
      // the next item (its table lookups overlap this item's loads)
      ChunkPos np;
      nxt[0] = grab_item(P, n_items, G, np);
      nxt[1] = np.bos; nxt[2] = np.t0; nxt[3] = np.t1;
      // the previous item's A store reads the region the decay tile is rebuilt in
      if (P.A) tc::bulk_wait_read_all();
    }
    const bool arrived = tc::mbar_wait(raw_ready, raw_phase, P.wait_polls);
    if (P.conv) zero_foreign_halo(ps, pos);
    cp_async_wait<0>();
    if (threadIdx.x >= LOADER_T0) ps.braw[threadIdx.x - LOADER_T0] = braw;
    if (__syncthreads_or(!arrived)) {
      // this item's inputs did not arrive in time: record it, let the copies in
      // flight land (bounded wait) and leave without touching another item
      if (threadIdx.x == 0) atomicExch(&g_kda_device_error, 8);
      tc::mbar_wait(raw_ready, raw_phase);
      if (threadIdx.x == 0) tc::bulk_wait_all();
      __syncthreads();
      return;
    }
    raw_phase ^= 1u;

    Strip s;
    prologue_compute(P.in, ps, pos, P.conv, s);
    // the prologue's products, so that the backward need not redo it: q, k, v
    // strips into [64][128] tiles over the dead raw inputs, then (with the decay
    // cumsum tile and beta, already in shared memory) five bulk stores issued by
    // one thread; they complete while the operands are built
    if (save_products) {
      const int tg = threadIdx.x >> 4, cg = threadIdx.x & 15;
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
      if (threadIdx.x == 0) {
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

    Operands op;
    op.Qa = reinterpret_cast<bf16*>(smem + IntraSmem::OPS);
    op.Ka = op.Qa + 64 * LD128;
    op.Kd = op.Ka + 64 * LD128;
    op.Kb = op.Kd + 64 * LD128;
    op.V = op.Kb + 64 * LD128;
    op.Ke = op.V + 64 * LD128;
    op.cvec = reinterpret_cast<float*>(smem + IntraSmem::CVEC);
    op.er = nullptr;
    op.ec = nullptr;
    {
      float qt[STRIP][8], kbar[STRIP][8];
      build_operands<true>(s, ps.gam, op, qt, kbar);
      const int tg = threadIdx.x >> 4, cg = threadIdx.x & 15;
#pragma unroll
      for (int r = 0; r < STRIP; ++r) {
        int t = STRIP * tg + r;
        if (t < nvalid) {
          size_t off = ((size_t)(pos.t0 + t) * H + h) * D + 8 * cg;
          *reinterpret_cast<bf16x8*>(P.Qt + off) = pack8(qt[r]);
          *reinterpret_cast<bf16x8*>(P.Kb + off) = pack8(kbar[r]);
        }
      }
      if (threadIdx.x < D)
        P.dC[((size_t)c * H + h) * D + threadIdx.x] = ex2(ps.gam[63 * LDG + threadIdx.x]);
    }
    if (save_products && threadIdx.x == 0) tc::bulk_wait_read_all();  // the raw region is reused from here on
    tc::fence_async_smem();  // this item's generic accesses of the raw rows precede the next item's bulk copies
    __syncthreads();
    // the next item's inputs stream in while this one's blocks are computed
    const int next = nxt[0];
    ChunkPos npos;
    npos.valid = next < n_items;
    npos.bos = nxt[1]; npos.t0 = nxt[2]; npos.t1 = nxt[3];
    if (npos.valid) braw = prologue_issue_loads(P.in, ps, npos, next / G, P.conv, raw_ready, P.maps);
    cp_async_commit();

    float* Lp = reinterpret_cast<float*>(smem + IntraSmem::LP);
    float* Ainv = reinterpret_cast<float*>(smem + IntraSmem::AINV);
    float* xtmp = reinterpret_cast<float*>(smem + IntraSmem::XTMP);
    bf16* Tbf = reinterpret_cast<bf16*>(smem + IntraSmem::TBF);
    bf16* Msm = reinterpret_cast<bf16*>(smem + IntraSmem::MSM);
    l_blocks(op, Lp);
    __syncthreads();
    // the diagonal inverse (warps 0-1) overlaps the M blocks (warps 4-15)
    {
      const int warp = threadIdx.x >> 5;
      if (warp < 2) {
        tri_inverse_diag(Lp, ps.beta, Ainv);
      } else if (warp >= 4) {
        if (warp < 14) lm_block_task(op, 1, warp - 4, Lp, Msm);
        zero_m_upper(Msm, 128, INTRA_THREADS - 128);
      }
    }
    __syncthreads();
    tri_inverse_offdiag(Lp, ps.beta, Ainv, xtmp);
    // T = A diag(beta) as bf16 (A's strictly-upper part is not stored: zeros)
    for (int i = threadIdx.x; i < 64 * 32; i += blockDim.x) {
      int r = i >> 5, cc = 2 * (i & 31);
      float x0 = (cc <= r) ? Ainv[r * LDF64 + cc] * ps.beta[cc] : 0.f;
      float x1 = (cc + 1 <= r) ? Ainv[r * LDF64 + cc + 1] * ps.beta[cc + 1] : 0.f;
      *reinterpret_cast<uint32_t*>(Tbf + r * LD64 + cc) = pack_bf16(x0, x1);
    }
    // A and L' for the backward, as bf16 tiles in its tcgen05 operand layout
    // (zeros above the diagonal), over the dead Qa and Kd operand tiles
    bf16* Asw = op.Qa;
    bf16* Lsw = op.Kd;
    if (P.A) {
      for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
        const int r = i >> 3, c8 = i & 7;
        float av[8], lv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int cc = 8 * c8 + u;
          av[u] = cc <= r ? Ainv[r * LDF64 + cc] : 0.f;
          lv[u] = cc < r ? Lp[r * LDF64 + cc] : 0.f;
        }
        *reinterpret_cast<bf16x8*>(Asw + sw64_chunk(r, c8)) = pack8(av);
        *reinterpret_cast<bf16x8*>(Lsw + sw64_chunk(r, c8)) = pack8(lv);
      }
    }
    store_rows64(P.M, Msm, LD64, nvalid, H, h, pos.t0);
    tc::fence_async_smem();  // A and L' (written by every thread) are read by the bulk stores below
    __syncthreads();
    // one bulk store each, completed before the exit
    if (P.A && threadIdx.x == 0) {
      const size_t tix = tile_index(P.seq, c, h);
      tc::bulk_s2g(P.A + tix * TILE64N64_ELEMS, Asw, TILE64N64_ELEMS * 2);
      tc::bulk_s2g(P.LP + tix * TILE64N64_ELEMS, Lsw, TILE64N64_ELEMS * 2);
      tc::bulk_commit();
    }

    // W = T Ke, U = T V ; warp w -> rows 16(w&3), cols 32(w>>2)
    {
      const int warp = threadIdx.x >> 5;
      const int m0 = 16 * (warp & 3), n0 = 32 * (warp >> 2);
      float accW[4][4], accU[4][4];
      zero_acc<4>(accW);
      zero_acc<4>(accU);
      warp_mma<4, false, true>(accW, Tbf, LD64, m0, op.Ke, LD128, n0, 0, 64);
      warp_mma<4, false, true>(accU, Tbf, LD64, m0, op.V, LD128, n0, 0, 64);
      // straight from the fragments as 16-byte runs (quad transpose), no staging
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        uint32_t ww[4], wu[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ww[j] = pack_bf16(accW[j][e], accW[j][e + 1]);
          wu[j] = pack_bf16(accU[j][e], accU[j][e + 1]);
        }
        quad_transpose4(ww);
        quad_transpose4(wu);
        const int r = m0 + acc_row(e);
        if (r < nvalid) {
          const size_t off = ((size_t)(pos.t0 + r) * H + h) * D + n0 + 8 * (threadIdx.x & 3);
          *reinterpret_cast<uint4*>(P.W + off) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
          *reinterpret_cast<uint4*>(P.U + off) = make_uint4(wu[0], wu[1], wu[2], wu[3]);
        }
      }
    }
    if (next >= n_items) break;
    item = next;
    pos = npos;
  }
  if (P.A && threadIdx.x == 0) tc::bulk_wait_all();  // the A store reads shared memory
}


// ---------------------------------------------------------------- state pass
struct FwdStateParams {
  SeqInfo seq;
  int H;
  const bf16 *W, *U, *Qt, *Kb, *M;
  const float* dC;
  const float* h0;       // [N][H][128][128] or null
  bf16* o;               // [T_total][H][128]
  bf16* hs;              // [chunks][H] st128 tiles: chunk-start states, or null
  bf16* E;               // [chunks][H] acc64 tiles: v_new, or null
  float* ht;             // [N][H][128][128] or null
};

__device__ __forceinline__ void load_tile128(bf16* dst, const bf16* src, int t0, int nvalid, int H, int h) {
  for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
    int r = i >> 4, cc = i & 15;
    bool ok = r < nvalid;
    const bf16* gp = src + (ok ? ((size_t)(t0 + r) * H + h) * D + cc * 8 : 0);
    cp_async16(dst + r * LD128 + cc * 8, gp, ok);
  }
}
__device__ __forceinline__ void load_tile64(bf16* dst, const bf16* src, int t0, int nvalid, int H, int h) {
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    int r = i >> 3, cc = i & 7;
    bool ok = r < nvalid;
    const bf16* gp = src + (ok ? ((size_t)(t0 + r) * H + h) * 64 + cc * 8 : 0);
    cp_async16(dst + r * LD64 + cc * 8, gp, ok);
  }
}
__device__ __forceinline__ void load_vec128(float* dst, const float* src) {
  for (int i = threadIdx.x; i < 32; i += blockDim.x) cp_async16(dst + 4 * i, src + 4 * i, true);
}

}  // namespace kda
