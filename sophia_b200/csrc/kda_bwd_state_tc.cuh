// Reverse state pass of the chunked KDA backward on the fifth-generation
// tensor cores (tcgen05 + TMEM).
//
// One CTA (288 threads) per (sequence, head) walks the chunks last to first,
// carrying the gradient of the chunk-end state dS (128x128 fp32 in TMEM, one
// lane per state row k).  Per chunk, with S0 the chunk-start state saved by
// the forward (bf16):
//   phase A (MMA): dE  = M^T dO + Kbar dS      (M=64, TMEM region R1, lanes +0)
//                  dKb = E dS^T                (M=64, R1, lanes +16)
//                  dM  = dO E^T                (M=64, N=64, R3)
//     meanwhile:   dS <- diag(2^Gam_C) dS in TMEM; the previous chunk's dQt/dW out
//   epilogue A:    dE out, -dE -> bf16 operand tile; dKb, tril(dM) out;
//                  dGC = rowsum((2^Gam_C dS) o S0)
//   phase B (MMA): dS += Qt^T dO + W^T (-dE)   (M=128, R0)
//                  dQt = dO S0^T, dW = (-dE) S0^T (M=64, R2, lanes +0 / +16)
//   epilogue B:    dS -> bf16 operand tile of the next chunk (dh0 after the first chunk)
// Warp-specialised: warps 0-7 (the consumers) hold the state rows and issue the
// MMAs from one thread; warp 8 is the producer, whose first lane loads by TMA
// into three rings paced by full / empty mbarriers:
//   * the phase-A stage (double-buffered, one chunk ahead): M, dO, Kbar as
//     128B-swizzled boxes, v_new (E) by one bulk copy of the forward's
//     swizzled tile, and 2^Gam_C;
//   * Qt and W, reloaded once the dS update of the chunk before has read them;
//   * S0 (one bulk copy of the forward's swizzled chunk-start state), reloaded
//     once the dQt/dW MMAs of the chunk before have read it.
// The dM epilogue runs while phase B computes.  Rows past the sequence end (the
// last chunk only) arrive with the next sequence's data: the consumers zero
// them in M, dO and Kbar, so dE, dM and dS see exactly the zero rows of a
// zero-filled load.  Completion waits are bounded: on a timeout the CTA records
// an error and leaves through its cleanup path (the producer stops issuing and
// waits for its copies in flight; TMEM is always released).  dE, dW and dM
// leave as whole per-(chunk, head) tiles in the 128B-swizzled operand layout
// (the backward chunk kernel bulk-loads them as operands), dKb and dQt in
// epilogue order (acc64).
#pragma once

#include "kda_fwd.cuh"
#include "kda_fwd_state_tc.cuh"

namespace kda {

struct BwdStateParams {
  SeqInfo seq;
  int H;
  const bf16 *W, *Qt, *Kb, *M, *dO;  // [T_total][H][128] (M: [T_total][H][64])
  const bf16 *E, *hs;                // [chunks][H] 128B-swizzled operand tiles (64 x 128, 128 x 128)
  const float* dC;
  const float* dht;  // [N][H][128][128] or null
  bf16 *dE, *dW, *dM;              // [chunks][H] 128B-swizzled operand tiles (dM: 64 x 64)
  bf16 *dQt, *dKb;                 // [chunks][H] acc64 tiles
  float* dGC;        // [chunks][H][128]
  float* dh0;        // [N][H][128][128] or null
  // M as [T_total][H][64] and dO, Kbar, Qt, W as [T_total][H][128] bf16, for
  // 128B-swizzled TMA boxes of 64 channels x 64 rows (one operand atom each)
  CUtensorMap maps[5];
};

struct BwdStateTcSmem {
  static constexpr int TILE = 16384;                    // [64][128] bf16, two 8 KB atoms
  // stage (double-buffered): phase-A operands of one chunk
  static constexpr int M = 0, DO = 8192, KB = DO + TILE, E = KB + TILE;
  static constexpr int STAGE = E + TILE;                // 57344
  static constexpr int QT = 2 * STAGE, W = QT + TILE;
  static constexpr int S0 = W + TILE;                   // [128][128] bf16, two 16 KB atoms
  static constexpr int DS = S0 + 32768;                 // [128][128] bf16, two 16 KB atoms
  static constexpr int NDE = DS + 32768;                // [64][128] bf16
  static constexpr int DC = NDE + TILE;                 // [2][128] fp32 (per stage)
  static constexpr int GCP = DC + 1024;                 // [2][128] fp32 dGC half-row partials
  static constexpr int MISC = GCP + 1024;               // 12 mbarriers, TMEM slot, abort flag
  static constexpr int END = MISC + 128;
};
static_assert(BwdStateTcSmem::END <= 232448, "bwd state (tcgen05) shared memory");

// Eight fp32 values -> one bf16 16-byte chunk.
__device__ __forceinline__ void store_chunk8(bf16* dst, const float* a) {
  uint4 pk;
  pk.x = pack_bf16(a[0], a[1]);
  pk.y = pack_bf16(a[2], a[3]);
  pk.z = pack_bf16(a[4], a[5]);
  pk.w = pack_bf16(a[6], a[7]);
  *reinterpret_cast<uint4*>(dst) = pk;
}

constexpr uint32_t BSTATE_STAGE_BYTES = 8192 + 3 * BwdStateTcSmem::TILE + 512;  // M, dO, Kbar, E, 2^Gam_C
constexpr uint32_t BSTATE_QW_BYTES = 2 * BwdStateTcSmem::TILE;
constexpr uint32_t BSTATE_S0_BYTES = STATE_ELEMS * 2;

__global__ void __launch_bounds__(STATE_THREADS, 1) kda_bwd_state_tc_kernel(const __grid_constant__ BwdStateParams P) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];  // 1 KB-aligned dynamic shared memory
  unsigned char* smem = tc_smem;
  using S_ = BwdStateTcSmem;
  const int n = blockIdx.x, h = blockIdx.y, H = P.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hf = (warp >> 2) & 1;  // TMEM lane quarter, column half
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  const int nchunks = seq_nchunks(P.seq, n);
  const int cbase = seq_chunk_base(P.seq, n);
  const int krow = 32 * q + lane;  // state row of this thread (M=128 layout)
  const int arow = 16 * q + (lane & 15);  // chunk row of this thread (M=64 layout)
  const bool hi = lane >= 16;             // second M=64 accumulator (lanes +16)

  if (nchunks == 0) {  // empty sequence: dh0 = dht
    if (P.dh0) {
      const float* src = P.dht ? P.dht + ((size_t)n * H + h) * D * D : nullptr;
      float* dst = P.dh0 + ((size_t)n * H + h) * D * D;
      for (int i = tid; i < D * D; i += blockDim.x) dst[i] = src ? src[i] : 0.f;
    }
    return;
  }
  if (smem_u32(smem) & 1023) {  // swizzled atoms need 1 KB alignment
    if (tid == 0) atomicExch(&g_kda_device_error, 2);
    return;
  }
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + S_::MISC);  // A1, A2, B1, B2
  uint64_t* fullA = mbar + 4;    // [2] phase-A stage landed
  uint64_t* emptyA = mbar + 6;   // [2] phase-A stage read
  uint64_t* fullQW = mbar + 8;   // Qt, W landed
  uint64_t* emptyQW = mbar + 9;  // Qt, W read
  uint64_t* fullS0 = mbar + 10;  // S0 landed
  uint64_t* emptyS0 = mbar + 11; // S0 read
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbar + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  unsigned char* sQt = smem + S_::QT;
  unsigned char* sW = smem + S_::W;
  unsigned char* sS0 = smem + S_::S0;
  unsigned char* sDS = smem + S_::DS;
  unsigned char* sNDE = smem + S_::NDE;
  float* gcp = reinterpret_cast<float*>(smem + S_::GCP);

  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < 12; ++i) tc::mbar_init(mbar + i, 1);
    tc::fence_mbar_init();
    *abort_flag = 0;
  }
  tc::fence_before_sync();
  __syncthreads();  // the last barrier of all 288 threads
  tc::fence_after_sync();
  auto stage = [&](int ci) { return smem + (ci & 1) * S_::STAGE; };
  auto stage_dc = [&](int ci) { return reinterpret_cast<float*>(smem + S_::DC) + (ci & 1) * D; };
  const int last = nchunks - 1;

  if (warp == STATE_CONSUMERS / 32) {
    // ---- producer.  Chunk ci = last - it; its stage is ci & 1 and that
    // stage's use (it >> 1); the Qt/W and S0 buffers are used once per chunk.
    if (lane != 0) return;
    auto load_stage = [&](int ci) {
      unsigned char* b = stage(ci);
      const int t0 = bos + ci * C;
      uint64_t* f = fullA + (ci & 1);
      tc::mbar_expect_tx(f, BSTATE_STAGE_BYTES);
      tc::tma_load_3d(b + S_::M, &P.maps[0], 0, h, t0, f);
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        tc::tma_load_3d(b + S_::DO + a * 8192, &P.maps[1], 64 * a, h, t0, f);
        tc::tma_load_3d(b + S_::KB + a * 8192, &P.maps[2], 64 * a, h, t0, f);
      }
      tc::bulk_g2s(b + S_::E, P.E + tile_index(P.seq, cbase + ci, h) * TILE64_ELEMS, TILE64_ELEMS * 2, f);
      tc::bulk_g2s(stage_dc(ci), P.dC + ((size_t)(cbase + ci) * H + h) * D, 512, f);
    };
    auto load_qw = [&](int ci) {
      const int t0 = bos + ci * C;
      tc::mbar_expect_tx(fullQW, BSTATE_QW_BYTES);
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        tc::tma_load_3d(sQt + a * 8192, &P.maps[3], 64 * a, h, t0, fullQW);
        tc::tma_load_3d(sW + a * 8192, &P.maps[4], 64 * a, h, t0, fullQW);
      }
    };
    auto load_s0 = [&](int ci) {
      tc::mbar_expect_tx(fullS0, BSTATE_S0_BYTES);
      tc::bulk_g2s(sS0, P.hs + tile_index(P.seq, cbase + ci, h) * STATE_ELEMS, BSTATE_S0_BYTES, fullS0);
    };
    // last issued use of each ring (-1: none), for the drain below
    int lastA[2] = {-1, -1}, lastQW = -1, lastS0 = -1;
    load_stage(last); lastA[last & 1] = 0;
    load_qw(last); lastQW = 0;
    load_s0(last); lastS0 = 0;
    if (last >= 1) { load_stage(last - 1); lastA[(last - 1) & 1] = 0; }
    for (int it = 1; it <= last; ++it) {
      const int ci = last - it;
      if (!tc::mbar_wait(emptyQW, (it - 1) & 1) || *abort_flag) break;
      load_qw(ci); lastQW = it;
      if (!tc::mbar_wait(emptyS0, (it - 1) & 1) || *abort_flag) break;
      load_s0(ci); lastS0 = it;
      if (ci >= 1) {
        const int u = (it + 1) >> 1;  // use of stage (ci - 1) & 1 by chunk ci - 1
        if (!tc::mbar_wait(emptyA + ((ci - 1) & 1), (u - 1) & 1) || *abort_flag) break;
        load_stage(ci - 1); lastA[(ci - 1) & 1] = u;
      }
    }
    // no copy may still be writing shared memory when the CTA ends
    for (int s2 = 0; s2 < 2; ++s2)
      if (lastA[s2] >= 0) tc::mbar_wait(fullA + s2, lastA[s2] & 1);
    if (lastQW >= 0) tc::mbar_wait(fullQW, lastQW & 1);
    if (lastS0 >= 0) tc::mbar_wait(fullS0, lastS0 & 1);
    return;
  }

  // ---- consumers (256 threads)
  // on a timeout: stop, release a producer waiting for a buffer, and leave
  auto give_up = [&]() {
    *abort_flag = 1;
    if (tid == 0) {
      mbar_arrive(emptyA); mbar_arrive(emptyA + 1); mbar_arrive(emptyQW); mbar_arrive(emptyS0);
    }
  };
  // dS row krow, columns [64 hf, 64 hf + 64) -> bf16 operand tile
  auto store_ds = [&](const float (&v)[64]) {
    unsigned char* atom = sDS + hf * 16384;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 pk;
      pk.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
      pk.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
      pk.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
      pk.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
      *reinterpret_cast<uint4*>(atom + krow * 128 + ((c ^ (krow & 7)) << 4)) = pk;
    }
  };

  // dht -> registers and the bf16 operand tile
  float v[64];
  {
    const float* src = P.dht ? P.dht + (((size_t)n * H + h) * D + krow) * D + 64 * hf : nullptr;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      const float4 x = src ? *reinterpret_cast<const float4*>(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
    }
    store_ds(v);
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  consumer_sync();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t tq = (uint32_t)(32 * q) << 16;
  const uint32_t tR0 = tbase + tq + 64 * hf;         // dS (this thread's lane, its column half)
  const uint32_t tR1 = tbase + tq + 128 + 64 * hf;   // dE / dKb
  const uint32_t tR2 = tbase + tq + 256 + 64 * hf;   // dQt / dW
  const uint32_t tR3 = tbase + tq + 384 + 32 * hf;   // dM
  const uint32_t idA1 = tc::idesc_bf16(64, 128, true, true);    // M^T dO
  const uint32_t idA2 = tc::idesc_bf16(64, 128, false, true);   // Kbar dS
  const uint32_t idKK = tc::idesc_bf16(64, 128, false, false);  // E dS^T, dO S0^T, (-dE) S0^T
  const uint32_t idM = tc::idesc_bf16(64, 64, false, false);    // dO E^T
  const uint32_t idB = tc::idesc_bf16(128, 128, true, true);    // Qt^T dO, W^T (-dE)

  // dQt (acc64 tile) / dW (128B-swizzled operand tile) of chunk cp (R2); whole
  // tiles: rows past the end are zero
  auto r2_epilogue = [&](int cp) {
    bf16* tile = (hi ? P.dW : P.dQt) + tile_index(P.seq, cbase + cp, h) * TILE64_ELEMS;
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      float a[32];
      tc::tmem_ld32(tR2 + c0, a);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int v0 = 64 * hf + c0 + 8 * c;
        store_chunk8(tile + (hi ? sw64_chunk(arow, v0 >> 3) : acc64_off(arow, v0)), a + 8 * c);
      }
    }
  };

  bool ok = true;
  int it = 0;
  for (int ci = last; ci >= 0; --ci, ++it) {
    const int t0 = bos + ci * C, nv = min(C, eos - t0);
    const size_t cidx = (size_t)(cbase + ci) * H + h;
    const size_t tix = tile_index(P.seq, cbase + ci, h);
    unsigned char* st = stage(ci);
    const float* dC = stage_dc(ci);
    // this chunk's phase-A operands (loaded while the chunk before computed)
    if (!tc::mbar_wait(fullA + (ci & 1), (it >> 1) & 1)) *abort_flag = 1;
    if (nv < C) {
      // a partial (last) chunk: the rows past the end belong to the next sequence
      for (int i = tid; i < (C - nv) * 8 * 5; i += STATE_CONSUMERS) {
        const int r = nv + i / 40, j = i % 40, t = j >> 3, c8 = j & 7;
        unsigned char* base = st + (t == 0 ? S_::M : (t <= 2 ? S_::DO + (t - 1) * 8192 : S_::KB + (t - 3) * 8192));
        *reinterpret_cast<uint4*>(base + r * 128 + (c8 << 4)) = make_uint4(0u, 0u, 0u, 0u);
      }
      tc::fence_async_smem();
      consumer_sync();
    }
    // (a timed-out wait is acted on after the next barrier, by every thread alike)
    // ---- phase A MMAs
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t m0 = smem_u32(st + S_::M), do0 = smem_u32(st + S_::DO);
      const uint32_t kb0 = smem_u32(st + S_::KB), e0 = smem_u32(st + S_::E), s0 = smem_u32(sDS);
      // dE = M^T dO + Kbar dS
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tbase + 128, tc::smem_desc(m0 + ks * 2048, 8192, 1024),
                     tc::smem_desc(do0 + ks * 2048, 8192, 1024), idA1, ks > 0);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16(tbase + 128, tc::smem_desc(kb0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024),
                     tc::smem_desc(s0 + ks * 2048, 16384, 1024), idA2, true);
      // dKb = E dS^T
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16(tbase + (16u << 16) + 128, tc::smem_desc(e0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024),
                     tc::smem_desc(s0 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024), idKK, ks > 0);
      tc::mma_commit(mbar + 0);
      // dM = dO E^T
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        tc::mma_bf16(tbase + 384, tc::smem_desc(do0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024),
                     tc::smem_desc(e0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), idM, ks > 0);
      tc::mma_commit(mbar + 1);
    }
    // dS <- diag(2^Gam_C) dS (dS is R0 = v, the chunk-end gradient)
    {
      const float dc = dC[krow];
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] *= dc;
      float a[32], b[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) { a[i] = v[i]; b[i] = v[32 + i]; }
      tc::tmem_st32(tR0, a);
      tc::tmem_st32(tR0 + 32, b);
    }
    // dQt / dW of the chunk after this one; its MMAs were the last readers of S0
    // and of that chunk's stage: both go back to the producer
    if (ci < last) {
      if (!tc::mbar_wait(mbar + 3, (it - 1) & 1)) *abort_flag = 1;
      tc::fence_after_sync();
      if (tid == 0) { mbar_arrive(emptyS0); mbar_arrive(emptyA + ((ci + 1) & 1)); }
      r2_epilogue(ci + 1);
    }
    // ---- epilogue A
    if (!tc::mbar_wait(mbar + 0, it & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    {
      bf16* tile = (hi ? P.dKb : P.dE) + tix * TILE64_ELEMS;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 32) {
        float a[32];
        tc::tmem_ld32(tR1 + c0, a);
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // dKb: acc64 tile; dE: 128B-swizzled operand tile
          const int v0 = 64 * hf + c0 + 8 * c;
          store_chunk8(tile + (hi ? acc64_off(arow, v0) : sw64_chunk(arow, v0 >> 3)), a + 8 * c);
        }
        if (!hi) {  // -dE -> operand tile (rows past the end stay zero)
          unsigned char* atom = sNDE + hf * 8192;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int chunk = (c0 >> 3) + c;
            uint4 pk = make_uint4(0u, 0u, 0u, 0u);
            if (arow < nv) {
              pk.x = pack_bf16(-a[8 * c + 0], -a[8 * c + 1]);
              pk.y = pack_bf16(-a[8 * c + 2], -a[8 * c + 3]);
              pk.z = pack_bf16(-a[8 * c + 4], -a[8 * c + 5]);
              pk.w = pack_bf16(-a[8 * c + 6], -a[8 * c + 7]);
            }
            *reinterpret_cast<uint4*>(atom + arow * 128 + ((chunk ^ (arow & 7)) << 4)) = pk;
          }
        }
      }
    }
    // dGC: half-row partials of rowsum((2^Gam_C dS) o S0)
    if (!tc::mbar_wait(fullS0, it & 1)) *abort_flag = 1;  // S0 of this chunk
    {
      const unsigned char* atom = sS0 + hf * 16384;
      float part = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 s = *reinterpret_cast<const uint4*>(atom + krow * 128 + ((c ^ (krow & 7)) << 4));
        const float2 s0 = unpack_bf16(s.x), s1 = unpack_bf16(s.y), s2 = unpack_bf16(s.z), s3 = unpack_bf16(s.w);
        part += v[8 * c + 0] * s0.x + v[8 * c + 1] * s0.y + v[8 * c + 2] * s1.x + v[8 * c + 3] * s1.y +
                v[8 * c + 4] * s2.x + v[8 * c + 5] * s2.y + v[8 * c + 6] * s3.x + v[8 * c + 7] * s3.y;
      }
      gcp[hf * D + krow] = part;
    }
    if (tid == 0 && !tc::mbar_wait(fullQW, it & 1)) *abort_flag = 1;  // Qt, W of this chunk (phase B)
    tc::fence_async_smem();
    tc::fence_before_sync();
    consumer_sync();
    if (*abort_flag) { ok = false; break; }
    if (tid < D) P.dGC[cidx * D + tid] = gcp[tid] + gcp[D + tid];
    // ---- phase B MMAs
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t do0 = smem_u32(st + S_::DO), qt0 = smem_u32(sQt), w0 = smem_u32(sW);
      const uint32_t nde0 = smem_u32(sNDE), s00 = smem_u32(sS0);
      // dS += Qt^T dO + W^T (-dE)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tbase, tc::smem_desc(qt0 + ks * 2048, 8192, 1024), tc::smem_desc(do0 + ks * 2048, 8192, 1024),
                     idB, true);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        tc::mma_bf16(tbase, tc::smem_desc(w0 + ks * 2048, 8192, 1024), tc::smem_desc(nde0 + ks * 2048, 8192, 1024),
                     idB, true);
      tc::mma_commit(mbar + 2);
      // dQt = dO S0^T, dW = (-dE) S0^T
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t bd = tc::smem_desc(s00 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
        tc::mma_bf16(tbase + 256, tc::smem_desc(do0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), bd, idKK, ks > 0);
        tc::mma_bf16(tbase + (16u << 16) + 256, tc::smem_desc(nde0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), bd,
                     idKK, ks > 0);
      }
      tc::mma_commit(mbar + 3);
    }
    // tril(dM) out (off the dS chain: phase B does not touch R3)
    if (!tc::mbar_wait(mbar + 1, it & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    {
      float a[32];
      tc::tmem_ld32(tR3, a);
      if (!hi) {
        const int cb = 32 * hf;
        float m[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) m[i] = cb + i <= arow ? a[i] : 0.f;
        bf16* tile = P.dM + tix * TILE64N64_ELEMS;
#pragma unroll
        for (int c = 0; c < 4; ++c) store_chunk8(tile + sw64_chunk(arow, (cb >> 3) + c), m + 8 * c);
      }
    }
    // ---- epilogue B: dS of the chunk before -> operand tile (or dh0)
    if (!tc::mbar_wait(mbar + 2, it & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    if (tid == 0) mbar_arrive(emptyQW);  // the dS update has read Qt and W
    {
      float a[32], b[32];
      tc::tmem_ld32(tR0, a);
      tc::tmem_ld32(tR0 + 32, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) { v[i] = a[i]; v[32 + i] = b[i]; }
    }
    if (ci > 0) {
      store_ds(v);
    } else if (P.dh0) {
      float* dst = P.dh0 + (((size_t)n * H + h) * D + krow) * D + 64 * hf;
#pragma unroll
      for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    consumer_sync();
    if (*abort_flag) { ok = false; break; }
  }
  if (ok) {  // dQt / dW of the first chunk
    if (!tc::mbar_wait(mbar + 3, (it - 1) & 1)) ok = false;
    tc::fence_after_sync();
    if (ok) r2_epilogue(0);
  }
  if (!ok) {
    if (tid == 0) atomicExch(&g_kda_device_error, 1);
    give_up();
  }
  tc::fence_before_sync();
  consumer_sync();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

}  // namespace kda
