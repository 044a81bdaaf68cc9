// Forward state pass on the fifth-generation tensor cores (tcgen05 + TMEM).
//
// One CTA (288 threads) per (sequence, head) walks the chunks in order.  The
// 128x128 fp32 state S lives in TMEM (columns 128..255, one lane per state
// row k); its bf16 copy in shared memory (128B-swizzled, rows k) is the B
// operand of the chunk products.  E and O accumulate in one of two 128-column
// TMEM buffers (E in lanes 0-15 and O in lanes 16-31 of each quarter),
// alternating by chunk.  Per chunk, only true dependencies sit between the
// MMAs:
//   MMA  E_acc = W S, O_acc = Qt S       (M=64 each, from the bf16 state tile)
//     meanwhile: S <- diag(2^Gam_C) S in TMEM from the registers of the last
//     S epilogue, the chunk-start state out, the previous chunk's o staged in
//     shared memory
//   epilogue: E = U - E_acc -> bf16 tile (B operand) and v_new for the backward
//   MMA  O_acc += M E ; S += Kbar^T E    (M=64 / M=128)
//     meanwhile: the staged o rows of the previous chunk leave, coalesced
//   epilogue: S -> registers -> bf16 tile for the next chunk.
// Warp-specialised: warps 0-7 (the consumers) hold the state rows and issue
// the MMAs from one thread; warp 8 is the producer, whose first lane brings
// each chunk's W, Qt, Kbar, U and M tiles in by TMA (128B-swizzled boxes that
// land as tcgen05 operand atoms) plus its decay vector by a bulk copy, into a
// two-stage ring paced by full / empty mbarriers.  Rows past the sequence end
// arrive with the next sequence's (or zero) data: E is zeroed there, so they
// add nothing to the state, and their o rows are not stored.  Completion is
// tracked with mbarriers whose waits are bounded: on a timeout the CTA records
// an error and leaves through its cleanup path (the producer stops issuing and
// waits for its copies in flight; TMEM is always released).  v_new (E) and the
// chunk-start states leave as per-(chunk, head) tiles by bulk stores of the
// shared-memory operand tiles themselves (128B-swizzled), so the backward's
// bulk loads land them directly as operands.
#pragma once

#include "kda_fwd.cuh"
#include "kda_tc.cuh"

namespace kda {

struct StateTcSmem {
  static constexpr int TILE = 16384;                    // [64][128] bf16, two 8 KB atoms
  static constexpr int W = 0, QT = TILE, KB = 2 * TILE, U = 3 * TILE, M = 4 * TILE;  // M: one 8 KB atom
  static constexpr int DC = M + 8192;                   // 128 fp32
  static constexpr int STAGE = 74752;                   // 73 KB per stage (1 KB aligned)
  static constexpr int NSTAGE = 2;                      // current chunk + the next one
  static constexpr int S = NSTAGE * STAGE;              // [128][128] bf16, two 16 KB atoms
  static constexpr int E = S + 32768;                   // [64][128] bf16, two 8 KB atoms
  static constexpr int OST = E + 16384;                 // [64][LD128] bf16 staged o rows
  static constexpr int MISC = OST + 64 * LD128 * 2;     // mbarriers (E, S, full x 2, empty x 2), TMEM slot, abort flag
  static constexpr int END = MISC + 64;
  static_assert(DC + 512 <= STAGE, "stage overflow");
  static_assert(STAGE % 1024 == 0 && QT % 1024 == 0 && M % 1024 == 0, "TMA destinations of swizzled boxes");
  static_assert(END <= 232448, "fwd state (tcgen05) shared memory");
};

constexpr int STATE_CONSUMERS = 256;                      // warps 0-7
constexpr int STATE_THREADS = STATE_CONSUMERS + 32;         // + the producer warp
constexpr uint32_t STATE_STAGE_BYTES = 4 * StateTcSmem::TILE + 8192 + 512;

// Barrier of the consumer warps only (named barrier 1; the producer warp never joins).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;\n" ::"n"(STATE_CONSUMERS) : "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(mbar)) : "memory");
}

__global__ void __launch_bounds__(STATE_THREADS, 1) kda_fwd_state_tc_kernel(const __grid_constant__ FwdStateParams P) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];  // 1 KB-aligned dynamic shared memory
  unsigned char* smem = tc_smem;
  const int n = blockIdx.x, h = blockIdx.y, H = P.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = warp & 3, half = (warp >> 2) & 1;  // TMEM lane quarter, column half
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  const int nchunks = seq_nchunks(P.seq, n);
  const int cbase = seq_chunk_base(P.seq, n);
  uint64_t* mbarE = reinterpret_cast<uint64_t*>(smem + StateTcSmem::MISC);
  uint64_t* mbarS = mbarE + 1;
  uint64_t* full = mbarE + 2;   // [2]: a stage's copies landed
  uint64_t* empty = mbarE + 4;  // [2]: a stage's MMAs and reads are done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbarE + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);
  unsigned char* sS = smem + StateTcSmem::S;
  unsigned char* sE = smem + StateTcSmem::E;

  if (smem_u32(smem) & 1023) {  // swizzled atoms need 1 KB alignment
    if (tid == 0) atomicExch(&g_kda_device_error, 2);
    return;
  }
  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    tc::mbar_init(mbarE, 1);
    tc::mbar_init(mbarS, 1);
    for (int i = 0; i < 4; ++i) tc::mbar_init(full + i, 1);  // full[0..1], empty[0..1]
    tc::fence_mbar_init();
    *abort_flag = 0;
  }
  tc::fence_before_sync();
  __syncthreads();  // the last barrier of all 288 threads
  tc::fence_after_sync();

  if (warp == STATE_CONSUMERS / 32) {
    // ---- producer: chunk ci into stage ci % 2 once the stage's previous chunk is done
    if (lane != 0 || P.withhold_loads) return;
    int issued = 0;
    for (int ci = 0; ci < nchunks; ++ci) {
      const int st = ci & 1;
      if (ci >= 2 && !tc::mbar_wait(empty + st, ((ci >> 1) - 1) & 1)) break;
      if (*abort_flag) break;
      unsigned char* base = smem + st * StateTcSmem::STAGE;
      const int t0 = bos + ci * C;
      tc::mbar_expect_tx(full + st, STATE_STAGE_BYTES);
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        tc::tma_load_3d(base + StateTcSmem::W + a * 8192, &P.maps[0], 64 * a, h, t0, full + st);
        tc::tma_load_3d(base + StateTcSmem::QT + a * 8192, &P.maps[1], 64 * a, h, t0, full + st);
        tc::tma_load_3d(base + StateTcSmem::KB + a * 8192, &P.maps[2], 64 * a, h, t0, full + st);
        tc::tma_load_3d(base + StateTcSmem::U + a * 8192, &P.maps[3], 64 * a, h, t0, full + st);
      }
      tc::tma_load_3d(base + StateTcSmem::M, &P.maps[4], 0, h, t0, full + st);
      tc::bulk_g2s(base + StateTcSmem::DC, P.dC + ((size_t)(cbase + ci) * H + h) * D, 512, full + st);
      issued = ci + 1;
    }
    // no copy may still be writing shared memory when the CTA ends
    for (int ci = issued - 2; ci < issued; ++ci)
      if (ci >= 0) tc::mbar_wait(full + (ci & 1), (ci >> 1) & 1);
    return;
  }

  // ---- consumers (256 threads)
  const uint32_t tbase = *tslot;
  const uint32_t tq = (uint32_t)(32 * sub) << 16;
  const uint32_t tS = tbase + tq + 128 + 64 * half;  // state rows
  // E/O buffer b: lane 0 (E) / lane 16 (O) accumulators at column base 0 or 256
  auto eo_col = [&](int b) { return b ? 256u : 0u; };
  auto tEO = [&](int b) { return tbase + tq + eo_col(b) + 64 * half; };
  const int krow = 32 * sub + lane;                  // state row of this thread
  const int arow = 16 * sub + (lane & 15);           // chunk row of this thread (M=64 layout)
  const uint32_t idE = tc::idesc_bf16(64, 128, false, true);
  const uint32_t idS = tc::idesc_bf16(128, 128, true, true);
  bf16* ost = reinterpret_cast<bf16*>(smem + StateTcSmem::OST);
  // on a timeout: stop, release a producer waiting for a stage, and leave
  auto give_up = [&]() {
    *abort_flag = 1;
    if (tid == 0) { mbar_arrive(empty); mbar_arrive(empty + 1); }
  };

  // state row krow, columns [64 half, 64 half + 64): fp32 -> bf16 operand tile
  auto store_tile = [&](const float (&v)[64]) {
    unsigned char* atom = sS + half * 16384;
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
  // O rows of buffer b (lanes 16-31) -> staging tile
  auto stage_o = [&](int b) {
#pragma unroll
    for (int c0 = 0; c0 < 64; c0 += 32) {
      float acc[32];
      tc::tmem_ld32(tEO(b) + c0, acc);
      if (lane >= 16) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 pk;
          pk.x = pack_bf16(acc[8 * c + 0], acc[8 * c + 1]);
          pk.y = pack_bf16(acc[8 * c + 2], acc[8 * c + 3]);
          pk.z = pack_bf16(acc[8 * c + 4], acc[8 * c + 5]);
          pk.w = pack_bf16(acc[8 * c + 6], acc[8 * c + 7]);
          *reinterpret_cast<uint4*>(ost + arow * LD128 + 64 * half + c0 + 8 * c) = pk;
        }
      }
    }
  };
  // staged o rows of chunk ci -> global, 16 threads per 256-byte row
  auto copy_o = [&](int ci) {
    const int t0 = bos + ci * C, nv = min(C, eos - t0);
    for (int i = tid; i < 64 * 16; i += STATE_CONSUMERS) {
      const int r = i >> 4, cc = i & 15;
      if (r < nv)
        *reinterpret_cast<uint4*>(P.o + ((size_t)(t0 + r) * H + h) * D + 8 * cc) =
            *reinterpret_cast<const uint4*>(ost + r * LD128 + 8 * cc);
    }
  };

  // v: this thread's state row (64 columns), unscaled, from an S epilogue (or
  // h0) to the next chunk's scaling
  float v[64];
  if (nchunks > 0) {
    const float* h0 = P.h0 ? P.h0 + (((size_t)n * H + h) * D + krow) * D + 64 * half : nullptr;
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      float4 x = h0 ? *reinterpret_cast<const float4*>(h0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
    }
    store_tile(v);
  } else if (P.ht) {
    // empty sequence: the final state is the initial state
    const float* h0 = P.h0 ? P.h0 + (((size_t)n * H + h) * D + krow) * D + 64 * half : nullptr;
    float* dst = P.ht + (((size_t)n * H + h) * D + krow) * D + 64 * half;
    for (int i = 0; i < 64; ++i) dst[i] = h0 ? h0[i] : 0.f;
  }
  tc::fence_async_smem();
  tc::fence_before_sync();
  consumer_sync();

  bool ok = true;
  for (int ci = 0; ci < nchunks && ok; ++ci) {
    const int stg = ci & 1;
    unsigned char* buf = smem + stg * StateTcSmem::STAGE;
    const bool last = ci + 1 == nchunks;
    const int eo = ci & 1;
    const int nv = min(C, eos - (bos + ci * C));
    // this chunk's operands (loaded while the chunk before computed)
    if (!tc::mbar_wait(full + stg, (ci >> 1) & 1, P.wait_polls)) *abort_flag = 1;
    if (tid == 0 && P.E) tc::bulk_wait_read_all();  // v_new of the chunk before has left sE
    consumer_sync();
    if (*abort_flag) { ok = false; break; }
    // E = W S, O = Qt S into buffer eo
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t w0 = smem_u32(buf + StateTcSmem::W), q0 = smem_u32(buf + StateTcSmem::QT);
      const uint32_t s0 = smem_u32(sS);
      const uint32_t dE = tbase + eo_col(eo);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint64_t bd = tc::smem_desc(s0 + ks * 2048, 16384, 1024);
        tc::mma_bf16(dE, tc::smem_desc(w0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), bd, idE, ks > 0);
        tc::mma_bf16(dE + (16u << 16), tc::smem_desc(q0 + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), bd, idE,
                     ks > 0);
      }
      tc::mma_commit(mbarE);
      // the chunk-start state for the backward: the bf16 operand tile itself
      // (128B-swizzled, the layout the backward's operand slot takes)
      if (P.hs) {
        tc::bulk_s2g(P.hs + tile_index(P.seq, cbase + ci, h) * STATE_ELEMS, sS, STATE_ELEMS * 2);
        tc::bulk_commit();
      }
    }
    // S <- diag(2^Gam_C) S in TMEM from the registers
    {
      const float dc = reinterpret_cast<const float*>(buf + StateTcSmem::DC)[krow];
      float a[32], b[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) { a[i] = v[i] * dc; b[i] = v[32 + i] * dc; }
      tc::tmem_st32(tS, a);
      tc::tmem_st32(tS + 32, b);
    }
    if (ci > 0) stage_o(eo ^ 1);  // o of the previous chunk (its MMAs are complete)
    if (!tc::mbar_wait(mbarE, ci & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    // E = U - E_acc (threads holding E rows: lanes 0-15); rows past the sequence
    // end are zero (their operand rows belong to the next sequence)
    {
      const int r = arow;
      const bool live = r < nv;
      const unsigned char* uat = buf + StateTcSmem::U + half * 8192;
      unsigned char* eat = sE + half * 8192;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 32) {
        float acc[32];
        tc::tmem_ld32(tEO(eo) + c0, acc);
        if (lane < 16) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int chunk = (c0 >> 3) + c;
            const uint32_t off = r * 128 + ((chunk ^ (r & 7)) << 4);
            uint4 u = *reinterpret_cast<const uint4*>(uat + off);
            float2 u0 = unpack_bf16(u.x), u1 = unpack_bf16(u.y), u2 = unpack_bf16(u.z), u3 = unpack_bf16(u.w);
            uint4 e = make_uint4(0u, 0u, 0u, 0u);
            if (live) {
              e.x = pack_bf16(u0.x - acc[8 * c + 0], u0.y - acc[8 * c + 1]);
              e.y = pack_bf16(u1.x - acc[8 * c + 2], u1.y - acc[8 * c + 3]);
              e.z = pack_bf16(u2.x - acc[8 * c + 4], u2.y - acc[8 * c + 5]);
              e.w = pack_bf16(u3.x - acc[8 * c + 6], u3.y - acc[8 * c + 7]);
            }
            *reinterpret_cast<uint4*>(eat + off) = e;
          }
        }
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    if (tid == 0 && P.hs) tc::bulk_wait_read_all();  // the chunk-start state has left sS
    consumer_sync();
    if (*abort_flag) { ok = false; break; }
    // O += M E ; S += Kbar^T E; v_new (E, rows past the end zero) for the backward
    if (tid == 0) {
      tc::fence_after_sync();
      if (P.E) {
        tc::bulk_s2g(P.E + tile_index(P.seq, cbase + ci, h) * TILE64_ELEMS, sE, TILE64_ELEMS * 2);
        tc::bulk_commit();
      }
      const uint32_t m0 = smem_u32(buf + StateTcSmem::M), k0 = smem_u32(buf + StateTcSmem::KB);
      const uint32_t e0 = smem_u32(sE);
      const uint32_t dO = tbase + eo_col(eo) + (16u << 16);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint64_t ed = tc::smem_desc(e0 + ks * 2048, 8192, 1024);
        tc::mma_bf16(tbase + 128, tc::smem_desc(k0 + ks * 2048, 8192, 1024), ed, idS, true);
        tc::mma_bf16(dO, tc::smem_desc(m0 + ks * 32, 16, 1024), ed, idE, true);
      }
      tc::mma_commit(mbarS);
    }
    if (ci > 0) copy_o(ci - 1);  // staged before the barrier above
    if (!tc::mbar_wait(mbarS, ci & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    // every read of this stage is done (the MMAs, U, the decay vector): hand it back
    if (tid == 0) mbar_arrive(empty + stg);
    // S_{ci+1} -> registers -> operand tile (or the final state)
    {
      float a[32], bb[32];
      tc::tmem_ld32(tS, a);
      tc::tmem_ld32(tS + 32, bb);
#pragma unroll
      for (int i = 0; i < 32; ++i) { v[i] = a[i]; v[32 + i] = bb[i]; }
      if (last) {
        if (P.ht) {
          float* dst = P.ht + (((size_t)n * H + h) * D + krow) * D + 64 * half;
#pragma unroll
          for (int i = 0; i < 64; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      } else {
        store_tile(v);
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    consumer_sync();
    if (*abort_flag) ok = false;
  }
  if (ok && nchunks > 0) {  // o of the last chunk
    stage_o((nchunks - 1) & 1);
    consumer_sync();
    copy_o(nchunks - 1);
  }
  if (!ok) {
    if (tid == 0) atomicExch(&g_kda_device_error, 1);
    give_up();
  }
  if (tid == 0) tc::bulk_wait_all();  // the bulk stores read sS / sE
  tc::fence_before_sync();
  consumer_sync();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

}  // namespace kda
