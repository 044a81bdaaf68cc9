// Forward state pass on the fifth-generation tensor cores (tcgen05 + TMEM).
//
// One CTA (256 threads) per (sequence, head) walks the chunks in order.  The
// 128x128 fp32 state S lives in TMEM (columns 128..255, one lane per state
// row k); its bf16 copy in shared memory (128B-swizzled, rows k) is the B
// operand of the chunk products.  E and O accumulate in one of two 128-column
// TMEM buffers (E in lanes 0-15 and O in lanes 16-31 of each quarter),
// alternating by chunk.  Per chunk, only true dependencies sit between the
// MMAs:
//   MMA  E_acc = W S, O_acc = Qt S       (M=64 each, from the bf16 state tile)
//     meanwhile: S <- diag(2^Gam_C) S in TMEM from the registers of the last
//     S epilogue, the chunk-start state out, the previous chunk's o staged in
//     shared memory, the next chunk's loads issued
//   epilogue: E = U - E_acc -> bf16 tile (B operand) and v_new for the backward
//   MMA  O_acc += M E ; S += Kbar^T E    (M=64 / M=128)
//     meanwhile: the staged o rows of the previous chunk leave, coalesced
//   epilogue: S -> registers -> bf16 tile for the next chunk.
// One thread issues the MMAs; completion is tracked with mbarriers whose waits
// are bounded: on a timeout the CTA records an error and leaves through its
// cleanup path (TMEM is always released).  Chunk inputs are double-buffered
// with cp.async into swizzled tiles (the next chunk loads during this one);
// rows past the sequence end are zero.  v_new (E) and the chunk-start states
// are written as per-(chunk, head) tiles in epilogue order (acc64, st128), so
// each warp store is one contiguous run.
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
  static constexpr int MISC = OST + 64 * LD128 * 2;     // mbarriers, TMEM slot, abort flag
  static constexpr int END = MISC + 64;
  static_assert(DC + 512 <= STAGE, "stage overflow");
  static_assert(END <= 232448, "fwd state (tcgen05) shared memory");
};

__global__ void __launch_bounds__(256, 1) kda_fwd_state_tc_kernel(FwdStateParams P) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];  // 1 KB-aligned dynamic shared memory
  unsigned char* smem = tc_smem;
  const int n = blockIdx.x, h = blockIdx.y, H = P.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = warp & 3, half = warp >> 2;  // TMEM lane quarter, column half
  const int bos = seq_bos(P.seq, n), eos = seq_eos(P.seq, n);
  const int nchunks = seq_nchunks(P.seq, n);
  const int cbase = seq_chunk_base(P.seq, n);
  uint64_t* mbarE = reinterpret_cast<uint64_t*>(smem + StateTcSmem::MISC);
  uint64_t* mbarS = mbarE + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mbarE + 2);
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
    tc::fence_mbar_init();
    *abort_flag = 0;
  }
  bf16* ost = reinterpret_cast<bf16*>(smem + StateTcSmem::OST);
  auto issue = [&](int ci) {
    unsigned char* base = smem + (ci % StateTcSmem::NSTAGE) * StateTcSmem::STAGE;
    int t0 = bos + ci * C;
    int nv = min(C, eos - t0);
    tc::load_tile_sw128(base + StateTcSmem::W, P.W, t0, nv, H, h);
    tc::load_tile_sw128(base + StateTcSmem::QT, P.Qt, t0, nv, H, h);
    tc::load_tile_sw128(base + StateTcSmem::KB, P.Kb, t0, nv, H, h);
    tc::load_tile_sw128(base + StateTcSmem::U, P.U, t0, nv, H, h);
    tc::load_tile64_sw128(base + StateTcSmem::M, P.M, t0, nv, H, h);
    load_vec128(reinterpret_cast<float*>(base + StateTcSmem::DC), P.dC + ((size_t)(cbase + ci) * H + h) * D);
  };
  // one cp.async group per chunk (empty groups past the end keep the count uniform)
  if (nchunks > 0) issue(0);
  cp_async_commit();
  cp_async_wait<0>();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
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
  // the same row -> chunk-start state tile of the backward (st128 order)
  auto store_hs = [&](const float (&v)[64], int chunk) {
    if (!P.hs) return;
    bf16* dst = P.hs + tile_index(P.seq, chunk, h) * STATE_ELEMS;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 pk;
      pk.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
      pk.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
      pk.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
      pk.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
      *reinterpret_cast<uint4*>(dst + st128_off(krow, 64 * half + 8 * c)) = pk;
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
    for (int i = tid; i < 64 * 16; i += blockDim.x) {
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
  __syncthreads();

  bool ok = true;
  for (int ci = 0; ci < nchunks && ok; ++ci) {
    unsigned char* buf = smem + (ci % StateTcSmem::NSTAGE) * StateTcSmem::STAGE;
    const bool last = ci + 1 == nchunks;
    const int eo = ci & 1;
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
    }
    // S <- diag(2^Gam_C) S in TMEM from the registers; chunk-start state out
    {
      const float dc = reinterpret_cast<const float*>(buf + StateTcSmem::DC)[krow];
      float a[32], b[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) { a[i] = v[i] * dc; b[i] = v[32 + i] * dc; }
      tc::tmem_st32(tS, a);
      tc::tmem_st32(tS + 32, b);
      store_hs(v, cbase + ci);
    }
    if (ci > 0) stage_o(eo ^ 1);  // o of the previous chunk (its MMAs are complete)
    // stage (ci+1)%2 held chunk ci-1, whose MMAs are finished
    if (!last) issue(ci + 1);
    cp_async_commit();
    if (!tc::mbar_wait(mbarE, ci & 1)) *abort_flag = 1;
    tc::fence_after_sync();
    // E = U - E_acc (threads holding E rows: lanes 0-15)
    {
      const int r = arow;
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
            uint4 e;
            e.x = pack_bf16(u0.x - acc[8 * c + 0], u0.y - acc[8 * c + 1]);
            e.y = pack_bf16(u1.x - acc[8 * c + 2], u1.y - acc[8 * c + 3]);
            e.z = pack_bf16(u2.x - acc[8 * c + 4], u2.y - acc[8 * c + 5]);
            e.w = pack_bf16(u3.x - acc[8 * c + 6], u3.y - acc[8 * c + 7]);
            *reinterpret_cast<uint4*>(eat + off) = e;
            if (P.E)  // whole tile: rows past the end are zero
              *reinterpret_cast<uint4*>(P.E + tile_index(P.seq, cbase + ci, h) * TILE64_ELEMS +
                                        acc64_off(r, 64 * half + 8 * chunk)) = e;
          }
        }
      }
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    if (*abort_flag) { ok = false; break; }
    // O += M E ; S += Kbar^T E
    if (tid == 0) {
      tc::fence_after_sync();
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
    // the next chunk's inputs (its decay and operands are needed next)
    cp_async_wait<0>();
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
    __syncthreads();
    if (*abort_flag) ok = false;
  }
  if (ok && nchunks > 0) {  // o of the last chunk
    stage_o((nchunks - 1) & 1);
    __syncthreads();
    copy_o(nchunks - 1);
  }
  if (!ok && tid == 0) atomicExch(&g_kda_device_error, 1);
  cp_async_wait<0>();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

}  // namespace kda
