// Fifth-generation tensor-core (tcgen05) helpers for sm_100a: shared-memory
// matrix descriptors, instruction descriptors, TMEM allocation, MMA issue,
// completion tracking with mbarriers (every wait bounded) and TMEM <-> register
// moves.
//
// Operand tiles use the 128-byte swizzled canonical layouts:
//   * a row-major [rows][cols] bf16 tile is stored as column blocks of 64
//     elements ("atoms": rows x 128 bytes each, atom after atom); inside an
//     atom, row r occupies bytes [128 r, 128 r + 128) and its 16-byte chunk c
//     sits at chunk position c ^ (r & 7);
//   * K-major view (rows = M or N index, 64 K elements per atom row): 8-row
//     groups are SBO = 1024 bytes apart; the K step of 16 elements advances
//     the start address by 32 bytes inside an atom, by the atom size across;
//   * MN-major view (rows = K index, 64 M/N elements per atom row): 8-row K
//     groups are SBO = 1024 bytes apart, the next 64 M/N elements (next atom)
//     are LBO = atom size bytes apart; a K step of 16 advances by 2048 bytes.
// So the same [token][channel] tile serves as a K-major operand (channels as
// K) and as an MN-major operand (tokens as K).
#pragma once

#include <cuda.h>  // CUtensorMap

#include "kda_common.cuh"

namespace kda {

__device__ int g_kda_device_error;  // nonzero after a bounded wait timed out

namespace tc {

// 16-byte chunk position of element column `col` (0..63) of row `r` inside a
// 128B-swizzled atom, in bytes.
__device__ __forceinline__ uint32_t sw128_offset(int r, int col) {
  return (uint32_t)(r * 128 + ((((col >> 3) ^ (r & 7))) << 4) + ((col & 7) << 1));
}

// Shared-memory matrix descriptor (SWIZZLE_128B, descriptor version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, dense.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                          // D format f32
         | (1u << 7)                        // A format bf16
         | (1u << 10)                       // B format bf16
         | ((a_mn_major ? 1u : 0u) << 15)   // A major
         | ((b_mn_major ? 1u : 0u) << 16)   // B major
         | ((uint32_t)(N >> 3) << 17)       // N
         | ((uint32_t)(M >> 4) << 24);      // M
}

// TMEM allocation by one full warp; the column base is written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}

// D[tmem] (+)= A[smem] * B[smem], issued by a single thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate));
}

// Arrive on an mbarrier when all previously issued MMAs of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
      smem_u32(mbar)));
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::); }
// Generic-proxy shared-memory writes -> visible to the tensor cores.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::); }

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(mbar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::); }

// Waits for phase `parity` of the mbarrier to complete, polling at most
// `max_polls` times.  Returns false on timeout (the caller records an error
// and takes its exit path instead of spinning forever).
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t max_polls = (1u << 26)) {
  uint32_t addr = smem_u32(mbar);
  for (uint32_t i = 0; i < max_polls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

// One thread announces `bytes` of bulk-copy traffic on the mbarrier (and
// arrives on it); the copies complete the phase when all bytes have landed.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(mbar)), "r"(bytes)
               : "memory");
}
// Tiled TMA load of one box of a rank-3 tensor map (no swizzle; this CTA only)
// into shared memory; out-of-range elements arrive as zeros.  The map lives in
// kernel-parameter space (__grid_constant__); the innermost coordinate c0 must
// be a multiple of 16 bytes' worth of elements.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(mbar))
      : "memory");
}
// Bulk (TMA, non-tensor) copy of a contiguous global range into shared memory;
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(mbar))
      : "memory");
}

// Bulk (TMA, non-tensor) copy of a contiguous shared range to global memory,
// tracked by this thread's bulk async-groups.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Waits until this thread's bulk groups have completed (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// Waits until this thread's bulk stores have finished reading their shared-memory
// sources (the writes to global memory may still be in flight): enough to reuse the source.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
}

// 32 lanes x 32 consecutive fp32 columns: this thread gets its lane's columns
// [col, col + 32).  taddr = (lane base << 16) | column.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 8 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// tmem_ld8 without the completion wait: several loads can be in flight; the
// values are valid only after tmem_wait8 on them (the wait takes the registers
// as operands, so nothing reads them before it).
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait8(float (&v)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+f"(v[0]), "+f"(v[1]), "+f"(v[2]), "+f"(v[3]), "+f"(v[4]), "+f"(v[5]), "+f"(v[6]), "+f"(v[7])
               :
               : "memory");
}

// 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])));
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// cp.async of a [64 rows][128 cols] bf16 global tile (rows t0 + r of head h in a
// [T][H][128] tensor) into two 128B-swizzled atoms (cols 0-63 at dst, 64-127 at
// dst + 8192); rows r >= nvalid are zero-filled.
__device__ __forceinline__ void load_tile_sw128(unsigned char* dst, const bf16* src, int t0, int nvalid, int H, int h) {
  for (int i = threadIdx.x; i < 64 * 16; i += blockDim.x) {
    int r = i >> 4, cc = i & 15;
    bool ok = r < nvalid;
    const bf16* gp = src + (ok ? ((size_t)(t0 + r) * H + h) * D + cc * 8 : 0);
    unsigned char* sp = dst + (cc >> 3) * 8192 + r * 128 + (((cc & 7) ^ (r & 7)) << 4);
    cp_async16(sp, gp, ok);
  }
}
// Same for a [64][64] tile (one atom).
__device__ __forceinline__ void load_tile64_sw128(unsigned char* dst, const bf16* src, int t0, int nvalid, int H, int h) {
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    int r = i >> 3, cc = i & 7;
    bool ok = r < nvalid;
    const bf16* gp = src + (ok ? ((size_t)(t0 + r) * H + h) * 64 + cc * 8 : 0);
    cp_async16(dst + r * 128 + ((cc ^ (r & 7)) << 4), gp, ok);
  }
}

}  // namespace tc
}  // namespace kda
