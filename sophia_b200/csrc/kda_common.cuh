// Shared device helpers for the KDA kernels (sm_100a).
//
// Tile conventions used by every kernel:
//   * chunk of C = 64 tokens, head dim D = 128, sub-chunks of 16 tokens;
//   * bf16 tiles in shared memory are row-major with a padded row stride
//     (136 elements for 128-wide rows, 72 for 64-wide rows) so that eight
//     ldmatrix row addresses hit eight distinct 4-bank groups;
//   * warp-level tensor-core products use mma.sync m16n8k16 (bf16 in, fp32
//     accumulate) with fragments loaded by ldmatrix; the four operand
//     orientations (A or A^T, B or B^T) map to ldmatrix with or without .trans.
//   * decays are kept in log2 units (Gam2 = Gam / ln 2) so every exponential is
//     one ex2.approx.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kda {

constexpr int C = 64;        // chunk length
constexpr int D = 128;       // head dim (K = V = 128)
constexpr int SUB = 16;      // sub-chunk length
constexpr int LD128 = 136;   // padded row stride (elements) of 128-wide bf16 tiles
constexpr int LD64 = 72;     // padded row stride (elements) of 64-wide bf16 tiles
constexpr int LDF64 = 65;    // padded row stride (floats) of 64x64 fp32 tiles
constexpr int LDG = 132;     // padded row stride (floats) of the 64x128 fp32 decay tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

typedef __nv_bfloat16 bf16;

// ---------------------------------------------------------------- sequences
// Sequence n spans tokens [bos, eos) of the flattened [B*T] token axis.  Without
// cu_seqlens every sequence has T tokens; with it, the device-built chunk table
// maps a global chunk index to its sequence.
struct SeqInfo {
  const int* cu_seqlens;     // [N+1] or nullptr
  const int* chunk_offsets;  // [N+1] prefix sums of ceil(len/64) (varlen only)
  const int* chunk_seq;      // [max_chunks] sequence id per chunk (varlen only)
  int N;                     // number of sequences
  int T;                     // tokens per sequence when cu_seqlens == nullptr
  int nt;                    // chunks per sequence when cu_seqlens == nullptr
  int slots;                 // chunk slots per head of the per-(chunk, head) tile arrays
};

// Tile of (global chunk c, head h) in a per-(chunk, head) tile array: head-major,
// so one head's chunks (read by consecutive chunk-kernel CTAs, written in order
// by one state-kernel CTA) are adjacent.
__device__ __forceinline__ size_t tile_index(const SeqInfo& s, int c, int h) { return (size_t)h * s.slots + c; }

struct ChunkPos {
  int seq;     // sequence id
  int idx;     // chunk index inside the sequence
  int bos;     // first token of the sequence
  int t0;      // first token of the chunk
  int t1;      // one past the last valid token of the chunk
  bool valid;  // false for grid slots beyond the real chunk count
};

__device__ __forceinline__ int seq_bos(const SeqInfo& s, int n) {
  return s.cu_seqlens ? s.cu_seqlens[n] : n * s.T;
}
__device__ __forceinline__ int seq_eos(const SeqInfo& s, int n) {
  return s.cu_seqlens ? s.cu_seqlens[n + 1] : (n + 1) * s.T;
}
__device__ __forceinline__ int seq_chunk_base(const SeqInfo& s, int n) {
  return s.cu_seqlens ? s.chunk_offsets[n] : n * s.nt;
}
// Chunks of sequence n (0 for every sequence when the packed table is invalid).
__device__ __forceinline__ int seq_nchunks(const SeqInfo& s, int n) {
  return s.cu_seqlens ? s.chunk_offsets[n + 1] - s.chunk_offsets[n] : s.nt;
}

__device__ __forceinline__ ChunkPos chunk_pos(const SeqInfo& s, int c) {
  ChunkPos p;
  int total = s.cu_seqlens ? s.chunk_offsets[s.N] : s.N * s.nt;
  p.valid = c < total;
  if (!p.valid) { p.seq = 0; p.idx = 0; p.bos = 0; p.t0 = 0; p.t1 = 0; return p; }
  if (s.cu_seqlens) {
    p.seq = s.chunk_seq[c];
    p.idx = c - s.chunk_offsets[p.seq];
  } else {
    p.seq = c / s.nt;
    p.idx = c - p.seq * s.nt;
  }
  p.bos = seq_bos(s, p.seq);
  int eos = seq_eos(s, p.seq);
  p.t0 = p.bos + p.idx * C;
  p.t1 = min(p.t0 + C, eos);
  return p;
}

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  uint32_t s = smem_u32(smem);
  int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A(16x8 tf32, row) * B(8x8 tf32, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma1688_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
// logistic sigmoid from ex2 and rcp (relative error ~1e-7)
__device__ __forceinline__ float sigmoidf_(float x) { return rcp(1.f + ex2(-x * LOG2E)); }

// Sigmoid and SiLU through one tanh.approx: sigmoid(x) = (1 + tanh(x/2)) / 2,
// x * sigmoid(x) = h + h tanh(h) with h = x/2.  tanh.approx.f32 has a relative
// error below 2^-10.9, under the bf16 rounding the results go through; used for
// the ShortConv activation, where the forward and backward kernels must agree.
__device__ __forceinline__ float tanh_fast(float x) {
  float t;
  asm("tanh.approx.f32 %0, %1;\n" : "=f"(t) : "f"(x));
  return t;
}
__device__ __forceinline__ float sigmoid_fast(float x) { return fmaf(0.5f, tanh_fast(0.5f * x), 0.5f); }
__device__ __forceinline__ float silu_fast(float x) {
  float h = 0.5f * x;
  return fmaf(h, tanh_fast(h), h);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float2 unpack_bf16(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// ---------------------------------------------------------------- fragments
// A fragment (16x16) from a row-major [m][k] tile.
__device__ __forceinline__ void load_A(uint32_t (&a)[4], const bf16* base, int ld, int m0, int k0) {
  int l = threadIdx.x & 31;
  ldsm_x4(a, base + (m0 + (l & 15)) * ld + k0 + (l >> 4) * 8);
}
// A fragment of A = X^T where X is a row-major [k][m] tile.
__device__ __forceinline__ void load_AT(uint32_t (&a)[4], const bf16* base, int ld, int m0, int k0) {
  int l = threadIdx.x & 31;
  int i = l >> 3, r = l & 7;
  ldsm_x4_t(a, base + (k0 + (i >> 1) * 8 + r) * ld + m0 + (i & 1) * 8);
}
// B fragments for two adjacent n8 tiles (n0, n0+8) of B = Y^T where Y is a
// row-major [n][k] tile.  b[0..1] -> tile n0, b[2..3] -> tile n0+8.
__device__ __forceinline__ void load_B_nk(uint32_t (&b)[4], const bf16* base, int ld, int n0, int k0) {
  int l = threadIdx.x & 31;
  int i = l >> 3, r = l & 7;
  ldsm_x4(b, base + (n0 + (i >> 1) * 8 + r) * ld + k0 + (i & 1) * 8);
}
// B fragments for two adjacent n8 tiles from a row-major [k][n] tile.
__device__ __forceinline__ void load_B_kn(uint32_t (&b)[4], const bf16* base, int ld, int n0, int k0) {
  int l = threadIdx.x & 31;
  int i = l >> 3, r = l & 7;
  ldsm_x4_t(b, base + (k0 + (i & 1) * 8 + r) * ld + n0 + (i >> 1) * 8);
}

// Warp product acc[16 x (8*NT)] += op(A)[16 x K] * op(B)[K x (8*NT)].
//   TA = false: A is a row-major [m][k] tile; TA = true: A = X^T, X row-major [k][m].
//   TB = false: B = Y^T, Y row-major [n][k];  TB = true: B row-major [k][n].
template <int NT, bool TA, bool TB>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], const bf16* A, int lda, int m0,
                                         const bf16* B, int ldb, int n0, int k0, int K) {
  static_assert(NT % 2 == 0, "NT must be even");
#pragma unroll 2
  for (int kk = 0; kk < K; kk += 16) {
    uint32_t a[4];
    if (TA) load_AT(a, A, lda, m0, k0 + kk); else load_A(a, A, lda, m0, k0 + kk);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      if (TB) load_B_kn(b, B, ldb, n0 + 8 * j, k0 + kk); else load_B_nk(b, B, ldb, n0 + 8 * j, k0 + kk);
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}

// The same fragment loads for tiles in other layouts: a tile type provides
// at(row, col) for col a multiple of 8 (the start of a contiguous 16-byte run).
// As warp_mma with A negated (sign bits of the bf16 A fragments flipped).
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

struct PadTile {  // row-major with a padded row stride
  const bf16* p;
  int ld;
  __device__ __forceinline__ const bf16* at(int r, int c) const { return p + r * ld + c; }
};
struct Acc64Tile;  // defined with the tile layouts below

template <int NT, bool TA, bool TB, typename TAL, typename TBL>
__device__ __forceinline__ void warp_mma_t(float (&acc)[NT][4], const TAL& A, int m0, const TBL& B, int n0, int k0,
                                           int K) {
  static_assert(NT % 2 == 0, "NT must be even");
  const int l = threadIdx.x & 31, i = l >> 3, r = l & 7;
#pragma unroll 2
  for (int kk = 0; kk < K; kk += 16) {
    const int k = k0 + kk;
    uint32_t a[4];
    if (TA) ldsm_x4_t(a, A.at(k + (i >> 1) * 8 + r, m0 + (i & 1) * 8));
    else ldsm_x4(a, A.at(m0 + (l & 15), k + (l >> 4) * 8));
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      const int n = n0 + 8 * j;
      if (TB) ldsm_x4_t(b, B.at(k + (i & 1) * 8 + r, n + (i >> 1) * 8));
      else ldsm_x4(b, B.at(n + (i >> 1) * 8 + r, k + (i & 1) * 8));
      mma16816(acc[j], a, b[0], b[1]);
      mma16816(acc[j + 1], a, b[2], b[3]);
    }
  }
}

template <int NT>
__device__ __forceinline__ void zero_acc(float (&acc)[NT][4]) {
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
}

// Row/col of accumulator element e (0..3) of n8 tile j for this lane.
// Transposes the 4x4 matrix of 32-bit words held by a lane quad (lane t holds
// row t) with two xor-shuffle rounds: afterwards lane t holds column t.  For
// an accumulator row packed as w[j] = bf16 pair at columns 8j + 2t, 8j + 2t + 1
// this leaves lane t with the eight consecutive columns 8t .. 8t + 7.
__device__ __forceinline__ void quad_transpose4(uint32_t (&w)[4]) {
  const int t = threadIdx.x & 3;
  const bool hi2 = t & 2, hi1 = t & 1;
  uint32_t a0 = hi2 ? w[0] : w[2], a1 = hi2 ? w[1] : w[3];
  uint32_t b0 = __shfl_xor_sync(0xffffffffu, a0, 2), b1 = __shfl_xor_sync(0xffffffffu, a1, 2);
  if (hi2) { w[0] = b0; w[1] = b1; } else { w[2] = b0; w[3] = b1; }
  a0 = hi1 ? w[0] : w[1];
  a1 = hi1 ? w[2] : w[3];
  b0 = __shfl_xor_sync(0xffffffffu, a0, 1);
  b1 = __shfl_xor_sync(0xffffffffu, a1, 1);
  if (hi1) { w[0] = b0; w[2] = b1; } else { w[1] = b0; w[3] = b1; }
}

__device__ __forceinline__ int acc_row(int e) { return ((threadIdx.x & 31) >> 2) + ((e >> 1) << 3); }
__device__ __forceinline__ int acc_col(int j, int e) { return 8 * j + 2 * (threadIdx.x & 3) + (e & 1); }

// 16-byte vector of 8 bf16
// ---------------------------------------------------------------- tile layouts
// Per-(chunk, head) tiles exchanged between the state kernels and the chunk
// kernels are stored in the order their producing epilogue holds them, so that
// every warp store is one contiguous run; consumers gather 16-byte chunks.
// Offsets are in elements; (i, v) is row, column and every chunk of 8
// consecutive columns is contiguous.
//   acc64: a 64x128 tile produced from an M=64 TMEM accumulator (row i sits in
//          lane i%16 of warp quarter i/16; each thread holds 32-column blocks):
//          [quarter 4][column half 2][32-block 2][8-chunk 4][row lane 16][8]
//   acc64n64: a 64x64 tile from an N=64 M=64 accumulator (32 columns/thread):
//          [quarter 4][column half 2][8-chunk 4][row lane 16][8]
//   st128: a 128x128 state (row k in lane k%32 of warp quarter k/32):
//          [quarter 4][column half 2][8-chunk 8][row lane 32][8]
constexpr int TILE64_ELEMS = 64 * 128;
constexpr int TILE64N64_ELEMS = 64 * 64;
constexpr int A_TILE_ELEMS = 64 * LDF64;  // saved A: [64][LDF64] fp32, the inverse's own padded rows
constexpr int STATE_ELEMS = 128 * 128;
__host__ __device__ __forceinline__ uint32_t acc64_off(int i, int v) {
  return (uint32_t)((((((i >> 4) * 2 + (v >> 6)) * 2 + ((v >> 5) & 1)) * 4 + ((v >> 3) & 3)) * 16 + (i & 15)) * 8 +
                    (v & 7));
}
__host__ __device__ __forceinline__ uint32_t acc64n64_off(int i, int j) {
  return (uint32_t)(((((i >> 4) * 2 + (j >> 5)) * 4 + ((j >> 3) & 3)) * 16 + (i & 15)) * 8 + (j & 7));
}
__host__ __device__ __forceinline__ uint32_t st128_off(int k, int v) {
  return (uint32_t)(((((k >> 5) * 2 + (v >> 6)) * 8 + ((v >> 3) & 7)) * 32 + (k & 31)) * 8 + (v & 7));
}
// A 64x128 acc64 tile in shared memory, as it arrives by a plain byte copy:
// the eight rows an ldmatrix reads (one 16-row group, one 8-column chunk) are
// one contiguous 128-byte run, so the reads are conflict-free.
struct Acc64Tile {
  const bf16* p;
  __device__ __forceinline__ const bf16* at(int r, int c) const { return p + acc64_off(r, c); }
};
// Inverse maps of a 16-byte chunk index (element offset / 8) to (row, 8-chunk).
__device__ __forceinline__ void acc64_chunk(int idx, int& row, int& cc) {
  const int lane = idx & 15, c = (idx >> 4) & 3, c0 = (idx >> 6) & 1, hf = (idx >> 7) & 1, q = idx >> 8;
  row = 16 * q + lane;
  cc = hf * 8 + c0 * 4 + c;
}
__device__ __forceinline__ void acc64n64_chunk(int idx, int& row, int& cc) {
  const int lane = idx & 15, c = (idx >> 4) & 3, hf = (idx >> 6) & 1, q = idx >> 7;
  row = 16 * q + lane;
  cc = hf * 4 + c;
}
__device__ __forceinline__ void st128_chunk(int idx, int& row, int& cc) {
  const int lane = idx & 31, c = (idx >> 5) & 7, hf = (idx >> 8) & 1, q = idx >> 9;
  row = 32 * q + lane;
  cc = hf * 8 + c;
}

// Element offset of 16-byte chunk c8 (columns 8*c8 .. 8*c8+7) of row r in a
// 128B-swizzled bf16 tile of 64 rows: 64-column atoms of 64 x 128 bytes one
// after the other, chunk position c8 ^ (r & 7) inside a row (the tcgen05
// operand layout of kda_tc.cuh).
__host__ __device__ __forceinline__ uint32_t sw64_chunk(int r, int c8) {
  return (uint32_t)((c8 >> 3) * 4096 + r * 64 + (((c8 & 7) ^ (r & 7)) << 3));
}

struct alignas(16) bf16x8 { uint32_t u[4]; };

__device__ __forceinline__ void unpack8(const bf16x8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) { float2 p = unpack_bf16(v.u[i]); f[2 * i] = p.x; f[2 * i + 1] = p.y; }
}
__device__ __forceinline__ bf16x8 pack8(const float (&f)[8]) {
  bf16x8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.u[i] = pack_bf16(f[2 * i], f[2 * i + 1]);
  return v;
}

}  // namespace kda
