// Shared device helpers for the KDA kernels (sm_100a).
//
// Tile conventions used by every kernel:
//   * chunk of C = 64 tokens, head dim D = 128, sub-chunks of 16 tokens;
//   * tensor-core operands are 128B-swizzled bf16 tiles (sw64_chunk below and
//     kda_tc.cuh); the warp-level products are the tf32 16x16 blocks of the
//     UT inverse (mma.sync m16n8k8);
//   * staged output rows use a padded row stride (LD128 = 136 elements);
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

// ---------------------------------------------------------------- tile layouts
// Per-(chunk, head) tiles that a kernel consumes as tcgen05 operands are stored
// in the 128B-swizzled operand layout (sw64_chunk), so one bulk copy lands them.
// The dQt and dKbar tiles, which the backward chunk kernel reads element-wise,
// are stored in the order their producing epilogue holds them, so that every
// warp store is one contiguous run.
// Offsets are in elements; (i, v) is row, column and every chunk of 8
// consecutive columns is contiguous.
//   acc64: a 64x128 tile produced from an M=64 TMEM accumulator (row i sits in
//          lane i%16 of warp quarter i/16; each thread holds 32-column blocks):
//          [quarter 4][column half 2][32-block 2][8-chunk 4][row lane 16][8]
constexpr int TILE64_ELEMS = 64 * 128;
constexpr int TILE64N64_ELEMS = 64 * 64;
constexpr int A_TILE_ELEMS = 64 * LDF64;  // saved A: [64][LDF64] fp32, the inverse's own padded rows
constexpr int STATE_ELEMS = 128 * 128;
__host__ __device__ __forceinline__ uint32_t acc64_off(int i, int v) {
  return (uint32_t)((((((i >> 4) * 2 + (v >> 6)) * 2 + ((v >> 5) & 1)) * 4 + ((v >> 3) & 3)) * 16 + (i & 15)) * 8 +
                    (v & 7));
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
