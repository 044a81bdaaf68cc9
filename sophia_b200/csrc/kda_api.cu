// C ABI of the KDA layer (declared in include/kda_b200.h): argument checks,
// buffer carving and kernel launches.  No allocation, no host sync.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kda_b200.h"
#include "kda_bwd_intra.cuh"
#include "kda_fwd_state_tc.cuh"
#include "kda_bwd_state_tc.cuh"
#include "kda_recurrent.cuh"
#include "kda_post.cuh"
#include "kda_gated_norm.cuh"
#include "kda_f32.cuh"
#include "kda_pack.cuh"

using namespace kda;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int64_t max_chunks(int64_t tokens, int N) { return tokens / C + N; }

// Sub-buffer carving of a caller buffer.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* p) : base(static_cast<char*>(p)) {}
  template <typename T>
  T* take(size_t bytes) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += align256(bytes);
    return p;
  }
};

struct SavedView {
  bf16 *W, *U, *Qt, *Kb, *E, *M, *hs;
  float* dC;
  bf16* A;   // [slots x H] bf16 64x64 swizzled tiles of A = (I + diag(beta) L')^-1 (training only)
  bf16* LP;  // [slots x H] bf16 64x64 swizzled tiles of L' (training only)
  // the forward prologue's products for the backward (training only):
  bf16 *QN, *KN, *VN;  // [slots x H] [64][128] bf16: scaled normalised q, normalised k, post-conv v
  float *GM, *BT;      // [slots x H] [64][LDG] fp32 in-chunk log2 decay cumsum, [slots x H][64] fp32 beta
};

SavedView carve_saved(Carver& cv, int64_t TT, int H, int64_t mc, bool with_bwd) {
  SavedView s;
  const size_t row = (size_t)TT * H * D * 2;
  s.W = cv.take<bf16>(row);
  s.U = cv.take<bf16>(row);
  s.Qt = cv.take<bf16>(row);
  s.Kb = cv.take<bf16>(row);
  s.M = cv.take<bf16>((size_t)TT * H * 64 * 2);
  s.dC = cv.take<float>((size_t)mc * H * D * 4);
  if (with_bwd) {
    s.E = cv.take<bf16>((size_t)mc * H * TILE64_ELEMS * 2);
    s.hs = cv.take<bf16>((size_t)mc * H * STATE_ELEMS * 2);
    s.A = cv.take<bf16>((size_t)mc * H * TILE64N64_ELEMS * 2);
    s.LP = cv.take<bf16>((size_t)mc * H * TILE64N64_ELEMS * 2);
    s.QN = cv.take<bf16>((size_t)mc * H * TILE64_ELEMS * 2);
    s.KN = cv.take<bf16>((size_t)mc * H * TILE64_ELEMS * 2);
    s.VN = cv.take<bf16>((size_t)mc * H * TILE64_ELEMS * 2);
    s.GM = cv.take<float>((size_t)mc * H * 64 * LDG * 4);
    s.BT = cv.take<float>((size_t)mc * H * 64 * 4);
  } else {
    s.E = nullptr;
    s.hs = nullptr;
    s.A = nullptr;
    s.LP = nullptr;
    s.QN = s.KN = s.VN = nullptr;
    s.GM = s.BT = nullptr;
  }
  return s;
}

struct Table {
  int* offsets;
  int* chunk_seq;
  int* err;
  int* item_counter;  // the forward chunk kernel's dynamic item counter
};

Table carve_table(Carver& cv, int N, int64_t mc) {
  Table t;
  t.offsets = cv.take<int>((size_t)(N + 1) * 4);
  t.chunk_seq = cv.take<int>((size_t)mc * 4);
  t.err = cv.take<int>(4);
  t.item_counter = cv.take<int>(4);
  return t;
}

struct BwdView {
  bf16 *dE, *dQt, *dW, *dKb, *dM, *dq_hat, *dk_hat, *dv_hat;
  float *dGC, *partA, *partB, *partW;
};

BwdView carve_bwd(Carver& cv, int64_t TT, int H, int64_t mc) {
  BwdView b;
  const size_t row = (size_t)TT * H * D * 2;
  const size_t tile = (size_t)mc * H * TILE64_ELEMS * 2;
  b.dE = cv.take<bf16>(tile);
  b.dQt = cv.take<bf16>(tile);
  b.dW = cv.take<bf16>(tile);
  b.dKb = cv.take<bf16>(tile);
  b.dq_hat = cv.take<bf16>(row);
  b.dk_hat = cv.take<bf16>(row);
  b.dv_hat = cv.take<bf16>(row);
  b.dM = cv.take<bf16>((size_t)mc * H * TILE64N64_ELEMS * 2);
  b.dGC = cv.take<float>((size_t)mc * H * D * 4);
  b.partA = cv.take<float>((size_t)mc * H * D * 4);
  b.partB = cv.take<float>((size_t)mc * H * D * 4);
  b.partW = cv.take<float>((size_t)mc * 3 * H * D * 4 * 4);
  return b;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

struct Problem {
  int B, T, H, N;
  bool packed, conv;
  int64_t TT, mc;
  int grid_chunks;
  SeqInfo seq;
};

int check_common(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* A_log,
                 const float* dt_bias, const float* cq, const float* ck, const float* cvv, const int32_t* cu, int B,
                 int T, int H, int D_, int N, float lower_bound, Problem& pr) {
  if (D_ != D) return fail(KDA_ERR_UNSUPPORTED, "head dim must be 128, got " + std::to_string(D_));
  if (B < 1 || T < 0 || H < 1) return fail(KDA_ERR_INVALID, "B >= 1, T >= 0 and H >= 1 are required");
  if (!(lower_bound >= -5.f && lower_bound < 0.f))
    return fail(KDA_ERR_INVALID, "`lower_bound` must be in the safe range [-5, 0), got " + std::to_string(lower_bound));
  const bool empty = (int64_t)B * T == 0;  // empty tensors may have null data
  if (!empty && (!q || !k || !v || !g || !beta || !A_log || !dt_bias)) return fail(KDA_ERR_INVALID, "null input pointer");
  const bool anyconv = cq || ck || cvv, allconv = cq && ck && cvv;
  if (anyconv && !allconv) return fail(KDA_ERR_INVALID, "conv taps must be given for all of q, k, v or none");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(g, 16))
    return fail(KDA_ERR_INVALID, "q, k, v and g must be 16-byte aligned");
  if (!aligned(dt_bias, 16)) return fail(KDA_ERR_INVALID, "dt_bias must be 16-byte aligned");
  if (allconv && (!aligned(cq, 16) || !aligned(ck, 16) || !aligned(cvv, 16)))
    return fail(KDA_ERR_INVALID, "conv taps must be 16-byte aligned");
  if (cu) {
    if (B != 1)
      return fail(KDA_ERR_INVALID, "The batch size is expected to be 1 rather than " + std::to_string(B) +
                                       " when using `cu_seqlens`.");
    if (N < 1) return fail(KDA_ERR_INVALID, "N >= 1 sequences are required with cu_seqlens");
  } else if (N != B) {
    return fail(KDA_ERR_INVALID, "N must equal B without cu_seqlens");
  }
  pr.B = B; pr.T = T; pr.H = H; pr.N = N;
  pr.packed = cu != nullptr;
  pr.conv = allconv;
  pr.TT = (int64_t)B * T;
  pr.mc = max_chunks(pr.TT, N);
  pr.seq.cu_seqlens = cu;
  pr.seq.chunk_offsets = nullptr;
  pr.seq.chunk_seq = nullptr;
  pr.seq.N = N;
  pr.seq.T = T;
  pr.seq.nt = (T + C - 1) / C;
  pr.seq.slots = (int)pr.mc;
  pr.grid_chunks = pr.packed ? (int)pr.mc : B * pr.seq.nt;
  if (pr.mc > (int64_t)INT32_MAX / 2) return fail(KDA_ERR_INVALID, "too many tokens");
  return KDA_OK;
}

// ---- optional per-launch device timing (CUDA events on the launch stream)
enum KernelId {
  K_TABLE = 0, K_FWD_INTRA, K_FWD_STATE, K_BWD_STATE, K_BWD_INTRA, K_BWD_POST, K_REDUCE, K_RECURRENT,
  K_GNORM_FWD, K_GNORM_BWD, K_F32_PREP, K_F32_FWD, K_F32_BWD, K_F32_DC, K_F32_CONV, K_DOC_BOUNDS, K_COUNT
};
const char* const kKernelNames[K_COUNT] = {"chunk_table", "fwd_intra", "fwd_state",       "bwd_state",
                                           "bwd_intra",   "bwd_post",  "reduce",          "recurrent",
                                           "gated_norm_fwd", "gated_norm_bwd", "f32_prep", "f32_fwd",
                                           "f32_bwd",     "f32_dc",    "f32_conv_bwd",    "doc_bounds"};

struct Timing {
  std::mutex mu;
  bool on = false;
  std::vector<cudaEvent_t> pool;  // pairs (start, stop)
  std::vector<int> ids;           // kernel id of each recorded pair
  size_t used = 0;
};
Timing g_timing;

struct TimedLaunch {
  cudaEvent_t stop = nullptr;
  cudaStream_t st;
  TimedLaunch(int id, cudaStream_t s) : st(s) {
    if (!g_timing.on) return;
    std::lock_guard<std::mutex> lk(g_timing.mu);
    if (g_timing.used + 2 > g_timing.pool.size()) {
      for (int i = 0; i < 64; ++i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return;
        g_timing.pool.push_back(e);
      }
    }
    cudaEvent_t start = g_timing.pool[g_timing.used];
    stop = g_timing.pool[g_timing.used + 1];
    g_timing.used += 2;
    g_timing.ids.push_back(id);
    cudaEventRecord(start, st);
  }
  ~TimedLaunch() {
    if (stop) cudaEventRecord(stop, st);
  }
};

int launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(KDA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return KDA_OK;
}

// Poll limit of the forward chunk kernel's wait for its prefetched inputs
// (kda_b200_debug_set_input_wait_polls lowers it in tests).
constexpr uint32_t kDefaultWaitPolls = 1u << 26;
std::atomic<uint32_t> g_input_wait_polls{kDefaultWaitPolls};
// The forward state pass's test hook (kda_b200_debug_set_state_wait).
std::atomic<uint32_t> g_state_wait_polls{kDefaultWaitPolls};
std::atomic<int> g_state_withhold_loads{0};

// SMs of the current device (queried once per device).
int sm_count() {
  static std::atomic<int> counts[64];  // zero-initialised (static storage); concurrent first calls store the same value
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = counts[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
  counts[dev].store(n, std::memory_order_relaxed);
  return n;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor map of a [TT][H][128] bf16 activation whose boxes are `rows` tokens x
// 128 channels of one head (no swizzle; rows outside [0, TT) read as zeros).
int encode_rows_map(CUtensorMap* m, const void* base, int H, long long TT, int rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(KDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)TT};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2};
  const cuuint32_t box[3] = {(cuuint32_t)D, 1u, (cuuint32_t)rows};
  const cuuint32_t elem[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KDA_ERR_CUDA, "tensor map encoding failed (CUresult " + std::to_string((int)r) + ")");
  return KDA_OK;
}

// A [TT][H][inner] bf16 tensor (inner = 64 or 128) for 128B-swizzled TMA boxes of
// 64 channels x 64 rows: each box lands as one tcgen05 operand atom.
int encode_sw128_map(CUtensorMap* m, const void* base, int H, long long TT, int inner) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(KDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)H, (cuuint64_t)TT};
  const cuuint64_t strides[2] = {(cuuint64_t)inner * 2, (cuuint64_t)H * inner * 2};
  const cuuint32_t box[3] = {64u, 1u, 64u};
  const cuuint32_t elem[3] = {1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(KDA_ERR_CUDA, "tensor map encoding failed (CUresult " + std::to_string((int)r) + ")");
  return KDA_OK;
}

template <typename K>
int set_smem(K kernel, int bytes, const char* name) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(KDA_ERR_CUDA, std::string(name) + " smem attribute: " + cudaGetErrorString(e));
  return KDA_OK;
}

int build_table(Problem& pr, Table& t, cudaStream_t st) {
  if (!pr.packed) return KDA_OK;
  {
    TimedLaunch tl(K_TABLE, st);
    kda_chunk_table_kernel<<<1, 1024, 0, st>>>(pr.seq.cu_seqlens, pr.N, (long long)pr.TT, t.offsets, t.chunk_seq,
                                               t.err);
  }
  pr.seq.chunk_offsets = t.offsets;
  pr.seq.chunk_seq = t.chunk_seq;
  return launch_check("chunk table");
}

PrologueIn prologue_in(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* A_log,
                       const float* dt_bias, const float* cq, const float* ck, const float* cvv, int H, float scale,
                       float lb) {
  PrologueIn in;
  in.q = static_cast<const bf16*>(q);
  in.k = static_cast<const bf16*>(k);
  in.v = static_cast<const bf16*>(v);
  in.g = static_cast<const bf16*>(g);
  in.beta = static_cast<const bf16*>(beta);
  in.A_log = A_log;
  in.dt_bias = dt_bias;
  in.conv_q = cq;
  in.conv_k = ck;
  in.conv_v = cvv;
  in.H = H;
  in.scale = scale;
  in.lower_bound = lb;
  return in;
}

// ---- fp32 mode: buffer carving
struct F32SavedView {
  float *qh, *kh, *alpha, *r, *bt, *ck;
};

// Training: everything the backward reads.  Inference (with_bwd = false): the
// prep outputs only (no r, no chunk-start states).
F32SavedView carve_f32_saved(Carver& cv, int64_t TT, int H, int64_t mc, bool with_bwd) {
  F32SavedView s;
  const size_t row = (size_t)TT * H * D * 4;
  s.qh = cv.take<float>(row);
  s.kh = cv.take<float>(row);
  s.alpha = cv.take<float>(row);
  s.bt = cv.take<float>((size_t)TT * H * 4);
  s.r = with_bwd ? cv.take<float>(row) : nullptr;
  s.ck = with_bwd ? cv.take<float>((size_t)mc * H * STATE_ELEMS * 4) : nullptr;
  return s;
}

struct F32BwdView {
  float *dqh_p, *dkh_p, *dal_p, *dbt_p, *dvh, *dcq, *dck, *dcv, *partA, *partB, *partW, *scratch;
};

// Persistent grid of the fp32 backward recurrence: up to four CTAs per SM (the
// register limit of its 128-thread CTAs), so that up to 4 x SMs items run at once;
// each CTA owns one F32_SCRATCH_FLOATS slice of the scratch.
constexpr int F32_BWD_CTAS_PER_SM = 4;
int f32_bwd_ctas(int64_t items) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(items, F32_BWD_CTAS_PER_SM * (int64_t)sm_count()));
}

F32BwdView carve_f32_bwd(Carver& cv, int64_t TT, int H, int N, int64_t mc) {
  F32BwdView b;
  const size_t row = (size_t)TT * H * D * 4;
  b.dqh_p = cv.take<float>(F32_GROUPS * row);
  b.dkh_p = cv.take<float>(F32_GROUPS * row);
  b.dal_p = cv.take<float>(F32_GROUPS * row);
  b.dbt_p = cv.take<float>((size_t)F32_GROUPS * TT * H * 4);
  b.dvh = cv.take<float>(row);
  b.dcq = cv.take<float>(row);
  b.dck = cv.take<float>(row);
  b.dcv = cv.take<float>(row);
  b.partA = cv.take<float>((size_t)mc * H * D * 4);
  b.partB = cv.take<float>((size_t)mc * H * D * 4);
  b.partW = cv.take<float>((size_t)mc * 3 * H * D * 4 * 4);
  b.scratch = cv.take<float>((size_t)f32_bwd_ctas((int64_t)N * H * F32_GROUPS) * F32_SCRATCH_FLOATS * 4);
  return b;
}

F32Inputs f32_inputs(const float* q, const float* k, const float* v, const float* g, const float* beta,
                     const float* A_log, const float* dt_bias, const float* cq, const float* ck, const float* cvv, int H,
                     bool conv, float scale, float lb) {
  F32Inputs in;
  in.q = q; in.k = k; in.v = v; in.g = g; in.beta = beta;
  in.A_log = A_log;
  in.dt_bias = dt_bias;
  in.conv_q = cq; in.conv_k = ck; in.conv_v = cvv;
  in.H = H;
  in.conv = conv;
  in.scale = scale;
  in.lower_bound = lb;
  return in;
}

int row_grid(const Problem& pr) { return (pr.grid_chunks + F32_WARPS_PER_CTA - 1) / F32_WARPS_PER_CTA; }

}  // namespace

// ---- gated output norm of the mixer (attention.py:416-419, ops.py:49-64)
namespace {
// One wave: as many CTAs as fit on the device at once (grid-stride loops inside).
template <typename K>
int gn_resident(K kernel) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, GN_THREADS, 0) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  return per_sm * sm_count();
}
int gn_grid(long long rows, bool bwd) {
  const long long steps = ((rows + 1) / 2 + GN_THREADS / 32 - 1) / (GN_THREADS / 32);
  const int resident = bwd ? gn_resident(kda_gated_norm_bwd_kernel) : gn_resident(kda_gated_norm_fwd_kernel);
  return (int)std::max<long long>(1, std::min<long long>(steps, resident));
}
int gn_check(long long rows, int D_, const void* a, const void* b, const float* w, const void* c, int fp32_io) {
  if (D_ != D) return fail(KDA_ERR_UNSUPPORTED, "head dim must be 128, got " + std::to_string(D_));
  if (rows < 0) return fail(KDA_ERR_INVALID, "rows must be >= 0");
  if (fp32_io != 0 && fp32_io != 1) return fail(KDA_ERR_INVALID, "fp32_io must be 0 or 1");
  if (rows == 0) return KDA_OK;  // empty tensors may have null data
  if (!a || !b || !w || !c) return fail(KDA_ERR_INVALID, "null pointer");
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(c, 16) || !aligned(w, 4))
    return fail(KDA_ERR_INVALID, "row tensors must be 16-byte aligned");
  return KDA_OK;
}
}  // namespace

extern "C" {

const char* kda_b200_version(void) { return "kda_b200 0.1.0 (sm_100a)"; }

const char* kda_b200_last_error(void) { return g_last_error.c_str(); }

size_t kda_b200_saved_bytes(int64_t total_tokens, int H, int N, int packed) {
  (void)packed;
  Carver cv(nullptr);
  carve_saved(cv, total_tokens, H, max_chunks(total_tokens, N), true);
  return cv.off;
}

size_t kda_b200_fwd_workspace_bytes(int64_t total_tokens, int H, int N, int packed, int training) {
  (void)packed;
  Carver cv(nullptr);
  int64_t mc = max_chunks(total_tokens, N);
  carve_table(cv, N, mc);
  if (!training) carve_saved(cv, total_tokens, H, mc, false);
  return cv.off;
}

size_t kda_b200_bwd_workspace_bytes(int64_t total_tokens, int H, int N, int packed) {
  (void)packed;
  Carver cv(nullptr);
  int64_t mc = max_chunks(total_tokens, N);
  carve_table(cv, N, mc);
  carve_bwd(cv, total_tokens, H, mc);
  return cv.off;
}

int kda_b200_chunk_table(const int32_t* cu_seqlens, int N, int64_t total_tokens, int32_t* offsets,
                         int32_t* chunk_seq, int32_t* error_flag, void* stream) {
  if (!cu_seqlens || !offsets || !chunk_seq || !error_flag || N < 1)
    return fail(KDA_ERR_INVALID, "chunk table needs cu_seqlens, offsets, chunk_seq, error_flag and N >= 1");
  kda_chunk_table_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(cu_seqlens, N, (long long)total_tokens,
                                                                            offsets, chunk_seq, error_flag);
  return launch_check("chunk table");
}

int kda_b200_doc_cu_seqlens(const int32_t* tokens, int64_t total_tokens, int window, int eos_id, int capacity,
                            int32_t* cu_seqlens, int32_t* n_docs, void* stream) {
  if (total_tokens < 0 || total_tokens > INT32_MAX) return fail(KDA_ERR_INVALID, "total_tokens must be in [0, 2^31)");
  if (window < 1) return fail(KDA_ERR_INVALID, "window must be >= 1");
  if (capacity < 1) return fail(KDA_ERR_INVALID, "capacity must be >= 1");
  if (!cu_seqlens || !n_docs || (total_tokens > 0 && !tokens))
    return fail(KDA_ERR_INVALID, "doc_cu_seqlens needs tokens, cu_seqlens and n_docs");
  {
    TimedLaunch tl(K_DOC_BOUNDS, static_cast<cudaStream_t>(stream));
    kda_doc_bounds_kernel<<<1, PACK_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        tokens, (long long)total_tokens, window, eos_id, capacity, cu_seqlens, n_docs);
  }
  return launch_check("doc cu_seqlens");
}

int kda_b200_recurrent(const void* q, const void* k, const void* v, const void* g, const void* beta,
                       const float* A_log, const float* dt_bias, const float* h0, const int32_t* cu_seqlens, int B,
                       int T, int H, int D_, int N, int fp32_inputs, float scale, float lower_bound, void* o,
                       float* ht, void* stream) {
  return kda_b200_decode(q, k, v, g, beta, A_log, dt_bias, nullptr, nullptr, nullptr, nullptr, h0, cu_seqlens, B, T,
                         H, D_, N, fp32_inputs, scale, lower_bound, o, ht, stream);
}

int kda_b200_decode(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                    const float* conv_v, float* conv_state, const float* h0, const int32_t* cu_seqlens, int B,
                    int T, int H, int D_, int N, int fp32_inputs, float scale, float lower_bound, void* o, float* ht,
                    void* stream) {
  const bool anyconv = conv_q || conv_k || conv_v || conv_state;
  if (anyconv && !(conv_q && conv_k && conv_v && conv_state))
    return fail(KDA_ERR_INVALID, "conv taps of q, k, v and the conv history must be given together or not at all");
  if (anyconv && (!aligned(conv_q, 16) || !aligned(conv_k, 16) || !aligned(conv_v, 16)))
    return fail(KDA_ERR_INVALID, "conv taps must be 16-byte aligned");
  if (D_ != D) return fail(KDA_ERR_UNSUPPORTED, "head dim must be 128, got " + std::to_string(D_));
  if (B < 1 || T < 0 || H < 1) return fail(KDA_ERR_INVALID, "B >= 1, T >= 0 and H >= 1 are required");
  if (!(lower_bound >= -5.f && lower_bound < 0.f))
    return fail(KDA_ERR_INVALID, "`lower_bound` must be in the safe range [-5, 0), got " + std::to_string(lower_bound));
  if (!q || !k || !v || !g || !beta || !A_log || !dt_bias || !o) return fail(KDA_ERR_INVALID, "null pointer");
  if (cu_seqlens) {
    if (B != 1)
      return fail(KDA_ERR_INVALID, "The batch size is expected to be 1 rather than " + std::to_string(B) +
                                       " when using `cu_seqlens`.");
    if (N < 1) return fail(KDA_ERR_INVALID, "N >= 1 sequences are required with cu_seqlens");
  } else if (N != B) {
    return fail(KDA_ERR_INVALID, "N must equal B without cu_seqlens");
  }
  RecurrentParams rp;
  rp.seq.cu_seqlens = cu_seqlens;
  rp.seq.chunk_offsets = nullptr;
  rp.seq.chunk_seq = nullptr;
  rp.seq.N = N;
  rp.seq.T = T;
  rp.seq.nt = (T + C - 1) / C;
  rp.seq.slots = 0;
  rp.H = H;
  rp.fp32_inputs = fp32_inputs != 0;
  rp.q = q; rp.k = k; rp.v = v; rp.g = g; rp.beta = beta;
  rp.A_log = A_log;
  rp.dt_bias = dt_bias;
  rp.h0 = h0;
  rp.scale = scale;
  rp.lower_bound = lower_bound;
  rp.o = o;
  rp.ht = ht;
  rp.total_tokens = (long long)B * T;
  rp.conv_q = conv_q; rp.conv_k = conv_k; rp.conv_v = conv_v;
  rp.conv_state = conv_state;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc;
  if ((rc = set_smem(kda_recurrent_kernel, REC_SMEM, "recurrent"))) return rc;
  {
    TimedLaunch tl(K_RECURRENT, st);
    kda_recurrent_kernel<<<dim3(N, H), REC_THREADS, REC_SMEM, st>>>(rp);
  }
  return launch_check("recurrent");
}

int kda_b200_fwd(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* A_log,
                 const float* dt_bias, const float* conv_q, const float* conv_k, const float* conv_v, const float* h0,
                 const int32_t* cu_seqlens, int B, int T, int H, int D_, int N, float scale, float lower_bound,
                 void* o, float* ht, void* saved, size_t saved_bytes, void* workspace, size_t workspace_bytes,
                 void* stream) {
  Problem pr;
  int rc = check_common(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, cu_seqlens, B, T, H, D_, N,
                        lower_bound, pr);
  if (rc) return rc;
  if (!o && pr.TT > 0) return fail(KDA_ERR_INVALID, "null output pointer");
  if (!aligned(o, 16)) return fail(KDA_ERR_INVALID, "o must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool training = saved != nullptr;
  size_t need_ws = kda_b200_fwd_workspace_bytes(pr.TT, H, N, pr.packed, training);
  if (!workspace || workspace_bytes < need_ws)
    return fail(KDA_ERR_INVALID, "workspace too small: need " + std::to_string(need_ws) + " bytes");
  if (training && saved_bytes < kda_b200_saved_bytes(pr.TT, H, N, pr.packed))
    return fail(KDA_ERR_INVALID, "saved buffer too small");
  if (pr.TT == 0) {
    if (ht) {
      size_t bytes = (size_t)N * H * D * D * 4;
      cudaError_t e = h0 ? cudaMemcpyAsync(ht, h0, bytes, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(ht, 0, bytes, st);
      if (e != cudaSuccess) return fail(KDA_ERR_CUDA, cudaGetErrorString(e));
    }
    return KDA_OK;
  }
  Carver wcv(workspace);
  Table tab = carve_table(wcv, N, pr.mc);
  Carver scv(training ? saved : nullptr);
  SavedView sv = training ? carve_saved(scv, pr.TT, H, pr.mc, true) : carve_saved(wcv, pr.TT, H, pr.mc, false);
  if ((rc = build_table(pr, tab, st))) return rc;

  FwdIntraParams ip;
  ip.in = prologue_in(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, H, scale, lower_bound);
  ip.seq = pr.seq;
  ip.conv = pr.conv;
  ip.W = sv.W; ip.U = sv.U; ip.Qt = sv.Qt; ip.Kb = sv.Kb; ip.M = sv.M; ip.dC = sv.dC; ip.A = sv.A; ip.LP = sv.LP;
  ip.QN = sv.QN; ip.KN = sv.KN; ip.VN = sv.VN; ip.GM = sv.GM; ip.BT = sv.BT;
  ip.grid_chunks = pr.grid_chunks;
  ip.item_counter = tab.item_counter;
  ip.wait_polls = g_input_wait_polls.load(std::memory_order_relaxed);
  if ((rc = encode_rows_map(&ip.maps[0], q, H, pr.TT, 67)) || (rc = encode_rows_map(&ip.maps[1], k, H, pr.TT, 67)) ||
      (rc = encode_rows_map(&ip.maps[2], v, H, pr.TT, 67)) || (rc = encode_rows_map(&ip.maps[3], g, H, pr.TT, 64)))
    return rc;
  if ((rc = set_smem(kda_fwd_intra_kernel, IntraSmem::END, "fwd intra"))) return rc;
  {
    // persistent: one CTA per SM (the shared-memory plan allows one) walks the items;
    // those past the grid come from a counter that starts at zero
    const long long items = (long long)pr.grid_chunks * H;
    if (items > INT_MAX) return fail(KDA_ERR_INVALID, "more than 2^31 (chunk, head) items");
    const int ctas = (int)std::min<long long>(items, sm_count());
    const cudaError_t e = cudaMemsetAsync(tab.item_counter, 0, sizeof(int), st);
    if (e != cudaSuccess) return fail(KDA_ERR_CUDA, std::string("item counter: ") + cudaGetErrorString(e));
    TimedLaunch tl(K_FWD_INTRA, st);
    kda_fwd_intra_kernel<<<ctas, INTRA_THREADS, IntraSmem::END, st>>>(ip);
  }
  if ((rc = launch_check("fwd intra"))) return rc;

  FwdStateParams sp;
  sp.seq = pr.seq;
  sp.H = H;
  sp.W = sv.W; sp.U = sv.U; sp.Qt = sv.Qt; sp.Kb = sv.Kb; sp.M = sv.M; sp.dC = sv.dC;
  sp.h0 = h0;
  sp.o = static_cast<bf16*>(o);
  sp.hs = sv.hs;
  sp.E = sv.E;
  sp.ht = ht;
  sp.wait_polls = g_state_wait_polls.load(std::memory_order_relaxed);
  sp.withhold_loads = g_state_withhold_loads.load(std::memory_order_relaxed);
  if ((rc = encode_sw128_map(&sp.maps[0], sv.W, H, pr.TT, D)) || (rc = encode_sw128_map(&sp.maps[1], sv.Qt, H, pr.TT, D)) ||
      (rc = encode_sw128_map(&sp.maps[2], sv.Kb, H, pr.TT, D)) || (rc = encode_sw128_map(&sp.maps[3], sv.U, H, pr.TT, D)) ||
      (rc = encode_sw128_map(&sp.maps[4], sv.M, H, pr.TT, 64)))
    return rc;
  if ((rc = set_smem(kda_fwd_state_tc_kernel, StateTcSmem::END, "fwd state"))) return rc;
  {
    TimedLaunch tl(K_FWD_STATE, st);
    kda_fwd_state_tc_kernel<<<dim3(N, H), STATE_THREADS, StateTcSmem::END, st>>>(sp);
  }
  return launch_check("fwd state");
}

int kda_b200_bwd(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* A_log,
                 const float* dt_bias, const float* conv_q, const float* conv_k, const float* conv_v, const float* h0,
                 const int32_t* cu_seqlens, int B, int T, int H, int D_, int N, float scale, float lower_bound,
                 const void* saved, size_t saved_bytes, const void* do_, const float* dht, void* dq, void* dk,
                 void* dv, void* dg, void* dbeta, float* dA_log, float* ddt_bias, float* dconv_q, float* dconv_k,
                 float* dconv_v, float* dh0, void* workspace, size_t workspace_bytes, void* stream) {
  (void)h0;
  Problem pr;
  int rc = check_common(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, cu_seqlens, B, T, H, D_, N,
                        lower_bound, pr);
  if (rc) return rc;
  if (!saved || saved_bytes < kda_b200_saved_bytes(pr.TT, H, N, pr.packed))
    return fail(KDA_ERR_INVALID, "saved buffer missing or too small");
  if ((pr.TT > 0 && (!do_ || !dq || !dk || !dv || !dg || !dbeta)) || !dA_log || !ddt_bias)
    return fail(KDA_ERR_INVALID, "null gradient pointer");
  if (pr.conv && (!dconv_q || !dconv_k || !dconv_v)) return fail(KDA_ERR_INVALID, "null conv gradient pointer");
  if (!aligned(do_, 16) || !aligned(dq, 16) || !aligned(dk, 16) || !aligned(dv, 16) || !aligned(dg, 4))
    return fail(KDA_ERR_INVALID, "gradient tensors must be 16-byte aligned");
  size_t need_ws = kda_b200_bwd_workspace_bytes(pr.TT, H, N, pr.packed);
  if (!workspace || workspace_bytes < need_ws)
    return fail(KDA_ERR_INVALID, "workspace too small: need " + std::to_string(need_ws) + " bytes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pr.TT == 0) {
    cudaMemsetAsync(dA_log, 0, (size_t)H * 4, st);
    cudaMemsetAsync(ddt_bias, 0, (size_t)H * D * 4, st);
    if (pr.conv) {
      cudaMemsetAsync(dconv_q, 0, (size_t)H * D * 16, st);
      cudaMemsetAsync(dconv_k, 0, (size_t)H * D * 16, st);
      cudaMemsetAsync(dconv_v, 0, (size_t)H * D * 16, st);
    }
    if (dh0) {
      size_t bytes = (size_t)N * H * D * D * 4;
      if (dht) cudaMemcpyAsync(dh0, dht, bytes, cudaMemcpyDeviceToDevice, st);
      else cudaMemsetAsync(dh0, 0, bytes, st);
    }
    return launch_check("empty backward");
  }
  Carver wcv(workspace);
  Table tab = carve_table(wcv, N, pr.mc);
  BwdView bv = carve_bwd(wcv, pr.TT, H, pr.mc);
  Carver scv(const_cast<void*>(saved));
  SavedView sv = carve_saved(scv, pr.TT, H, pr.mc, true);
  if ((rc = build_table(pr, tab, st))) return rc;

  BwdStateParams bs;
  bs.seq = pr.seq;
  bs.H = H;
  bs.W = sv.W; bs.Qt = sv.Qt; bs.Kb = sv.Kb; bs.M = sv.M; bs.E = sv.E; bs.hs = sv.hs;
  bs.dO = static_cast<const bf16*>(do_);
  bs.dC = sv.dC;
  bs.dht = dht;
  bs.dE = bv.dE; bs.dQt = bv.dQt; bs.dW = bv.dW; bs.dKb = bv.dKb; bs.dM = bv.dM; bs.dGC = bv.dGC;
  bs.dh0 = dh0;
  if ((rc = encode_sw128_map(&bs.maps[0], sv.M, H, pr.TT, 64)) || (rc = encode_sw128_map(&bs.maps[1], do_, H, pr.TT, D)) ||
      (rc = encode_sw128_map(&bs.maps[2], sv.Kb, H, pr.TT, D)) || (rc = encode_sw128_map(&bs.maps[3], sv.Qt, H, pr.TT, D)) ||
      (rc = encode_sw128_map(&bs.maps[4], sv.W, H, pr.TT, D)))
    return rc;
  if ((rc = set_smem(kda_bwd_state_tc_kernel, BwdStateTcSmem::END, "bwd state"))) return rc;
  {
    TimedLaunch tl(K_BWD_STATE, st);
    kda_bwd_state_tc_kernel<<<dim3(N, H), STATE_THREADS, BwdStateTcSmem::END, st>>>(bs);
  }
  if ((rc = launch_check("bwd state"))) return rc;

  BwdIntraParams bi;
  bi.in = prologue_in(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, H, scale, lower_bound);
  bi.seq = pr.seq;
  bi.conv = pr.conv;
  bi.dE = bv.dE; bi.dW = bv.dW; bi.dQt = bv.dQt; bi.dKb = bv.dKb; bi.dM = bv.dM; bi.dGC = bv.dGC;
  bi.A = sv.A;
  bi.LP = sv.LP;
  bi.QN = sv.QN; bi.KN = sv.KN; bi.VN = sv.VN; bi.GM = sv.GM; bi.BT = sv.BT;
  bi.dq_hat = bv.dq_hat;
  bi.dk_hat = bv.dk_hat;
  bi.dv = pr.conv ? bv.dv_hat : static_cast<bf16*>(dv);
  bi.dg = static_cast<bf16*>(dg);
  bi.dbeta = static_cast<bf16*>(dbeta);
  bi.partA = bv.partA;
  bi.partB = bv.partB;
  if ((rc = set_smem(kda_bwd_intra_kernel, BwdIntraSmem::END, "bwd intra"))) return rc;
  {
    TimedLaunch tl(K_BWD_INTRA, st);
    kda_bwd_intra_kernel<<<dim3(pr.grid_chunks, H), INTRA_THREADS, BwdIntraSmem::END, st>>>(bi);
  }
  if ((rc = launch_check("bwd intra"))) return rc;

  PostParams pp;
  pp.seq = pr.seq;
  pp.H = H;
  pp.conv = pr.conv;
  pp.scale = scale;
  pp.q = static_cast<const bf16*>(q);
  pp.k = static_cast<const bf16*>(k);
  pp.v = static_cast<const bf16*>(v);
  pp.conv_q = conv_q; pp.conv_k = conv_k; pp.conv_v = conv_v;
  pp.dq_hat = bv.dq_hat; pp.dk_hat = bv.dk_hat; pp.dv_hat = bv.dv_hat;
  pp.dq = static_cast<bf16*>(dq);
  pp.dk = static_cast<bf16*>(dk);
  pp.dv = static_cast<bf16*>(dv);
  pp.partW = bv.partW;
  {
    TimedLaunch tl(K_BWD_POST, st);
    if (pr.conv)
      kda_bwd_post_conv_kernel<<<dim3((pr.grid_chunks + POST_CHUNKS_PER_CTA - 1) / POST_CHUNKS_PER_CTA, H, 3),
                                 32 * POST_CHUNKS_PER_CTA, 0, st>>>(pp);
    else
      kda_bwd_post_norm_kernel<<<dim3(pr.grid_chunks, H, 2), POST_THREADS, 0, st>>>(pp);
  }
  if ((rc = launch_check("bwd post"))) return rc;

  ReduceParams rp;
  rp.seq = pr.seq;
  rp.H = H;
  rp.conv = pr.conv;
  rp.partA = bv.partA; rp.partB = bv.partB; rp.partW = bv.partW;
  rp.dA_log = dA_log; rp.ddt_bias = ddt_bias;
  rp.dconv_q = dconv_q; rp.dconv_k = dconv_k; rp.dconv_v = dconv_v;
  {
    TimedLaunch tl(K_REDUCE, st);
    kda_reduce_kernel<<<dim3(2 * H + (pr.conv ? 12 * H : 0)), 256, 0, st>>>(rp);
  }
  return launch_check("reduce");
}

// ---- fp32 mode -------------------------------------------------------------
size_t kda_b200_f32_saved_bytes(int64_t total_tokens, int H, int N) {
  Carver cv(nullptr);
  carve_f32_saved(cv, total_tokens, H, max_chunks(total_tokens, N), true);
  return cv.off;
}

size_t kda_b200_f32_fwd_workspace_bytes(int64_t total_tokens, int H, int N, int training) {
  Carver cv(nullptr);
  const int64_t mc = max_chunks(total_tokens, N);
  carve_table(cv, N, mc);
  cv.take<float>((size_t)total_tokens * H * D * 4);  // post-conv v
  if (!training) carve_f32_saved(cv, total_tokens, H, mc, false);
  return cv.off;
}

size_t kda_b200_f32_bwd_workspace_bytes(int64_t total_tokens, int H, int N) {
  Carver cv(nullptr);
  const int64_t mc = max_chunks(total_tokens, N);
  carve_table(cv, N, mc);
  carve_f32_bwd(cv, total_tokens, H, N, mc);
  return cv.off;
}

int kda_b200_fwd_f32(const float* q, const float* k, const float* v, const float* g, const float* beta,
                     const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D_,
                     int N, float scale, float lower_bound, float* o, float* ht, void* saved, size_t saved_bytes,
                     void* workspace, size_t workspace_bytes, void* stream) {
  Problem pr;
  int rc = check_common(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, cu_seqlens, B, T, H, D_, N,
                        lower_bound, pr);
  if (rc) return rc;
  if (!o && pr.TT > 0) return fail(KDA_ERR_INVALID, "null output pointer");
  if (!aligned(o, 16) || !aligned(A_log, 4)) return fail(KDA_ERR_INVALID, "o must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool training = saved != nullptr;
  const size_t need_ws = kda_b200_f32_fwd_workspace_bytes(pr.TT, H, N, training);
  if (!workspace || workspace_bytes < need_ws)
    return fail(KDA_ERR_INVALID, "workspace too small: need " + std::to_string(need_ws) + " bytes");
  if (training && saved_bytes < kda_b200_f32_saved_bytes(pr.TT, H, N)) return fail(KDA_ERR_INVALID, "saved buffer too small");
  if (pr.TT == 0) {
    if (ht) {
      const size_t bytes = (size_t)N * H * D * D * 4;
      cudaError_t e = h0 ? cudaMemcpyAsync(ht, h0, bytes, cudaMemcpyDeviceToDevice, st) : cudaMemsetAsync(ht, 0, bytes, st);
      if (e != cudaSuccess) return fail(KDA_ERR_CUDA, cudaGetErrorString(e));
    }
    return KDA_OK;
  }
  Carver wcv(workspace);
  Table tab = carve_table(wcv, N, pr.mc);
  float* vh = wcv.take<float>((size_t)pr.TT * H * D * 4);
  Carver scv(training ? saved : nullptr);
  F32SavedView sv = training ? carve_f32_saved(scv, pr.TT, H, pr.mc, true) : carve_f32_saved(wcv, pr.TT, H, pr.mc, false);
  if ((rc = build_table(pr, tab, st))) return rc;

  F32PrepParams pp;
  pp.seq = pr.seq;
  pp.in = f32_inputs(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, H, pr.conv, scale, lower_bound);
  pp.qh = sv.qh; pp.kh = sv.kh; pp.vh = vh; pp.alpha = sv.alpha; pp.bt = sv.bt;
  {
    TimedLaunch tl(K_F32_PREP, st);
    kda_f32_prep_kernel<<<dim3(row_grid(pr), H), 32 * F32_WARPS_PER_CTA, 0, st>>>(pp);
  }
  if ((rc = launch_check("fp32 prep"))) return rc;

  F32FwdParams fp;
  fp.seq = pr.seq;
  fp.H = H;
  fp.qh = sv.qh; fp.kh = sv.kh; fp.vh = vh; fp.alpha = sv.alpha; fp.bt = sv.bt;
  fp.h0 = h0;
  fp.o = o;
  fp.r = sv.r;
  fp.ck = sv.ck;
  fp.ht = ht;
  fp.total_tokens = pr.TT;
  {
    TimedLaunch tl(K_F32_FWD, st);
    kda_f32_fwd_kernel<<<dim3(N, H, F32_FWD_GROUPS), 32, 0, st>>>(fp);
  }
  return launch_check("fp32 forward");
}

int kda_b200_bwd_f32(const float* q, const float* k, const float* v, const float* g, const float* beta,
                     const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D_,
                     int N, float scale, float lower_bound, const void* saved, size_t saved_bytes, const float* do_,
                     const float* dht, float* dq, float* dk, float* dv, float* dg, float* dbeta, float* dA_log,
                     float* ddt_bias, float* dconv_q, float* dconv_k, float* dconv_v, float* dh0, void* workspace,
                     size_t workspace_bytes, void* stream) {
  (void)h0;
  Problem pr;
  int rc = check_common(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, cu_seqlens, B, T, H, D_, N,
                        lower_bound, pr);
  if (rc) return rc;
  if (!saved || saved_bytes < kda_b200_f32_saved_bytes(pr.TT, H, N))
    return fail(KDA_ERR_INVALID, "saved buffer missing or too small");
  if ((pr.TT > 0 && (!do_ || !dq || !dk || !dv || !dg || !dbeta)) || !dA_log || !ddt_bias)
    return fail(KDA_ERR_INVALID, "null gradient pointer");
  if (pr.conv && (!dconv_q || !dconv_k || !dconv_v)) return fail(KDA_ERR_INVALID, "null conv gradient pointer");
  if (!aligned(do_, 16) || !aligned(dq, 16) || !aligned(dk, 16) || !aligned(dv, 16) || !aligned(dg, 16) ||
      !aligned(ddt_bias, 16) || (pr.conv && (!aligned(dconv_q, 16) || !aligned(dconv_k, 16) || !aligned(dconv_v, 16))) ||
      (dh0 && !aligned(dh0, 16)) || (dht && !aligned(dht, 16)))
    return fail(KDA_ERR_INVALID, "gradient tensors must be 16-byte aligned");
  const size_t need_ws = kda_b200_f32_bwd_workspace_bytes(pr.TT, H, N);
  if (!workspace || workspace_bytes < need_ws)
    return fail(KDA_ERR_INVALID, "workspace too small: need " + std::to_string(need_ws) + " bytes");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pr.TT == 0) {
    cudaMemsetAsync(dA_log, 0, (size_t)H * 4, st);
    cudaMemsetAsync(ddt_bias, 0, (size_t)H * D * 4, st);
    if (pr.conv) {
      cudaMemsetAsync(dconv_q, 0, (size_t)H * D * 16, st);
      cudaMemsetAsync(dconv_k, 0, (size_t)H * D * 16, st);
      cudaMemsetAsync(dconv_v, 0, (size_t)H * D * 16, st);
    }
    if (dh0) {
      const size_t bytes = (size_t)N * H * D * D * 4;
      if (dht) cudaMemcpyAsync(dh0, dht, bytes, cudaMemcpyDeviceToDevice, st);
      else cudaMemsetAsync(dh0, 0, bytes, st);
    }
    return launch_check("empty backward");
  }
  Carver wcv(workspace);
  Table tab = carve_table(wcv, N, pr.mc);
  F32BwdView bv = carve_f32_bwd(wcv, pr.TT, H, N, pr.mc);
  Carver scv(const_cast<void*>(saved));
  F32SavedView sv = carve_f32_saved(scv, pr.TT, H, pr.mc, true);
  if ((rc = build_table(pr, tab, st))) return rc;

  F32BwdParams bp;
  bp.seq = pr.seq;
  bp.H = H;
  bp.qh = sv.qh; bp.kh = sv.kh; bp.alpha = sv.alpha; bp.bt = sv.bt; bp.r = sv.r; bp.ck = sv.ck;
  bp.dO = do_;
  bp.dht = dht;
  bp.scratch = bv.scratch;
  bp.dqh_p = bv.dqh_p; bp.dkh_p = bv.dkh_p; bp.dal_p = bv.dal_p; bp.dbt_p = bv.dbt_p;
  bp.dvh = bv.dvh;
  bp.dh0 = dh0;
  bp.total_tokens = pr.TT;
  bp.items = N * H * F32_GROUPS;
  {
    TimedLaunch tl(K_F32_BWD, st);
    kda_f32_bwd_kernel<<<f32_bwd_ctas(bp.items), F32_BWD_THREADS, 0, st>>>(bp);
  }
  if ((rc = launch_check("fp32 backward"))) return rc;

  const F32Inputs in = f32_inputs(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, H, pr.conv, scale,
                                  lower_bound);
  F32DcParams dp;
  dp.seq = pr.seq;
  dp.in = in;
  dp.total_tokens = pr.TT;
  dp.dqh_p = bv.dqh_p; dp.dkh_p = bv.dkh_p; dp.dal_p = bv.dal_p; dp.dbt_p = bv.dbt_p; dp.dvh = bv.dvh;
  dp.alpha = sv.alpha; dp.bt = sv.bt;
  dp.dq = pr.conv ? bv.dcq : dq;
  dp.dk = pr.conv ? bv.dck : dk;
  dp.dv = pr.conv ? bv.dcv : dv;
  dp.dg = dg;
  dp.dbeta = dbeta;
  dp.partA = bv.partA; dp.partB = bv.partB;
  {
    TimedLaunch tl(K_F32_DC, st);
    kda_f32_dc_kernel<<<dim3(row_grid(pr), H), 32 * F32_WARPS_PER_CTA, 0, st>>>(dp);
  }
  if ((rc = launch_check("fp32 gate/norm backward"))) return rc;

  if (pr.conv) {
    F32ConvParams cp;
    cp.seq = pr.seq;
    cp.in = in;
    cp.dcq = bv.dcq; cp.dck = bv.dck; cp.dcv = bv.dcv;
    cp.dq = dq; cp.dk = dk; cp.dv = dv;
    cp.partW = bv.partW;
    {
      TimedLaunch tl(K_F32_CONV, st);
      kda_f32_conv_bwd_kernel<<<dim3(row_grid(pr), H, 3), 32 * F32_WARPS_PER_CTA, 0, st>>>(cp);
    }
    if ((rc = launch_check("fp32 conv backward"))) return rc;
  }

  ReduceParams rp;
  rp.seq = pr.seq;
  rp.H = H;
  rp.conv = pr.conv;
  rp.partA = bv.partA; rp.partB = bv.partB; rp.partW = bv.partW;
  rp.dA_log = dA_log; rp.ddt_bias = ddt_bias;
  rp.dconv_q = dconv_q; rp.dconv_k = dconv_k; rp.dconv_v = dconv_v;
  {
    TimedLaunch tl(K_REDUCE, st);
    kda_reduce_kernel<<<dim3(2 * H + (pr.conv ? 12 * H : 0)), 256, 0, st>>>(rp);
  }
  return launch_check("reduce");
}

int kda_b200_debug_set_input_wait_polls(unsigned int polls) {
  g_input_wait_polls.store(polls ? polls : kDefaultWaitPolls, std::memory_order_relaxed);
  return KDA_OK;
}

int kda_b200_debug_set_state_wait(unsigned int polls, int withhold_loads) {
  g_state_wait_polls.store(polls ? polls : kDefaultWaitPolls, std::memory_order_relaxed);
  g_state_withhold_loads.store(withhold_loads ? 1 : 0, std::memory_order_relaxed);
  return KDA_OK;
}

int kda_b200_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kda_device_error, sizeof(int)) != cudaSuccess)
    return -fail(KDA_ERR_CUDA, "reading the device error flag failed");
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(g_kda_device_error, &z, sizeof(int));
  }
  return v;
}

int kda_b200_timing_enable(int on) {
  std::lock_guard<std::mutex> lk(g_timing.mu);
  g_timing.on = on != 0;
  return KDA_OK;
}

int kda_b200_timing_reset(void) {
  std::lock_guard<std::mutex> lk(g_timing.mu);
  g_timing.used = 0;
  g_timing.ids.clear();
  return KDA_OK;
}

int kda_b200_timing_read(int max_kernels, const char** names, int* launches, float* total_ms) {
  std::lock_guard<std::mutex> lk(g_timing.mu);
  if (max_kernels < K_COUNT || !names || !launches || !total_ms)
    return -fail(KDA_ERR_INVALID, "timing_read needs room for " + std::to_string((int)K_COUNT) + " kernels");
  for (int k = 0; k < K_COUNT; ++k) {
    names[k] = kKernelNames[k];
    launches[k] = 0;
    total_ms[k] = 0.f;
  }
  for (size_t i = 0; i < g_timing.ids.size(); ++i) {
    cudaEvent_t a = g_timing.pool[2 * i], b = g_timing.pool[2 * i + 1];
    if (cudaEventSynchronize(b) != cudaSuccess) return -fail(KDA_ERR_CUDA, "timing event");
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, a, b) != cudaSuccess) return -fail(KDA_ERR_CUDA, "timing elapsed");
    launches[g_timing.ids[i]] += 1;
    total_ms[g_timing.ids[i]] += ms;
  }
  return K_COUNT;
}

// ---- forward without allocation ------------------------------------------
// The scratch of kda_b200_fwd_noalloc: a static device array, so no caller
// has to allocate.  Host code must not use the symbol as a pointer (that is a
// host-side stand-in); its device address is resolved per device below.
static __device__ __align__(256) unsigned char kda_noalloc_scratch[KDA_NOALLOC_SCRATCH_BYTES];

int kda_b200_fwd_noalloc(const void* q, const void* k, const void* v, const void* g, const void* beta,
                         const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                         const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H,
                         int D_, int N, float scale, float lower_bound, void* o, float* ht, void* stream) {
  if (B < 1 || T < 0 || H < 1 || N < 1) return fail(KDA_ERR_INVALID, "B >= 1, T >= 0, H >= 1 and N >= 1 are required");
  const size_t need = kda_b200_fwd_workspace_bytes((int64_t)B * T, H, N, cu_seqlens != nullptr, 0);
  if (need > KDA_NOALLOC_SCRATCH_BYTES)
    return fail(KDA_ERR_INVALID, "kda_b200_fwd_noalloc: this problem needs " + std::to_string(need) +
                                     " bytes of scratch but the static scratch holds " +
                                     std::to_string(KDA_NOALLOC_SCRATCH_BYTES) +
                                     "; call kda_b200_fwd with a caller-provided workspace instead");
  // The address is resolved on every call (the runtime keeps it per context), so it
  // stays valid across cudaDeviceReset and context re-creation.
  void* scratch = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&scratch, kda_noalloc_scratch);
  if (e != cudaSuccess || !scratch)
    return fail(KDA_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
  return kda_b200_fwd(q, k, v, g, beta, A_log, dt_bias, conv_q, conv_k, conv_v, h0, cu_seqlens, B, T, H, D_, N, scale,
                      lower_bound, o, ht, nullptr, 0, scratch, KDA_NOALLOC_SCRATCH_BYTES, stream);
}


size_t kda_b200_gated_norm_workspace_bytes(long long rows, int D_) {
  if (D_ != D || rows < 0) return 0;
  return (size_t)gn_grid(rows, true) * D * sizeof(float);
}

int kda_b200_gated_norm_fwd(const void* o, const void* g, const float* weight, long long rows, int D_, float eps,
                            int fp32_io, void* y, void* stream) {
  int rc;
  if ((rc = gn_check(rows, D_, o, g, weight, y, fp32_io))) return rc;
  if (rows == 0) return KDA_OK;
  GatedNormParams gp{};
  gp.o = o; gp.g = g; gp.w = weight; gp.y = y;
  gp.rows = rows; gp.eps = eps; gp.fp32 = fp32_io != 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    TimedLaunch tl(K_GNORM_FWD, st);
    kda_gated_norm_fwd_kernel<<<gn_grid(rows, false), GN_THREADS, 0, st>>>(gp);
  }
  return launch_check("gated norm fwd");
}

int kda_b200_gated_norm_bwd(const void* dy, const void* o, const void* g, const float* weight, long long rows,
                            int D_, float eps, int fp32_io, void* d_o, void* d_g, float* d_weight, void* workspace,
                            size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = gn_check(rows, D_, o, g, weight, dy, fp32_io))) return rc;
  if (!d_weight) return fail(KDA_ERR_INVALID, "null pointer");
  if (rows > 0 && (!d_o || !d_g)) return fail(KDA_ERR_INVALID, "null pointer");
  if (rows > 0 && (!aligned(d_o, 16) || !aligned(d_g, 16)))
    return fail(KDA_ERR_INVALID, "row tensors must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(d_weight, 0, D * sizeof(float), st);
    return e == cudaSuccess ? KDA_OK : fail(KDA_ERR_CUDA, cudaGetErrorString(e));
  }
  const int grid = gn_grid(rows, true);
  if (!workspace || workspace_bytes < (size_t)grid * D * sizeof(float) || !aligned(workspace, 16))
    return fail(KDA_ERR_INVALID, "workspace too small: kda_b200_gated_norm_workspace_bytes() bytes are needed");
  GatedNormParams gp{};
  gp.o = o; gp.g = g; gp.dy = dy; gp.w = weight;
  gp.d_o = d_o; gp.d_g = d_g; gp.partial = static_cast<float*>(workspace);
  gp.rows = rows; gp.eps = eps; gp.fp32 = fp32_io != 0;
  {
    TimedLaunch tl(K_GNORM_BWD, st);
    kda_gated_norm_bwd_kernel<<<grid, GN_THREADS, 0, st>>>(gp);
    kda_gated_norm_reduce_kernel<<<1, D * GN_REDUCE_SLICES, 0, st>>>(gp.partial, grid, d_weight);
  }
  return launch_check("gated norm bwd");
}

}  // extern "C"
