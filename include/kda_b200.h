/*
 * kda_b200 -- C ABI of the B200 (sm_100a) Kimi Delta Attention layer.
 *
 * The reference (Sophia) reaches this path through two Python seams, and this
 * ABI is what those seams bind to (sophia_b200/_lib.py is the ctypes binding):
 *
 *   SophiaKDA._fla_chunk_kda() -> chunk_kda(q, k, v, g, beta, ...)
 *       ml/runtime/model/attention.py:305-312 (seam), called at :349-365 with
 *       use_qk_l2norm_in_kernel / use_gate_in_kernel / use_beta_sigmoid_in_kernel
 *       / safe_gate all true and lower_bound = kda_decay_lower_bound; the
 *       callee's contract is flash-linear-attention's chunk_kda
 *       (fla/ops/kda/chunk.py:167-411).  -> kda_b200_fwd / kda_b200_bwd with
 *       the conv taps set to NULL.
 *   CausalDepthwiseConv1d.forward (attention.py:32-60) followed by the
 *       recurrence (attention.py:373-410) -> kda_b200_fwd / kda_b200_bwd with
 *       the three conv tap tensors: the ShortConv+SiLU is fused into the chunk
 *       prologue.
 *
 * Conventions
 *   - Every pointer is a device pointer; `stream` is a cudaStream_t.  Nothing
 *     allocates: the caller passes the `saved` (forward -> backward) and
 *     `workspace` buffers whose sizes the *_bytes functions return.  Nothing
 *     synchronises with the host, so calls can be captured in CUDA graphs.
 *   - q, k, v, g, o and all their gradients are bf16 [B, T, H, 128]; beta and
 *     dbeta are bf16 [B, T, H] (fp32 for the *_f32 entry points); A_log [H],
 *     dt_bias [H*128], conv taps [H*128, 4], states [N, H, 128, 128] are fp32.
 *   - cu_seqlens (int32 [N+1], device) packs N sequences along T (then B == 1);
 *     the recurrent state and the conv history restart at every boundary.
 *   - Return value: KDA_OK or an error code; kda_b200_last_error() describes
 *     the last failure of the calling thread.
 */
#ifndef KDA_B200_H_
#define KDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_OK 0
#define KDA_ERR_INVALID 1     /* bad shape, pointer, alignment or parameter   */
#define KDA_ERR_UNSUPPORTED 2 /* valid in the reference but not implemented  */
#define KDA_ERR_CUDA 3        /* a CUDA launch failed                          */

/* Library version string. */
const char* kda_b200_version(void);

/* Description of the last error returned to the calling thread. */
const char* kda_b200_last_error(void);

/* Bytes of the forward -> backward buffer (chunk intermediates, chunk-start
 * states, v_new).  total_tokens = B*T; N = number of sequences. */
size_t kda_b200_saved_bytes(int64_t total_tokens, int H, int N, int packed);

/* Bytes of scratch for kda_b200_fwd.  training = 0 means `saved` is NULL and
 * the intermediates live in the workspace instead. */
size_t kda_b200_fwd_workspace_bytes(int64_t total_tokens, int H, int N, int packed, int training);

/* Bytes of scratch for kda_b200_bwd. */
size_t kda_b200_bwd_workspace_bytes(int64_t total_tokens, int H, int N, int packed);

/*
 * Forward.  Replaces chunk_kda's forward (fla/ops/kda/chunk.py:22-115) in the
 * configuration of attention.py:349-365, optionally preceded by the ShortConv
 * of attention.py:32-60 when conv_q/conv_k/conv_v are non-NULL.
 *   h0: initial state or NULL (zeros).  ht: final state or NULL.
 *   saved: NULL for inference, else kda_b200_saved_bytes() bytes to hand to
 *   kda_b200_bwd.
 */
int kda_b200_fwd(const void* q, const void* k, const void* v, const void* g, const void* beta,
                 const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                 const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D,
                 int N, float scale, float lower_bound, void* o, float* ht, void* saved, size_t saved_bytes,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward.  Replaces ChunkKDAFunction.backward (fla/ops/kda/chunk.py:117-162)
 * plus, with conv taps, the autograd of attention.py:32-60.  Inputs as in the
 * forward plus `saved`, the output gradient do_ and the final-state gradient
 * dht (NULL = zero).  Writes dq, dk, dv (w.r.t. the inputs as given, i.e.
 * pre-conv when conv taps are set), dg (gate logits), dbeta (beta logits),
 * dA_log [H], ddt_bias [H*128], dconv_* [H*128, 4] (when conv) and dh0 (when
 * non-NULL).
 */
int kda_b200_bwd(const void* q, const void* k, const void* v, const void* g, const void* beta,
                 const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                 const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D,
                 int N, float scale, float lower_bound, const void* saved, size_t saved_bytes, const void* do_,
                 const float* dht, void* dq, void* dk, void* dv, void* dg, void* dbeta, float* dA_log,
                 float* ddt_bias, float* dconv_q, float* dconv_k, float* dconv_v, float* dh0, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * fp32 mode.  Replaces chunk_kda's forward / backward (fla/ops/kda/chunk.py:
 * 22-162) when q, k, v, g and beta arrive in float32, the precision of the
 * reference's own recurrence (SophiaKDA._reference_kda,
 * ml/runtime/model/attention.py:260-294, float32 inside).  Same arguments and
 * meaning as kda_b200_fwd / kda_b200_bwd, except that every activation and
 * gradient (q, k, v, g, beta, o, do_, dq, dk, dv, dg, dbeta) is fp32
 * [B, T, H, 128] ([B, T, H] for beta) and the buffers are sized by the
 * kda_b200_f32_*_bytes functions.  All arithmetic is fp32 on CUDA cores (no
 * tensor-core rounding); the recurrence runs token by token in the
 * reference's order, so results agree with the reference to fp32 rounding.
 * The backward's scratch includes a per-CTA slice of 256 KiB for at most four
 * CTAs per SM (and at most one per (sequence, head, 32-column group)).
 */
size_t kda_b200_f32_saved_bytes(int64_t total_tokens, int H, int N);
size_t kda_b200_f32_fwd_workspace_bytes(int64_t total_tokens, int H, int N, int training);
size_t kda_b200_f32_bwd_workspace_bytes(int64_t total_tokens, int H, int N);
int kda_b200_fwd_f32(const float* q, const float* k, const float* v, const float* g, const float* beta,
                     const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D,
                     int N, float scale, float lower_bound, float* o, float* ht, void* saved, size_t saved_bytes,
                     void* workspace, size_t workspace_bytes, void* stream);
int kda_b200_bwd_f32(const float* q, const float* k, const float* v, const float* g, const float* beta,
                     const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                     const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H, int D,
                     int N, float scale, float lower_bound, const void* saved, size_t saved_bytes, const float* do_,
                     const float* dht, float* dq, float* dk, float* dv, float* dg, float* dbeta, float* dA_log,
                     float* ddt_bias, float* dconv_q, float* dconv_k, float* dconv_v, float* dh0, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * Packed-sequence chunk table (integer bookkeeping of prepare_chunk_indices /
 * prepare_chunk_offsets, fla/ops/utils/index.py:138-158), built on the device
 * without a host sync.  offsets: int32 [N+1]; chunk_seq: int32 [max_chunks]
 * with max_chunks >= total_tokens/64 + N; error_flag: int32, written 1 when
 * cu_seqlens does not start at 0, decreases, or does not end at total_tokens
 * (then every offset is 0 and the layer calls that use the table do nothing).
 * kda_b200_fwd / kda_b200_bwd build this table in their workspace.
 */
int kda_b200_chunk_table(const int32_t* cu_seqlens, int N, int64_t total_tokens, int32_t* offsets,
                         int32_t* chunk_seq, int32_t* error_flag, void* stream);

/*
 * Document boundaries of packed pretraining windows -> cu_seqlens, on the
 * device with no host synchronisation, so that it can sit inside a captured
 * CUDA graph.  Sophia's data path packs documents into fixed windows and runs
 * each window as one sequence with no reset at document ends
 * (ml/training/pretrain/engine/sm120_graph_runner.py:244-259); this entry
 * point gives the packed layer the boundaries instead.  tokens: int32
 * [total_tokens], windows of `window` tokens back to back.  A document starts
 * at every window start and after every token equal to eos_id.  cu_seqlens:
 * int32 [capacity + 1]: the first min(count, capacity) document starts in
 * order, then total_tokens in every later entry (empty sequences), so the
 * layer is called with N = capacity.  n_docs: int32 [1], the true document
 * count; when it exceeds the capacity the later boundaries are dropped (those
 * documents continue their predecessor's state, as the reference does).
 */
int kda_b200_doc_cu_seqlens(const int32_t* tokens, int64_t total_tokens, int window, int eos_id, int capacity,
                            int32_t* cu_seqlens, int32_t* n_docs, void* stream);

/*
 * Token-by-token recurrence for decode, fp32 state and arithmetic -- replaces
 * flash-linear-attention's fused_recurrent_kda (0.5.x, not vendored) at its
 * Sophia call site: the single-step decode of SophiaKDA._run_kda
 * (ml/runtime/model/attention.py:330-348, seam :296-304), with the in-kernel
 * L2 norms, gate and beta sigmoid of that call.  q, k, v, g: [B*T][H][128],
 * beta: [B*T][H], bf16 (fp32_inputs = 0) or fp32 (fp32_inputs = 1); o takes
 * the same dtype.  h0 / ht: [N][H][128][128] fp32 (either may be null).  With
 * cu_seqlens (B = 1) every sequence starts from its own h0 row.  Forward only;
 * no workspace.  A cu_seqlens entry outside [0, B*T] makes the kernel skip that
 * sequence and set kda_b200_device_error() to 3.
 */
int kda_b200_recurrent(const void* q, const void* k, const void* v, const void* g, const void* beta,
                       const float* A_log, const float* dt_bias, const float* h0, const int32_t* cu_seqlens, int B,
                       int T, int H, int D, int N, int fp32_inputs, float scale, float lower_bound, void* o,
                       float* ht, void* stream);

/*
 * Decode step of a cached SophiaKDA.forward with the ShortConv fused: replaces
 * _short_convolution with a conv history (ml/runtime/model/attention.py:226-258,
 * CausalDepthwiseConv1d.forward with history, :32-60) followed by
 * _run_kda's single-step decode (:330-348).  As kda_b200_recurrent, except
 * that q, k and v are the pre-conv projections and conv_q/conv_k/conv_v
 * ([H*128][4] fp32 taps) with conv_state ([N][3][H*128][3] fp32, the module's
 * conv_state rows: the last three inputs of q, k and v per channel, oldest
 * first) run the conv + SiLU in front of the recurrence; conv_state is read
 * at the start and rewritten with the last three inputs at the end.  Any
 * number of tokens per sequence.
 */
int kda_b200_decode(const void* q, const void* k, const void* v, const void* g, const void* beta,
                    const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                    const float* conv_v, float* conv_state, const float* h0, const int32_t* cu_seqlens, int B,
                    int T, int H, int D, int N, int fp32_inputs, float scale, float lower_bound, void* o, float* ht,
                    void* stream);

/*
 * Device-side failure flag of the tensor-core kernels.  Their waits on
 * asynchronous MMA completion are bounded; a wait that runs out makes the
 * kernel record a nonzero code here and return early (its outputs are then
 * invalid) instead of hanging the GPU.  Synchronises with the device; reset = 1
 * clears the flag.  Returns the flag, or minus an error code.  The reference
 * has no counterpart (its kernels run in Triton without such waits).
 */
int kda_b200_device_error(int reset);

/*
 * Codes of kda_b200_device_error():
 *   1, 2  a tensor-core completion wait of a state kernel ran out;
 *   3     a cu_seqlens table was malformed (does not start at 0, decreases, or
 *         does not end at the token count): the layer call did nothing;
 *   5, 7  a bulk-copy wait of the backward chunk kernel ran out;
 *   8     the forward chunk kernel's wait for its prefetched inputs ran out;
 *   9     a chunk kernel's dynamic shared memory was not 1 KB aligned (its
 *         swizzled tensor-core tiles need it): the kernel did nothing;
 *   10    a tensor-core completion wait of the forward chunk kernel ran out.
 * A kernel that records a timeout lets its copies in flight land (a second
 * bounded wait), frees what it holds and returns; later calls are unaffected.
 */

/*
 * Test hook of the bounded waits: the number of polls the forward chunk
 * kernel makes for an item's prefetched inputs before it records code 8 and
 * returns (0 restores the default, 2^26).  A test lowers it to 1 so that the
 * wait runs out without any fault, then checks the code.  Applies to calls
 * made after it.  No counterpart in the reference.
 */
int kda_b200_debug_set_input_wait_polls(unsigned int polls);

/*
 * Test hook of the forward state pass's producer/consumer protocol: `polls`
 * bounds the consumers' wait for each chunk's operands (0 restores the default,
 * 2^26), and a nonzero `withhold_loads` makes the producer warp issue no copy,
 * so that wait can only run out.  The consumers then record code 1, wake the
 * producer, release TMEM and return -- no fault and no hang.  Applies to calls
 * made after it.  No counterpart in the reference.
 */
int kda_b200_debug_set_state_wait(unsigned int polls, int withhold_loads);

/*
 * Per-kernel device timing, for benchmarks and profiling summaries.  While
 * enabled, every kernel launch of kda_b200_fwd / kda_b200_bwd is bracketed by
 * two cudaEventRecord calls on its stream.  kda_b200_timing_read synchronises
 * those events and returns, per kernel, its static name, the number of
 * launches and the summed milliseconds since the last reset.  It returns the
 * number of kernels (> 0), or minus an error code on failure.  The
 * reference has no counterpart (its tracing is version/hash records only,
 * ml/training/pretrain/engine/sm120_concurrent_ffn.py:468-477).
 */
int kda_b200_timing_enable(int on);
int kda_b200_timing_reset(void);
int kda_b200_timing_read(int max_kernels, const char** names, int* launches, float* total_ms);

/*
 * Forward (inference) that allocates nothing -- no counterpart in the
 * reference.  For callers that cannot allocate device memory themselves: a
 * host binding (cgo, JNI, a C serving loop) that has no device allocator of
 * its own, or a process that reserves all device memory up front and forbids
 * later allocations.  Same arguments and results as kda_b200_fwd with
 * saved = NULL, minus the workspace: the scratch is a static device array of
 * KDA_NOALLOC_SCRATCH_BYTES (64 MiB) that every GPU loading this library holds
 * until the process exits.
 *   - A call whose kda_b200_fwd_workspace_bytes(B*T, H, N, packed, 0) exceeds
 *     that size returns KDA_ERR_INVALID (no kernel runs).
 *   - Every call resolves the array's device address on the current device
 *     (cudaGetSymbolAddress, which the CUDA runtime keeps per context), so the
 *     address stays valid across cudaDeviceReset and context re-creation.  The
 *     first call on a device may load the module: make it before any stream
 *     capture begins.
 *   - All calls share the one array and it keeps the last call's contents;
 *     nothing in it has to start at zero (every call writes what it reads).
 *     Calls that overlap on the GPU (other streams, other host threads) race on
 *     it: serialise them.
 *   - No cudaMalloc, cudaFree or allocating library routine is called.
 */
#define KDA_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
int kda_b200_fwd_noalloc(const void* q, const void* k, const void* v, const void* g, const void* beta,
                         const float* A_log, const float* dt_bias, const float* conv_q, const float* conv_k,
                         const float* conv_v, const float* h0, const int32_t* cu_seqlens, int B, int T, int H,
                         int D, int N, float scale, float lower_bound, void* o, float* ht, void* stream);

/*
 * Gated output norm of the KDA mixer -- replaces, in SophiaKDA.forward
 * (ml/runtime/model/attention.py:416-419), the output RMSNorm over each head's
 * 128 channels (RMSNorm.forward, ml/runtime/model/ops.py:49-64, i.e.
 * torch.nn.functional.rms_norm with a fp32 weight) followed by the product
 * with sigmoid(gate logits):
 *     y = o / sqrt(mean(o^2) + eps) * weight * sigmoid(g)      per row of 128
 * o, g, y (and dy, d_o, d_g): [rows][128], all bf16 (fp32_io = 0) or all fp32
 * (fp32_io = 1), 16-byte aligned; weight: [128] fp32; arithmetic in fp32.
 * The backward writes d_o and d_g and stores (not accumulates) the weight
 * gradient, summed over rows in a fixed order, into d_weight [128] fp32; it
 * needs kda_b200_gated_norm_workspace_bytes(rows, 128) bytes of workspace.
 * rows = 0 is a no-op (d_weight is zeroed).  Errors as the other entry points:
 * D != 128 is KDA_ERR_UNSUPPORTED, bad shapes or pointers KDA_ERR_INVALID.
 */
size_t kda_b200_gated_norm_workspace_bytes(long long rows, int D);
int kda_b200_gated_norm_fwd(const void* o, const void* g, const float* weight, long long rows, int D, float eps,
                            int fp32_io, void* y, void* stream);
int kda_b200_gated_norm_bwd(const void* dy, const void* o, const void* g, const float* weight, long long rows,
                            int D, float eps, int fp32_io, void* d_o, void* d_g, float* d_weight, void* workspace,
                            size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_B200_H_ */
