/*
 * qf_b200.h -- C ABI of the B200 (sm_100a) W8A16 decode-GEMM library (libqf_b200.so).
 *
 * The library replaces the Triton kernel behind EurekaZang/qwen-a100-fastpath's vLLM plugin
 * (plugin/qwen_fastpath/w8a16.py) for the QWEN_FAST_LINEAR linear method and the QWEN_FAST_DRAFT_HEAD
 * int8 draft LM head.  Signatures carry plain pointers, sizes and a CUDA stream handle only; no
 * framework types.  All pointers are device pointers owned by the caller (borrowed for the call); every
 * entry point enqueues on `stream` and returns without synchronising, so calls can be captured into a
 * CUDA graph once the workspace exists.
 *
 * Layouts (the tensors vLLM already holds; no repacking, no second weight copy):
 *   x      bf16 [M, K], row stride ldx elements, unit column stride           (activations, M <= 16)
 *   w      int8 [N, K] row-major, row stride ldw bytes == vLLM's w_q [K, N] view with stride (1, ldw)
 *   scale  fp32 [N], per output channel (vLLM's w_s [N, 1] read flat)
 *   y      [M, N] row stride ldy elements, bf16 or fp32
 *
 * Math (matches w8a16.py:15-44): y[m,n] = round_out( scale[n] * sum_k x[m,k] * (float)w[n,k] ) with exact
 * bf16 x int8 products accumulated in fp32; with bias, round_bf16( (float)y_bf16 + (float)bias[n] ) as the
 * reference's separate `y + bias` (patches.py:96-97).
 *
 * Alignment: x, w 16-byte aligned; ldx % 8 == 0 (bf16 elements); ldw % 16 == 0 (bytes).  These are the
 * TMA tensor-map rules; a caller with other strides makes the rows contiguous first.
 *
 * Workspace: `ws` (>= qf_w8a16_workspace_bytes()) must be zero-filled once when allocated; every call
 * leaves its counters at zero again.  Calls that share a workspace must be ordered on one stream.  The
 * first word of the workspace is a sticky device error flag (see qf_workspace_status).
 *
 * Return values: QF_OK (0) or a negative QF_ERR_* code; qf_last_error_detail() gives a message
 * (thread-local).
 */
#ifndef QF_B200_H
#define QF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QF_ABI_VERSION 1

#define QF_OK 0
#define QF_ERR_INVALID (-1)   /* null pointer or bad argument */
#define QF_ERR_SHAPE (-2)     /* M, N, K or n_valid out of range */
#define QF_ERR_STRIDE (-3)    /* leading dimension smaller than the row */
#define QF_ERR_ALIGN (-4)     /* pointer or stride alignment not met */
#define QF_ERR_ARCH (-5)      /* current device is not compute capability 10.0 (B200 / sm_100a) */
#define QF_ERR_WORKSPACE (-6) /* workspace missing or too small */
#define QF_ERR_LAUNCH (-7)    /* CUDA runtime error at launch */
#define QF_ERR_DTYPE (-8)     /* unsupported output dtype */
#define QF_ERR_TIMEOUT (-9)   /* a bounded device-side wait expired (reported through the workspace) */
#define QF_ERR_DRIVER (-10)   /* driver entry point cuTensorMapEncodeTiled unavailable / rejected */

#define QF_DTYPE_BF16 0
#define QF_DTYPE_F32 1

#define QF_MAX_M 16        /* rows per call (the reference's SMALL_M, w8a16.py:12) */
#define QF_MAX_N 1048576   /* output channels per call (tile-counter capacity of the workspace) */

/* flags */
#define QF_FLAG_PDL 1u     /* launch with programmatic dependent launch: the weight prefetch of this call may
                              overlap the previous kernel on the stream (weights and scales must not be written
                              by that kernel; activations, outputs and workspace are only touched after it
                              completes) */

/* Bytes of workspace a call with these sizes needs (fixed prefix of counters + split-K partials + head
 * statistics).  No CUDA call is made. */
size_t qf_w8a16_workspace_bytes(int M, int N, int K);

/* Small-M W8A16 GEMM.  Replaces `w8a16_mm(x, w_t, w_scale, cfg, out_dtype)` (plugin/qwen_fastpath/w8a16.py:71-83)
 * plus the fused bias of `qf_int8_linear` (plugin/qwen_fastpath/patches.py:84-98).  bias: bf16 [N] or NULL.
 * y_dtype: QF_DTYPE_BF16 or QF_DTYPE_F32 (fp32 exports the pre-rounding accumulator * scale; bias is then
 * added in fp32).  1 <= M <= 16; M == 0 or N == 0 is a no-op; K == 0 writes zeros (+ bias). */
int qf_w8a16_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                  const void* bias, void* y, int64_t ldy, int y_dtype, int M, int N, int K,
                  void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* Int8 draft LM head with fused per-row statistics.  Replaces `int8_logits` + `compute_logits` +
 * `get_top_tokens` (plugin/qwen_fastpath/patches.py:157-185): bf16 logits [M, N] (ldl; NULL skips the
 * store), and over columns [0, n_valid) of the same bf16 logits: row_max (fp32), row_argmax (int64, first
 * index on ties, + vocab_offset) and row_lse (fp32 logsumexp).  Columns >= n_valid are the vocab padding
 * the reference masks to -inf (patches.py:182-184).  1 <= n_valid <= N; 1 <= M <= 16; K >= 1. */
int qf_w8a16_head(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                  void* logits, int64_t ldl, int M, int N, int K, int n_valid, int64_t vocab_offset,
                  float* row_max, int64_t* row_argmax, float* row_lse,
                  void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* Int8 draft head with a fused temperature draw for probabilistic drafting (no counterpart in the reference,
 * whose draft head is greedy only, patches.py:176-185).  Same GEMM and logits as qf_w8a16_head; the statistics
 * are of the scaled logits s = logit * inv_temperature (row_max, row_argmax, row_lse = logsumexp(s)), and each
 * row also gets one Gumbel-max draw from softmax(s) over columns [0, n_valid):
 *   row_sample = argmax_j s_j + g_j (+ vocab_offset), row_sample_score = that maximum, row_sample_logit = s at it,
 *   g_j = -log(-log u), u = ((word >> 9) + 1/2) * 2^-23, word = Philox4x32-10 (Salmon et al., SC 2011) of the
 *   counter (j + vocab_offset, m / 4, offset low, offset high) under the key (seed low, seed high), word m % 4.
 * The draft probability of the draw is exp(row_sample_logit - row_lse).  The noise depends only on (seed, offset,
 * global column, row), so vocab shards draw exactly what one unsharded head draws: take the shard with the
 * largest row_sample_score (lowest column on ties) and combine row_lse as for qf_w8a16_head.
 * inv_temperature finite and > 0; vocab_offset + N <= 2^32. */
int qf_w8a16_head_sample(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                         void* logits, int64_t ldl, int M, int N, int K, int n_valid, int64_t vocab_offset,
                         float inv_temperature, uint64_t seed, uint64_t offset, float* row_max,
                         int64_t* row_argmax, float* row_lse, int64_t* row_sample, float* row_sample_score,
                         float* row_sample_logit, void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* Small-M W8A16 GEMM that allocates nothing and takes no workspace.  No counterpart in the reference: it is
 * for callers that cannot allocate device memory themselves -- a host that embeds only this library through
 * the C ABI (a Go, Java or C binding with no device allocator of its own), or a latency-critical path that
 * must not call cudaMalloc, which can synchronise the device.  Same arguments and math as qf_w8a16_gemm
 * without ws / ws_bytes.  Its scratch (split-tile counters and fp32 partial tiles) is a fixed
 * QF_NOALLOC_SCRATCH_BYTES array inside the library, held by every GPU that loads the library until the
 * process exits.  N is limited to QF_NOALLOC_MAX_N because the array holds 8192 tile counters and a tile is at
 * least 32 output channels high (larger N returns QF_ERR_SHAPE), and the device may have at most 160 SMs (two
 * partial-tile slots per CTA).  The first call on a device (or the first qf_w8a16_noalloc_status) looks up that
 * array's device address (cudaGetSymbolAddress) and enqueues one zero fill of its counters on `stream`; it must
 * be made with the device current, before any stream capture.  Later calls enqueue only the kernel: each call
 * leaves the counters at zero for the next.  All calls share the one array, so calls whose kernels overlap on the
 * GPU (different streams) race: order them on one stream.  A device-side timeout is kept in the array until
 * qf_w8a16_noalloc_status reads it. */
#define QF_NOALLOC_MAX_N 262144
#define QF_NOALLOC_SCRATCH_BYTES 2675712u
int qf_w8a16_gemm_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                          const void* bias, void* y, int64_t ldy, int y_dtype, int M, int N, int K,
                          unsigned flags, void* stream);
/* Reads and clears the sticky device error flag of the allocation-free entry point's fixed scratch on the current
 * device (synchronises `stream`); *status receives QF_OK or QF_ERR_TIMEOUT.  After a timeout it also zeroes the
 * scratch's tile counters, so the next call starts clean.  No counterpart in the reference.  Not for the hot
 * path. */
int qf_w8a16_noalloc_status(void* stream, int* status);

/* gate_up projection with the MLP activation fused into its epilogue: w holds the merged [gate; up] weight (rows
 * [0, N/2) gate, [N/2, N) up, vLLM's MergedColumnParallelLinear), and the result is the activation
 * y[m, j] = bf16( bf16(silu(g[m, j])) * u[m, j] ), j < N/2, where g and u are the bf16 GEMM outputs of the gate and up
 * rows -- vLLM's SiluAndMul on the gate_up output (F.silu(x[..., :I]) * x[..., I:]; the reference plugin calls the
 * plain GEMM and leaves the activation to vLLM).  Saves the [M, N] intermediate and its separate kernel.  Arguments
 * as qf_w8a16_gemm (bf16 output [M, N/2], no bias); N even. */
int qf_w8a16_gemm_silu_mul(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale, void* y,
                           int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* ---- prefill (M > 16): dynamic per-token int8 activations x int8 weights on tcgen05 ----------------------------
 * Replaces the W8A8 fallback of qf_int8_linear for the rows the small-M path does not take
 * (plugin/qwen_fastpath/patches.py:99-100: vLLM's scaled_int8_quant + cutlass_scaled_mm, vllm==0.31.0):
 *   s_x[m] = max_k |x[m,k]| / 127,  q[m,k] = round_half_even_saturate_s8( x[m,k] * (127 / max_k |x[m,k]|) ),
 *   y[m,n] = bf16( s_x[m] * (w_scale[n] * float(sum_k q[m,k] * w[n,k])) ), with a bias: bf16( fma(s_x[m], t, bias[n]) ).
 * x bf16 [M, K] (row stride ldx, 2-byte aligned; 16-byte loads when 16-byte aligned with ldx % 8 == 0); w, w_scale,
 * bias, y as qf_w8a16_gemm (y bf16).  Any M >= 1.  The workspace (>= qf_w8a8_workspace_bytes(M, K), 256-byte aligned)
 * holds a 256-byte header (word 0: sticky error flag, see qf_workspace_status), then q int8 [M, ldq] with
 * ldq = K rounded up to 16, padded to 256 bytes, then s_x fp32 [M].  Two launches on `stream`: the quantization
 * (with QF_FLAG_PDL it may overlap the previous kernel's tail) and the GEMM (its first weight copies overlap the
 * quantization). */
size_t qf_w8a8_workspace_bytes(int M, int K);
int qf_w8a8_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* w_scale, const void* bias,
                 void* y, int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* ---- speculative-verification attention (QWEN_FAST_ATTN) -------------------------------------------------------
 * Replaces gqa_packed_spec_attention (plugin/qwen_fastpath/spec_attn.py:139-173), the path patch_flash_attention
 * routes uniform speculative-decode batches to (patches.py:10-69).  num_reqs requests x q_len query tokens each
 * (token b * q_len + qi); query qi of request b attends the cached keys [0, seq_lens[b] - q_len + qi] (this step's
 * keys are already in the cache); a row with no key gives zeros.  q: bf16 [num_reqs * q_len][num_heads][head_size]
 * with element strides (sq_t, sq_h, 1); k_cache / v_cache: bf16 [num_blocks][page_size][num_kv_heads][head_size]
 * views with element strides (s_b, s_t, s_h, 1) (any order of slot and head strides, the same for both);
 * block_table: int32 [num_reqs][*] (row stride s_bt; the page of slot pos is block_table[b][pos / page_size]);
 * seq_lens: int32 [num_reqs]; out: bf16, same layout as q with strides (so_t, so_h, 1).  Softmax scale `scale`;
 * num_heads a multiple of num_kv_heads; head_size 64, 128 or 256; q_len * num_heads / num_kv_heads <= 64;
 * page_size a multiple of 16; q, caches and out 16-byte aligned with strides multiples of 8 elements.  The workspace
 * (>= qf_spec_attn_workspace_bytes(...) for the current device, 256-byte aligned; word 0 is a sticky error flag read
 * by qf_workspace_status) holds the split partials; it need not be zeroed.  One or two launches on `stream`, no host
 * synchronisation and no host read of device data (CUDA-graph capturable); QF_FLAG_PDL lets the first launch overlap
 * the previous kernel's tail. */
size_t qf_spec_attn_workspace_bytes(int num_reqs, int q_len, int num_heads, int num_kv_heads, int head_size);
int qf_spec_attn(const void* q, int64_t sq_t, int64_t sq_h, const void* k_cache, int64_t sk_b, int64_t sk_t,
                 int64_t sk_h, const void* v_cache, int64_t sv_b, int64_t sv_t, int64_t sv_h, int num_blocks,
                 int page_size, const int32_t* block_table, int64_t s_bt, const int32_t* seq_lens, void* out,
                 int64_t so_t, int64_t so_h, int num_reqs, int q_len, int num_heads, int num_kv_heads, int head_size,
                 float scale, void* ws, size_t ws_bytes, unsigned flags, void* stream);

/* The W8A16 GEMM with the RMSNorm that precedes qkv and gate_up in a decoder layer fused into it (the reference plugin
 * leaves the norm to vLLM's RMSNorm: z = x + residual, new residual = bf16(z), normalized activation
 * bf16(bf16(z * rsqrt(mean(z^2) + eps)) * gamma)).  Here the activation fed to the contraction is bf16(bf16(z) * gamma)
 * and each token's fp32 accumulators are multiplied by rsqrt(mean(z^2) + eps) (z in fp32) before the scale and the
 * bf16 rounding: the per-token factor commutes with the k-sum, so only the rounding of the normalized activation
 * differs from the unfused sequence.  residual: bf16 [M, K] (ldr) or NULL (z = x); gamma: bf16 [K], 16-byte
 * aligned; residual_out: bf16 [M, K] (ldro) receiving bf16(z), or NULL; it must not overlap x or residual.  The
 * sums of z^2 come from the activation stages the kernel streams anyway (no extra pass over x).
 * silu_mul = 0: y = the GEMM output [M, N]; 1: w is the merged gate_up weight and y = bf16(bf16(silu(g)) * u)
 * [M, N/2] as qf_w8a16_gemm_silu_mul.  No bias.  K % 8 == 0, K <= 8192; other arguments as qf_w8a16_gemm. */
int qf_w8a16_gemm_rmsnorm(const void* x, int64_t ldx, const void* residual, int64_t ldr, const void* gamma, float eps,
                          void* residual_out, int64_t ldro, const int8_t* w, int64_t ldw, const float* scale, void* y,
                          int64_t ldy, int M, int N, int K, int silu_mul, void* ws, size_t ws_bytes, unsigned flags,
                          void* stream);

/* Load-time int8 quantizer of the draft LM head on the device: replaces the per-row symmetric quantizer the
 * reference runs in torch when the drafter loads (plugin/qwen_fastpath/patches.py:143-147).  w: bf16 [V, H] (row
 * stride ldw elements); q: int8 [V, H] (row stride ldq bytes); scale: fp32 [V].  s = max(max|w|, 1e-8) / 127,
 * q = clamp(round_half_even(w / s), -127, 127), the same fp32 operations as the reference (bit-identical).
 * H <= 8192. */
int qf_quantize_rows_int8(const void* w, int64_t ldw, int V, int H, int8_t* q, int64_t ldq, float* scale,
                          void* stream);

/* Reads and clears the workspace's sticky device error flag (synchronises `stream`).  *status receives
 * QF_OK or QF_ERR_TIMEOUT.  Not for the hot path. */
int qf_workspace_status(void* ws, void* stream, int* status);

/* ---- tensor parallelism: one-shot all-reduce over NVLink peer memory ----------------------------------------
 * Replaces the NCCL all-reduce that vLLM issues after a row-parallel layer (o_proj, down) under tensor
 * parallelism; the reference plugin has no code of its own here (it runs on one GPU and leaves the collective to
 * vLLM's NCCL).  Every rank of one node allocates one symmetric buffer of qf_allreduce_buffer_bytes(max_count)
 * bytes (qf_symm_alloc: zero-filled), exports it with qf_ipc_handle, opens the other ranks' buffers with
 * qf_ipc_open (CUDA IPC; peers reached over NVLink), and passes all `world` buffer pointers (its own at [rank]) to
 * every call.  Calls are collective: every rank makes the same sequence of calls with the same count.  The
 * epoch bookkeeping lives in the buffer, so calls can be captured in CUDA graphs. */
#define QF_AR_MAX_RANKS 8
#define QF_AR_MAX_CHUNKS 256    /* count <= 256 * 1024 elements */
#define QF_IPC_HANDLE_BYTES 64

/* Bytes of one rank's symmetric buffer for vectors of up to max_count bf16 elements (0 if max_count <= 0). */
size_t qf_allreduce_buffer_bytes(int max_count);
/* cudaMalloc + zero fill (synchronous) of a buffer to be shared between ranks; qf_symm_free releases it. */
int qf_symm_alloc(size_t bytes, void** dev_ptr);
int qf_symm_free(void* dev_ptr);
/* CUDA IPC handle (QF_IPC_HANDLE_BYTES bytes) of a qf_symm_alloc buffer; open / close another rank's buffer. */
int qf_ipc_handle(void* dev_ptr, void* handle_out);
int qf_ipc_open(const void* handle, void** peer_ptr);
int qf_ipc_close(void* peer_ptr);
/* out[i] = bf16( sum over ranks r = 0..world-1, in that order, of in_r[i] ), fp32 sums; identical on every rank.
 * in / out: bf16 [count], 16-byte aligned, may alias; count and max_count multiples of 8, count <= max_count <=
 * QF_AR_MAX_CHUNKS * 1024; bufs[r]: rank r's buffer (256-byte aligned).  Waits for the other ranks are bounded (2 s);
 * an expired wait is recorded in the buffer (qf_allreduce_status).  flags: QF_FLAG_PDL. */
int qf_allreduce_bf16(const void* in, void* out, int count, int max_count, int rank, int world,
                      void* const* bufs, unsigned flags, void* stream);
/* Reads and clears the sticky error word of this rank's buffer (synchronises `stream`). */
int qf_allreduce_status(void* own_buf, void* stream, int* status);
/* Bound of every wait on the other ranks in calls on this rank's buffer (qf_allreduce_bf16 and
 * qf_w8a16_gemm_allreduce), in microseconds; 0 restores the default of 2 s.  Stored in the buffer's header
 * (synchronises `stream`), so it also holds for calls captured in a CUDA graph.  An expired wait records
 * QF_ERR_TIMEOUT (qf_allreduce_status) and the kernel finishes without the missing contributions.  No counterpart
 * in the reference. */
int qf_allreduce_set_wait(void* own_buf, unsigned wait_us, void* stream);

/* Row-parallel W8A16 GEMM with the all-reduce fused into its epilogue: y = bf16( sum over ranks r, in rank order, of
 * bf16(scale * x_r . w_r) ) on every rank, where each rank holds its K-shard of x and w (vLLM's RowParallelLinear
 * followed by its NCCL all-reduce; no counterpart in the reference plugin).  Each finished output tile is pushed to
 * every rank's buffer over NVLink and summed as soon as all ranks' copies of that tile have arrived, so the
 * collective overlaps the GEMM's remaining tiles.  Collective: every rank calls it with the same M, N and K.
 * Arguments as qf_w8a16_gemm (bf16 output only, no bias) plus the qf_allreduce_bf16 buffers (bufs, max_count,
 * same buffers and epoch sequence: the two calls may be mixed on one set of buffers).  max_count must hold the
 * output with its tiles rounded up (N rounded up to 128, times M); at most QF_AR_MAX_CHUNKS output tiles. */
int qf_w8a16_gemm_allreduce(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const float* scale,
                            void* y, int64_t ldy, int M, int N, int K, void* ws, size_t ws_bytes,
                            int rank, int world, void* const* bufs, int max_count, unsigned flags, void* stream);

/* Static description of the error code. */
const char* qf_strerror(int code);
/* Message of the last failing call on this thread. */
const char* qf_last_error_detail(void);
/* QF_ABI_VERSION of the built library. */
int qf_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QF_B200_H */
