/*
 * qwen_megakernel.h -- C ABI of the B200 (sm_100a) Qwen3-0.6B decode megakernel.
 *
 * Everything here is plain C: raw device pointers, sizes, int/float scalars and
 * a cudaStream_t.  No torch types cross this boundary.  The shared library
 * libqwen_megakernel.so exports every function declared below.
 *
 * Reference interface this library replaces (AlpinDale/qwen_megakernel):
 *   - struct LDGLayerWeights          csrc/kernel.cu:76-88, csrc/torch_bindings.cpp:21-33
 *   - launch_ldg_decode_persistent    csrc/kernel.cu:1507, declared csrc/torch_bindings.cpp:35-43
 *   - launch_ldg_decode_direct        csrc/kernel.cu:1477, declared csrc/torch_bindings.cpp:45-53
 *   - launch_ldg_generate_nosync      csrc/kernel.cu:1547, declared csrc/torch_bindings.cpp:83-91
 * The three reference entry points keep their exact signatures and argument
 * meaning.  The qmk_* functions are additions (explicit workspace, forced
 * token streams, optional fp32 logits, error read-back, schedule queries).
 *
 * Data layouts (identical to the reference):
 *   embed_weight / lm_head_weight  bf16 [151936, 1024] row-major (tied)
 *   layer weights                  bf16 row-major [out, in] (HF nn.Linear)
 *   cos_table / sin_table          bf16 [rows >= last position + 1, 128]
 *                                  (rotate-half layout, halves duplicated)
 *   k_cache / v_cache              bf16 [num_layers, 8, max_seq_len, 128]
 */
#ifndef QWEN_MEGAKERNEL_H_
#define QWEN_MEGAKERNEL_H_

#include <stddef.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Model geometry (Qwen3-0.6B; reference qwen_megakernel/model.py:8-16). */
#define QMK_HIDDEN 1024
#define QMK_INTERMEDIATE 3072
#define QMK_NUM_Q_HEADS 16
#define QMK_NUM_KV_HEADS 8
#define QMK_HEAD_DIM 128
#define QMK_VOCAB 151936
#define QMK_MAX_LAYERS 64

/* Per-layer weight pointer table: 11 device pointers, 88 bytes, in the
 * reference order (csrc/kernel.cu:76-88; packed by model.py:97-108). */
typedef struct LDGLayerWeights {
  const void *input_layernorm_weight;     /* bf16 [1024]        */
  const void *q_proj_weight;              /* bf16 [2048, 1024]  */
  const void *k_proj_weight;              /* bf16 [1024, 1024]  */
  const void *v_proj_weight;              /* bf16 [1024, 1024]  */
  const void *q_norm_weight;              /* bf16 [128]         */
  const void *k_norm_weight;              /* bf16 [128]         */
  const void *o_proj_weight;              /* bf16 [1024, 2048]  */
  const void *post_attn_layernorm_weight; /* bf16 [1024]        */
  const void *gate_proj_weight;           /* bf16 [3072, 1024]  */
  const void *up_proj_weight;             /* bf16 [3072, 1024]  */
  const void *down_proj_weight;           /* bf16 [1024, 3072]  */
} LDGLayerWeights;

/* ------------------------------------------------------------------------- */
/* Reference entry points (same signatures as the reference).                */
/* They run on a library-owned workspace, one per device, allocated on first  */
/* use.  Like the reference's process-global barrier state (kernel.cu:1446-   */
/* 1473), that workspace is shared: concurrent calls on different streams of */
/* the same device race.  The scratch-buffer arguments (hidden_buffer ..      */
/* block_max_idxs) are accepted for ABI compatibility; only `g_normalized`    */
/* is written (the final RMSNorm output, fp32 [1024], as in the reference).   */
/* Errors: these return void; query qmk_get_last_error() after the call and  */
/* qmk_read_default_status() after a stream synchronize.                      */
/* ------------------------------------------------------------------------- */

/* One decode step: input_token_id at `position`; writes the greedy argmax to
 * *output_token_id (device int32).  Reference: csrc/kernel.cu:1477. */
void launch_ldg_decode_direct(
    int input_token_id, int *output_token_id, const void *embed_weight,
    const LDGLayerWeights *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table,
    void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
    void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
    void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
    void *block_max_idxs, int num_layers, int position, int max_seq_len,
    float attn_scale, cudaStream_t stream);

/* Same step; `cache_len` is accepted and ignored (the reference kernel also
 * derives it as position + 1).  Reference: csrc/kernel.cu:1507. */
void launch_ldg_decode_persistent(
    int input_token_id, int *output_token_id, const void *embed_weight,
    const LDGLayerWeights *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table,
    void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
    void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
    void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
    void *block_max_idxs, int num_layers, int position, int cache_len,
    int max_seq_len, float attn_scale, cudaStream_t stream);

/* num_steps greedy steps with device-side token feedback, no host sync:
 * step t consumes (t == 0 ? first_token_id : output_log[t-1]) at position
 * start_position + t and writes output_log[t].  Reference: kernel.cu:1547
 * (there: 4 launches per token; here: one launch for all steps). */
void launch_ldg_generate_nosync(
    int first_token_id, int num_steps, const void *embed_weight,
    const LDGLayerWeights *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight, const void *cos_table, const void *sin_table,
    void *k_cache, void *v_cache, void *hidden_buffer, void *g_activations,
    void *g_residual, void *g_q, void *g_k, void *g_v, void *g_attn_out,
    void *g_mlp_intermediate, void *g_normalized, void *block_max_vals,
    void *block_max_idxs, int *output_log, int num_layers, int start_position,
    int max_seq_len, float attn_scale, cudaStream_t stream);

/* ------------------------------------------------------------------------- */
/* Extended API (no reference counterpart: additions of this library).       */
/* ------------------------------------------------------------------------- */

/* Error codes (returned by qmk_* functions and written to the status block). */
#define QMK_OK 0
#define QMK_ERR_ARGS 1          /* invalid argument (host-side validation)   */
#define QMK_ERR_CUDA 2          /* a CUDA runtime call failed                */
#define QMK_ERR_LAUNCH 3        /* cooperative launch refused (co-residency) */
#define QMK_ERR_TIMEOUT 4       /* a bounded device-side wait expired        */
#define QMK_ERR_TOKEN 5         /* token id outside [0, vocab) on device     */
#define QMK_ERR_WORKSPACE 6     /* workspace too small / misaligned          */
#define QMK_ERR_SMEM 7          /* shared memory not 1 KB aligned on device  */

/* Host-visible status written by the kernel when it finishes (last CTA).
 * Lives in pinned, device-mapped host memory supplied by the caller. */
typedef struct QmkStatus {
  unsigned int error_code;  /* QMK_* device error of the last launch (0 = ok) */
  unsigned int error_info;  /* (cta << 16) | (site << 8) | layer              */
  unsigned int launches;    /* number of launches that completed              */
  unsigned int epoch;       /* flag epoch after the launch                    */
} QmkStatus;

typedef struct QmkRunArgs {
  const void *embed_weight;              /* bf16 [151936, 1024]               */
  const LDGLayerWeights *layer_weights;  /* device array [num_layers]         */
  const void *final_norm_weight;         /* bf16 [1024]                       */
  const void *lm_head_weight;            /* bf16 [151936, 1024]               */
  const void *cos_table;                 /* bf16 [>= start+steps, 128]        */
  const void *sin_table;                 /* bf16 [>= start+steps, 128]        */
  void *k_cache;                         /* bf16 [num_layers,8,max_seq,128]   */
  void *v_cache;
  void *workspace;                       /* device, qmk_workspace_bytes()     */
  size_t workspace_bytes;
  const int *forced_tokens;              /* device int32 [n_forced] or NULL   */
  int n_forced;                          /* steps t < n_forced read forced[t] */
  int first_token;                       /* step-0 token when n_forced == 0   */
  int start_position;
  int num_steps;
  int num_layers;
  int max_seq_len;
  float attn_scale;
  int *output_log;                       /* device int32 [num_steps] or NULL  */
  int *output_token;                     /* device int32 [1] or NULL          */
  float *logits;                         /* device fp32 [num_steps,151936] / NULL */
  float *final_hidden;                   /* device fp32 [1024] or NULL        */
  QmkStatus *status;                     /* mapped pinned host memory or NULL */
  unsigned long long timeout_ns;         /* per-wait limit; 0 = 1 s default   */
  int debug_stall;                       /* test hook, 0 = off; k > 0: CTA k-1 */
                                         /* waits (step 0, layer 0, O-proj input) */
                                         /* on a flag no CTA writes, so its       */
                                         /* bounded wait expires: the launch ends */
                                         /* with QMK_ERR_TIMEOUT in the status    */
  unsigned long long *trace;             /* optional device buffer of            */
                                         /* qmk_trace_words() uint64 globaltimer */
                                         /* stamps per CTA for step trace_step   */
  int trace_step;
  unsigned int poll_backoff_ns;          /* tuning: sleep between failed polls */
                                         /* of dataflow words (0 = spin; <= 4096) */
  unsigned int tuning;                   /* tuning flags (0 = default); bits 0-1: */
                                         /* store kind of dataflow words (0 red.max */
                                         /* atomic, 1 st.relaxed, 2 st.relaxed +   */
                                         /* fence per phase, 3 atom.exch)          */
  /* Sampling and stopping (no reference counterpart; zero = the reference's
   * greedy, fixed-length behaviour). */
  float temperature;                     /* 0: greedy argmax; > 0: sample from    */
                                         /* softmax(logits / temperature) by the */
                                         /* Gumbel-max trick, noise keyed by     */
                                         /* (seed, position, vocab index)        */
  unsigned long long seed;
  int stop_at_eos;                       /* nonzero: end the launch after the     */
  int eos_token;                         /* first GENERATED token == eos_token    */
                                         /* (forced tokens never stop it)         */
  int *steps_done;                       /* device int32 [1] or NULL: steps run   */
  int top_k;                             /* 1..QMK_TOP_K_MAX: sample only among   */
                                         /* the top_k logits (0: all)             */
} QmkRunArgs;

#define QMK_TOP_K_MAX 64

/* Bytes of device workspace one decoder needs (flags, dataflow buffers). */
size_t qmk_workspace_bytes(void);

/* Zero a workspace (stream-ordered).  Must be called once before first use. */
int qmk_workspace_init(void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* Launch the persistent decode kernel for args->num_steps steps (one
 * cooperative launch).  Returns QMK_OK or a host-side error code; device-side
 * errors are reported through args->status after the stream completes. */
int qmk_run(const QmkRunArgs *args, cudaStream_t stream);

/* ---- batched decode in the persistent kernel (no reference counterpart) --
 * QMK_BATCH_SEQS sequences decoded together greedily, each with its own K/V
 * cache (sequence s at element offset s * cache_seq_stride of k_cache /
 * v_cache, each in the reference layout [num_layers, 8, max_seq_len, 128])
 * and its own position.  Step t of sequence s consumes its step-t token at
 * cache position start_positions[s] + t (step 0: first_tokens[s], then the
 * greedy token of step t - 1) and writes that position's K/V; the greedy
 * token of step t goes to output_log[t * QMK_BATCH_SEQS + s].  Same kernel
 * as qmk_run: every weight tile is streamed once per step for all
 * sequences (q|k|v, gate/up and the LM head as tensor-core GEMVs with the
 * sequences as the N columns, O and down on the CUDA cores).  Uses the workspace of qmk_workspace_bytes(); device errors
 * are reported through status as for qmk_run. */
#define QMK_BATCH_SEQS 4

typedef struct QmkBatchRunArgs {
  const void *embed_weight;              /* bf16 [151936, 1024]               */
  const LDGLayerWeights *layer_weights;  /* device array [num_layers]         */
  const void *final_norm_weight;         /* bf16 [1024]                       */
  const void *lm_head_weight;            /* bf16 [151936, 1024]               */
  const void *cos_table;                 /* bf16 [>= max position + 1, 128]   */
  const void *sin_table;
  void *k_cache;                         /* bf16, see above                   */
  void *v_cache;
  long long cache_seq_stride;            /* elements between sequences' caches */
  void *workspace;                       /* device, qmk_workspace_bytes()     */
  size_t workspace_bytes;
  const int *first_tokens;               /* device int32 [QMK_BATCH_SEQS]     */
  int start_positions[QMK_BATCH_SEQS];   /* host values                       */
  int num_steps;
  int num_layers;
  int max_seq_len;
  float attn_scale;
  int *output_log;                       /* device int32 [num_steps][QMK_BATCH_SEQS] or NULL */
  QmkStatus *status;                     /* mapped pinned host memory or NULL */
  unsigned long long timeout_ns;         /* per-wait limit; 0 = 1 s default   */
} QmkBatchRunArgs;

int qmk_run_batch(const QmkBatchRunArgs *args, cudaStream_t stream);

/* Host-side error of the last qmk_* / launch_ldg_* call on this thread. */
int qmk_get_last_error(void);
const char *qmk_get_last_error_message(void);
const char *qmk_error_string(int code);

/* Status of the library-owned default workspace of the current device (used
 * by the three reference entry points).  Valid after a stream synchronize. */
int qmk_read_default_status(QmkStatus *out);

/* Number of CTAs (one per SM) the kernel launches on `device`. */
int qmk_num_ctas(int device);

/* KV splits per KV head the kernel uses for a launch whose last position is
 * `max_position` on `num_ctas` CTAs. */
int qmk_attention_splits(int num_ctas, int max_position);

/* Host-side description of the static work partition, for tests: fills
 * out[0..7] for CTA `cta` of `num_ctas` with
 *   {qkv_row0, qkv_row1, o_row0, o_row1, gu_row0, gu_row1, d_row0, d_row1}
 * and out[8..11] with {lm_row0, lm_row1, item (or -1), merge_task (or -1)}. */
int qmk_describe_partition(int num_ctas, int splits, int cta, int *out, int out_len);

/* uint64 words per CTA of the optional timeline trace (QmkRunArgs.trace):
 * per layer 16 slots (phase input-ready / done stamps, producer issue
 * window), then the LM-head slots. */
int qmk_trace_words(void);

/* ---- allocation-free variant (no counterpart in the reference) ----------
 * qmk_generate_static runs the same decode as launch_ldg_generate_nosync
 * above (first token, num_steps greedy steps from start_position, the token
 * of step t into entry t of a token log) but allocates nothing:
 * no cudaMalloc / cudaFree / cudaHostAlloc, no allocator of any library.
 * Its scratch -- the kernel workspace, the token log and a status block --
 * is one file-scope __device__ array of QMK_STATIC_SCRATCH_BYTES per device
 * in this library's static device memory.  It is meant for callers that
 * must not allocate on this path: a host framework that owns all device
 * memory through its own pool (a cudaMalloc behind its back can fail or
 * fragment it), and latency-critical loops where the implicit device-wide
 * synchronization of cudaMalloc / cudaFree is not acceptable.
 *
 *  - Limit: num_steps <= QMK_STATIC_MAX_STEPS (the token log's capacity);
 *    larger requests return QMK_ERR_ARGS without launching.
 *  - The first call on a device does one-time setup (cudaGetSymbolAddress
 *    of the scratch array, kernel attributes); make that first call before
 *    any stream capture.
 *  - The workspace part must start zeroed: static device memory is zero
 *    when the module loads and every launch leaves it valid for the next.
 *  - All calls on a device share the one scratch array: calls that overlap
 *    in time (different streams without ordering, or different host
 *    threads) race on it.  Serialize them, e.g. on one stream.
 *  - Results: qmk_static_scratch_ptrs gives the device addresses of the
 *    token log (int32 [QMK_STATIC_MAX_STEPS], entry t = token of step t of
 *    the last call) and of the QmkStatus block (device memory: copy it to
 *    the host after the stream completes). */
#define QMK_STATIC_MAX_STEPS 4096
#define QMK_STATIC_SCRATCH_BYTES (1024 * 1024)

int qmk_generate_static(int first_token_id, int num_steps, const void *embed_weight,
                        const LDGLayerWeights *layer_weights, const void *final_norm_weight,
                        const void *lm_head_weight, const void *cos_table, const void *sin_table,
                        void *k_cache, void *v_cache, int num_layers, int start_position,
                        int max_seq_len, float attn_scale, cudaStream_t stream);

/* Device addresses (current device) of the static token log and status
 * block used by qmk_generate_static; either pointer may be NULL. */
int qmk_static_scratch_ptrs(int **output_log, QmkStatus **status);

/* ---- token-parallel path: prefill and batched decode ---------------------
 * No counterpart in the reference, which processes a prompt one decode step
 * per token (qwen_megakernel/model.py:210-211) and decodes batch 1 only.
 * One call runs the whole model over `num_rows` rows at once: row r feeds
 * token tokens[r] of sequence row_seq[r] at position row_pos[r], writes its
 * K/V at that position of that sequence's cache and attends to positions
 * [0, row_pos[r]] of it.  Rows of one sequence at consecutive positions are
 * a causal prefill (every row sees the K/V the earlier rows write in the same
 * call); one row per sequence is a batched decode step.  The projections are
 * tensor-core GEMMs (this library's tcgen05 kernel, bf16 operands:
 * activations as a bf16 hi + lo pair, fp32 accumulate, so they keep the
 * decode kernel's fp32 precision);
 * norms, QK-norm + RoPE + K/V append, attention, SiLU and argmax are this
 * library's kernels.  Output rows out_rows[i] (i < num_out) get the final
 * RMSNorm, the LM head and the greedy argmax (lowest index on ties).
 *
 * Caches: sequence s uses k_cache + s * kv_seq_stride (elements), layout
 * bf16 [num_layers, 8, max_seq_len, 128] as above.  Token ids outside
 * [0, vocab) read token 0, rows whose sequence or position is out of range
 * are skipped; either sets a bit in *status (device uint32, optional):
 * QMK_BATCH_BAD_TOKEN / QMK_BATCH_BAD_ROW.  A K/V tile copy of the
 * attention that does not complete within 1 s sets QMK_BATCH_TIMEOUT (the
 * outputs of that call are then invalid); if the copies still in flight do
 * not land within a further 1 s either, QMK_BATCH_COPIES_PENDING is set too:
 * bulk copies may then still write shared memory after their CTA exited, so
 * the host should treat the context as suspect (reuse nothing computed on
 * that stream afterwards, recreate the context).  All launches are
 * stream-ordered and capturable in a CUDA graph (no allocation, no host
 * sync). */
#define QMK_BATCH_BAD_TOKEN 1u
#define QMK_BATCH_BAD_ROW 2u
#define QMK_BATCH_TIMEOUT 4u
#define QMK_BATCH_COPIES_PENDING 8u

typedef struct QmkBatchArgs {
  const void *embed_weight;              /* bf16 [151936, 1024]                 */
  const void *const *layer_ptrs;         /* HOST array [num_layers * 11] of the */
                                         /* device pointers, LDGLayerWeights   */
                                         /* order (the GEMMs are launched from */
                                         /* the host)                          */
  const void *const *fused_ptrs;         /* HOST array [num_layers * 2] or NULL:*/
                                         /* per layer a bf16 [4096, 1024] copy  */
                                         /* of q|k|v and a [6144, 1024] copy of */
                                         /* gate|up (one GEMM each; NULL: the   */
                                         /* separate matrices, 5 GEMMs)         */
  const void *final_norm_weight;         /* bf16 [1024]                         */
  const void *lm_head_weight;            /* bf16 [151936, 1024]                 */
  const void *cos_table;                 /* bf16 [max_seq_len, 128]             */
  const void *sin_table;
  void *k_cache;                         /* bf16, see above; 16-byte aligned    */
  void *v_cache;                         /* 16-byte aligned                     */
  long long kv_seq_stride;               /* elements between sequences' caches, */
                                         /* a multiple of 8 (16 bytes)          */
  int num_seqs;
  int num_layers;
  int max_seq_len;
  float attn_scale;
  int num_rows;                          /* 1 .. QMK_BATCH_MAX_ROWS             */
  const int *tokens;                     /* device int32 [num_rows]             */
  const int *row_seq;                    /* device int32 [num_rows]             */
  const int *row_pos;                    /* device int32 [num_rows]             */
  int num_out;                           /* 0 .. num_rows                       */
  const int *out_rows;                   /* device int32 [num_out]              */
  int *out_tokens;                       /* device int32 [num_out] or NULL      */
  float *logits;                         /* device fp32 [num_out, 151936] or NULL*/
  void *workspace;                       /* device, qmk_batch_workspace_bytes() */
  size_t workspace_bytes;
  unsigned int *status;                  /* device uint32 [1] or NULL           */
  int causal_run;                        /* nonzero: the caller guarantees that */
                                         /* row r is position r of sequence 0  */
                                         /* (a fresh prompt); for 64 < rows <= */
                                         /* QMK_BATCH_GEMM_ATTN_MAX_ROWS the   */
                                         /* attention then runs as two batched */
                                         /* tensor-core GEMMs per layer        */
} QmkBatchArgs;

#define QMK_BATCH_GEMM_ATTN_MAX_ROWS 2048

#define QMK_BATCH_MAX_ROWS 4096

/* Device workspace bytes for num_rows rows and num_out output rows
 * (256-byte aligned start required). */
size_t qmk_batch_workspace_bytes(int num_rows, int num_out);

/* Queue the forward pass on `stream`.  Returns QMK_OK or a host-side error
 * (QMK_ERR_ARGS, QMK_ERR_WORKSPACE, QMK_ERR_CUDA). */
int qmk_batch_forward(const QmkBatchArgs *args, cudaStream_t stream);

/* ---- tensor-core GEMM of the token-parallel path -------------------------
 * No reference counterpart (the reference has no token-parallel path).  The
 * GEMM qmk_batch_forward runs every projection and the prompt attention with
 * (tcgen05, TMEM accumulators, TMA operand ring), exported for tests and for
 * callers that want it directly:
 *   C[z][s] = A[z][:, K_s] * W[z][:, K_s]^T, z < batch, s < splits
 * with W bf16 [n, k] (row stride ldw elements, batch stride w_batch_stride),
 * A bf16 [rows, k] (lda, a_batch_stride), C fp32 [rows, n] (ldc,
 * c_batch_stride), split s of the K blocks into C + s * c_split_stride.
 * Operands 16-byte aligned, ldw / lda / batch strides multiples of 8,
 * splits > 1 only with k a multiple of 64.  A wait that exceeds 1 s sets
 * QMK_BATCH_TIMEOUT in *status (optional) and leaves C unwritten. */
int qmk_gemm_bf16_nt(const void *W, long long ldw, long long w_batch_stride, int n, const void *A, long long lda,
                     long long a_batch_stride, int rows, int k, int batch, int splits, float *C, long long ldc,
                     long long c_batch_stride, long long c_split_stride, unsigned int *status, cudaStream_t stream);

/* Library version string. */
const char *qmk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_MEGAKERNEL_H_ */
