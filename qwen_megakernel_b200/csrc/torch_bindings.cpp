// Torch operator boundary: TORCH_LIBRARY(qwen_megakernel_C, ...).
//
// The two reference operators keep their schemas byte-for-byte
// (reference csrc/torch_bindings.cpp:129-155):
//   decode(...)          -> launch_ldg_decode_direct          (torch_bindings.cpp:55-81)
//   generate_nosync(...) -> launch_ldg_generate_nosync + sync (torch_bindings.cpp:93-127)
// Unlike the reference they validate their inputs (device, dtype, shape,
// position bounds) and raise RuntimeError on bad arguments or on a device-side
// error reported by the kernel's status block.
//
// Added operators (no reference counterpart):
//   run(...)             -> qmk_run with a caller-owned workspace, optional
//                           forced-token stream, fp32 logits, status block, trace
//   run_batch(...)       -> qmk_run_batch: QMK_BATCH_SEQS sequences decoded
//                           together in the persistent kernel
//   workspace_bytes()    -> qmk_workspace_bytes
//   workspace_init(ws)   -> qmk_workspace_init
//   default_status()     -> qmk_read_default_status (after a synchronize)
//   num_ctas()           -> qmk_num_ctas(current device)
//   trace_words()        -> qmk_trace_words
#include <Python.h>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <torch/all.h>
#include <torch/library.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>

#include "qwen_megakernel.h"

namespace {

// Error messages are formatted with vsnprintf and handed to TORCH_CHECK as a
// plain C string.  This library is compiled against GCC 13 headers but runs
// on the process's newer libstdc++; iostream number formatting instantiated
// from the older headers crashed inside the newer runtime's facets, so no
// number is ever streamed through an iostream here.
[[noreturn]] void fail(const char *fmt, ...) {
  char buf[640];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  TORCH_CHECK(false, static_cast<const char *>(buf));
  abort();  // unreachable
}

#define QMK_CHECK(cond, ...)          \
  do {                                \
    if (!(cond)) fail(__VA_ARGS__);   \
  } while (0)

using ll = long long;

void check_cuda(const torch::Tensor &t, const char *name) {
  QMK_CHECK(t.is_cuda(), "%s must be a CUDA tensor", name);
  QMK_CHECK(t.is_contiguous(), "%s must be contiguous", name);
}

void check_dtype(const torch::Tensor &t, c10::ScalarType want, const char *name, const char *want_name) {
  check_cuda(t, name);
  QMK_CHECK(t.scalar_type() == want, "%s must be %s", name, want_name);
}

void check_same_device(const torch::Tensor &t, const torch::Tensor &ref, const char *name) {
  QMK_CHECK(t.device() == ref.device(), "%s is on cuda:%d but the weights are on cuda:%d", name,
            (int)t.device().index(), (int)ref.device().index());
}

// Shared checks of the model tensors of every operator.
void check_model(const torch::Tensor &embed_weight, const torch::Tensor &layer_weights_packed,
                 const torch::Tensor &final_norm_weight, const torch::Tensor &lm_head_weight,
                 const torch::Tensor &cos_table, const torch::Tensor &sin_table,
                 const torch::Tensor &k_cache, const torch::Tensor &v_cache, int64_t num_layers,
                 int64_t last_position, int64_t max_seq_len) {
  check_dtype(embed_weight, torch::kBFloat16, "embed_weight", "bfloat16");
  QMK_CHECK(embed_weight.dim() == 2 && embed_weight.size(0) == QMK_VOCAB && embed_weight.size(1) == QMK_HIDDEN,
            "embed_weight must be [%d, %d]", QMK_VOCAB, QMK_HIDDEN);
  check_dtype(lm_head_weight, torch::kBFloat16, "lm_head_weight", "bfloat16");
  QMK_CHECK(lm_head_weight.sizes() == embed_weight.sizes(), "lm_head_weight must be [%d, %d]", QMK_VOCAB,
            QMK_HIDDEN);
  check_dtype(final_norm_weight, torch::kBFloat16, "final_norm_weight", "bfloat16");
  QMK_CHECK(final_norm_weight.numel() == QMK_HIDDEN, "final_norm_weight must have %d elements", QMK_HIDDEN);
  check_cuda(layer_weights_packed, "layer_weights_packed");
  QMK_CHECK(num_layers >= 1 && num_layers <= QMK_MAX_LAYERS, "num_layers must be in [1, %d], got %lld",
            QMK_MAX_LAYERS, (ll)num_layers);
  QMK_CHECK(layer_weights_packed.nbytes() >= (size_t)num_layers * sizeof(LDGLayerWeights),
            "layer_weights_packed holds %lld bytes; %lld layers need %lld", (ll)layer_weights_packed.nbytes(),
            (ll)num_layers, (ll)(num_layers * (int64_t)sizeof(LDGLayerWeights)));
  check_dtype(cos_table, torch::kBFloat16, "cos_table", "bfloat16");
  check_dtype(sin_table, torch::kBFloat16, "sin_table", "bfloat16");
  QMK_CHECK(cos_table.dim() == 2 && cos_table.size(1) == QMK_HEAD_DIM, "cos_table must be [rows, %d]",
            QMK_HEAD_DIM);
  QMK_CHECK(sin_table.sizes() == cos_table.sizes(), "sin_table must match cos_table");
  QMK_CHECK(cos_table.size(0) > last_position, "cos/sin tables have %lld rows; position %lld needs %lld",
            (ll)cos_table.size(0), (ll)last_position, (ll)(last_position + 1));
  check_dtype(k_cache, torch::kBFloat16, "k_cache", "bfloat16");
  check_dtype(v_cache, torch::kBFloat16, "v_cache", "bfloat16");
  QMK_CHECK(k_cache.dim() == 4 && k_cache.size(0) >= num_layers && k_cache.size(1) == QMK_NUM_KV_HEADS &&
                k_cache.size(2) == max_seq_len && k_cache.size(3) == QMK_HEAD_DIM,
            "k_cache must be [>=num_layers, %d, max_seq_len=%lld, %d]", QMK_NUM_KV_HEADS, (ll)max_seq_len,
            QMK_HEAD_DIM);
  QMK_CHECK(v_cache.sizes() == k_cache.sizes(), "v_cache must match k_cache");
  QMK_CHECK(last_position < max_seq_len, "position %lld >= max_seq_len %lld", (ll)last_position,
            (ll)max_seq_len);
  const torch::Tensor *others[] = {&layer_weights_packed, &final_norm_weight, &lm_head_weight, &cos_table,
                                   &sin_table,            &k_cache,           &v_cache};
  for (const torch::Tensor *t : others) check_same_device(*t, embed_weight, "model tensor");
}

void check_token(int64_t tok, const char *name) {
  QMK_CHECK(tok >= 0 && tok < QMK_VOCAB, "%s %lld outside [0, %d)", name, (ll)tok, QMK_VOCAB);
}

void check_normalized(const torch::Tensor &normalized) {
  check_dtype(normalized, torch::kFloat32, "normalized", "float32");
  QMK_CHECK(normalized.numel() >= QMK_HIDDEN, "normalized must have >= %d elements", QMK_HIDDEN);
}

void raise_if_error(int rc) {
  if (rc != QMK_OK) fail("qwen_megakernel: %s: %s", qmk_error_string(rc), qmk_get_last_error_message());
}

void raise_if_status(const QmkStatus &st) {
  if (st.error_code != QMK_OK)
    fail("qwen_megakernel: device error: %s (cta %u, site %u, layer %u)", qmk_error_string((int)st.error_code),
         st.error_info >> 16, (st.error_info >> 8) & 0xffu, st.error_info & 0xffu);
}

}  // namespace

// Reference schema (torch_bindings.cpp:130-140).
void decode(torch::Tensor output_token, int64_t input_token_id, torch::Tensor embed_weight,
            torch::Tensor layer_weights_packed, torch::Tensor final_norm_weight,
            torch::Tensor lm_head_weight, torch::Tensor cos_table, torch::Tensor sin_table,
            torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor hidden_buffer,
            torch::Tensor activations, torch::Tensor residual, torch::Tensor q, torch::Tensor k,
            torch::Tensor v, torch::Tensor attn_out, torch::Tensor mlp_intermediate,
            torch::Tensor normalized, torch::Tensor block_max_vals, torch::Tensor block_max_idxs,
            int64_t num_layers, int64_t position, int64_t max_seq_len, double attn_scale) {
  QMK_CHECK(position >= 0, "position must be >= 0");
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, position, max_seq_len);
  check_token(input_token_id, "input_token_id");
  check_dtype(output_token, torch::kInt32, "output_token", "int32");
  QMK_CHECK(output_token.numel() >= 1, "output_token must have >= 1 element");
  check_normalized(normalized);
  c10::cuda::CUDAGuard guard(embed_weight.device());
  launch_ldg_decode_direct(
      (int)input_token_id, static_cast<int *>(output_token.data_ptr()), embed_weight.data_ptr(),
      reinterpret_cast<const LDGLayerWeights *>(layer_weights_packed.data_ptr()),
      final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
      sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), hidden_buffer.data_ptr(),
      activations.data_ptr(), residual.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
      attn_out.data_ptr(), mlp_intermediate.data_ptr(), normalized.data_ptr(),
      block_max_vals.data_ptr(), block_max_idxs.data_ptr(), (int)num_layers, (int)position,
      (int)max_seq_len, (float)attn_scale, c10::cuda::getCurrentCUDAStream().stream());
  raise_if_error(qmk_get_last_error());
}

// Reference schema (torch_bindings.cpp:143-153).  Synchronizes the stream
// before returning, like the reference (torch_bindings.cpp:124-125).
torch::Tensor generate_nosync(int64_t first_token_id, int64_t num_steps, torch::Tensor embed_weight,
                              torch::Tensor layer_weights_packed, torch::Tensor final_norm_weight,
                              torch::Tensor lm_head_weight, torch::Tensor cos_table,
                              torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
                              torch::Tensor hidden_buffer, torch::Tensor activations,
                              torch::Tensor residual, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                              torch::Tensor attn_out, torch::Tensor mlp_intermediate,
                              torch::Tensor normalized, torch::Tensor block_max_vals,
                              torch::Tensor block_max_idxs, int64_t num_layers,
                              int64_t start_position, int64_t max_seq_len, double attn_scale) {
  QMK_CHECK(num_steps >= 1, "num_steps must be >= 1");
  QMK_CHECK(start_position >= 0, "start_position must be >= 0");
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, start_position + num_steps - 1, max_seq_len);
  check_token(first_token_id, "first_token_id");
  check_normalized(normalized);
  c10::cuda::CUDAGuard guard(embed_weight.device());
  auto stream = c10::cuda::getCurrentCUDAStream().stream();
  auto output_log = torch::empty({num_steps}, torch::dtype(torch::kInt32).device(embed_weight.device()));
  launch_ldg_generate_nosync(
      (int)first_token_id, (int)num_steps, embed_weight.data_ptr(),
      reinterpret_cast<const LDGLayerWeights *>(layer_weights_packed.data_ptr()),
      final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
      sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), hidden_buffer.data_ptr(),
      activations.data_ptr(), residual.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
      attn_out.data_ptr(), mlp_intermediate.data_ptr(), normalized.data_ptr(),
      block_max_vals.data_ptr(), block_max_idxs.data_ptr(), static_cast<int *>(output_log.data_ptr()),
      (int)num_layers, (int)start_position, (int)max_seq_len, (float)attn_scale, stream);
  raise_if_error(qmk_get_last_error());
  cudaError_t e = cudaStreamSynchronize(stream);
  QMK_CHECK(e == cudaSuccess, "qwen_megakernel: cudaStreamSynchronize: %s", cudaGetErrorString(e));
  QmkStatus st;
  raise_if_error(qmk_read_default_status(&st));
  raise_if_status(st);
  return output_log;
}

// Extended operator: explicit workspace, forced tokens, logits, status, trace.
void run(torch::Tensor workspace, torch::Tensor embed_weight, torch::Tensor layer_weights_packed,
         torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
         torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
         std::optional<torch::Tensor> forced_tokens, int64_t first_token, int64_t start_position,
         int64_t num_steps, int64_t num_layers, int64_t max_seq_len, double attn_scale,
         std::optional<torch::Tensor> output_log, std::optional<torch::Tensor> output_token,
         std::optional<torch::Tensor> logits, std::optional<torch::Tensor> final_hidden,
         std::optional<torch::Tensor> status, int64_t timeout_ns, int64_t debug_stall,
         std::optional<torch::Tensor> trace, int64_t trace_step, int64_t poll_backoff_ns,
         int64_t tuning, double temperature, int64_t seed, int64_t stop_at_eos, int64_t eos_token,
         std::optional<torch::Tensor> steps_done, int64_t top_k) {
  QMK_CHECK(num_steps >= 1, "num_steps must be >= 1");
  QMK_CHECK(start_position >= 0, "start_position must be >= 0");
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, start_position + num_steps - 1, max_seq_len);
  check_cuda(workspace, "workspace");
  check_same_device(workspace, embed_weight, "workspace");
  QMK_CHECK(workspace.nbytes() >= qmk_workspace_bytes(), "workspace holds %lld bytes; needs %lld",
            (ll)workspace.nbytes(), (ll)qmk_workspace_bytes());
  QmkRunArgs a;
  memset(&a, 0, sizeof(a));
  int n_forced = 0;
  if (forced_tokens.has_value()) {
    const auto &f = *forced_tokens;
    check_dtype(f, torch::kInt32, "forced_tokens", "int32");
    check_same_device(f, embed_weight, "forced_tokens");
    n_forced = (int)std::min<int64_t>(f.numel(), num_steps);
    a.forced_tokens = static_cast<const int *>(f.data_ptr());
  } else {
    check_token(first_token, "first_token");
  }
  if (output_log.has_value()) {
    check_dtype(*output_log, torch::kInt32, "output_log", "int32");
    check_same_device(*output_log, embed_weight, "output_log");
    QMK_CHECK(output_log->numel() >= num_steps, "output_log must have >= num_steps elements");
    a.output_log = static_cast<int *>(output_log->data_ptr());
  }
  if (output_token.has_value()) {
    check_dtype(*output_token, torch::kInt32, "output_token", "int32");
    check_same_device(*output_token, embed_weight, "output_token");
    QMK_CHECK(output_token->numel() >= 1, "output_token must have >= 1 element");
    a.output_token = static_cast<int *>(output_token->data_ptr());
  }
  if (logits.has_value()) {
    check_dtype(*logits, torch::kFloat32, "logits", "float32");
    check_same_device(*logits, embed_weight, "logits");
    QMK_CHECK(logits->numel() >= num_steps * QMK_VOCAB, "logits must have >= num_steps * %d elements",
              QMK_VOCAB);
    a.logits = static_cast<float *>(logits->data_ptr());
  }
  if (final_hidden.has_value()) {
    check_dtype(*final_hidden, torch::kFloat32, "final_hidden", "float32");
    check_same_device(*final_hidden, embed_weight, "final_hidden");
    QMK_CHECK(final_hidden->numel() >= QMK_HIDDEN, "final_hidden must have >= %d elements", QMK_HIDDEN);
    a.final_hidden = static_cast<float *>(final_hidden->data_ptr());
  }
  if (status.has_value()) {
    const auto &s = *status;
    QMK_CHECK(!s.is_cuda() && s.is_pinned(), "status must be a pinned CPU tensor");
    QMK_CHECK(s.nbytes() >= sizeof(QmkStatus), "status must hold >= %d bytes", (int)sizeof(QmkStatus));
    void *dev = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&dev, s.data_ptr(), 0);
    QMK_CHECK(e == cudaSuccess, "status: cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
    a.status = static_cast<QmkStatus *>(dev);
  }
  if (trace.has_value()) {
    check_dtype(*trace, torch::kInt64, "trace", "int64");
    check_same_device(*trace, embed_weight, "trace");
    const int n = qmk_num_ctas((int)embed_weight.device().index());
    QMK_CHECK(n > 0 && trace->numel() >= (int64_t)n * qmk_trace_words(),
              "trace must have >= num_ctas * qmk_trace_words() = %lld elements",
              (ll)n * (ll)qmk_trace_words());
    a.trace = reinterpret_cast<unsigned long long *>(trace->data_ptr());
    a.trace_step = (int)trace_step;
  }
  a.embed_weight = embed_weight.data_ptr();
  a.layer_weights = reinterpret_cast<const LDGLayerWeights *>(layer_weights_packed.data_ptr());
  a.final_norm_weight = final_norm_weight.data_ptr();
  a.lm_head_weight = lm_head_weight.data_ptr();
  a.cos_table = cos_table.data_ptr();
  a.sin_table = sin_table.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.workspace = workspace.data_ptr();
  a.workspace_bytes = workspace.nbytes();
  a.n_forced = n_forced;
  a.first_token = (int)first_token;
  a.start_position = (int)start_position;
  a.num_steps = (int)num_steps;
  a.num_layers = (int)num_layers;
  a.max_seq_len = (int)max_seq_len;
  a.attn_scale = (float)attn_scale;
  a.timeout_ns = (unsigned long long)std::max<int64_t>(timeout_ns, 0);
  a.debug_stall = (int)debug_stall;
  a.poll_backoff_ns = (unsigned)std::min<int64_t>(std::max<int64_t>(poll_backoff_ns, 0), 4096);
  a.tuning = (unsigned)tuning;
  a.temperature = (float)temperature;
  a.seed = (unsigned long long)seed;
  a.stop_at_eos = stop_at_eos ? 1 : 0;
  a.eos_token = (int)eos_token;
  a.top_k = (int)top_k;
  if (steps_done.has_value()) {
    check_dtype(*steps_done, torch::kInt32, "steps_done", "int32");
    check_same_device(*steps_done, embed_weight, "steps_done");
    a.steps_done = static_cast<int *>(steps_done->data_ptr());
  }
  c10::cuda::CUDAGuard guard(embed_weight.device());
  raise_if_error(qmk_run(&a, c10::cuda::getCurrentCUDAStream().stream()));
}

// Batched decode in the persistent kernel: k_cache / v_cache are
// [QMK_BATCH_SEQS, num_layers, 8, max_seq_len, 128] (one reference-layout
// cache per sequence), first_tokens int32 [QMK_BATCH_SEQS] on the device,
// output_log int32 [num_steps, QMK_BATCH_SEQS].
void run_batch(torch::Tensor workspace, torch::Tensor embed_weight, torch::Tensor layer_weights_packed,
               torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
               torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor first_tokens,
               std::vector<int64_t> start_positions, int64_t num_steps, int64_t num_layers, int64_t max_seq_len,
               double attn_scale, std::optional<torch::Tensor> output_log, std::optional<torch::Tensor> status,
               int64_t timeout_ns) {
  QMK_CHECK(num_steps >= 1, "num_steps must be >= 1");
  QMK_CHECK((int)start_positions.size() == QMK_BATCH_SEQS, "start_positions must have %d entries", QMK_BATCH_SEQS);
  QMK_CHECK(k_cache.dim() == 5 && k_cache.size(0) == QMK_BATCH_SEQS && v_cache.sizes() == k_cache.sizes(),
            "k_cache / v_cache must be [%d, num_layers, 8, max_seq_len, 128]", QMK_BATCH_SEQS);
  QMK_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "caches must be contiguous");
  int64_t last = 0;
  for (int64_t s0 : start_positions) {
    QMK_CHECK(s0 >= 0, "start positions must be >= 0");
    last = std::max<int64_t>(last, s0 + num_steps - 1);
  }
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table, sin_table,
              k_cache.select(0, 0), v_cache.select(0, 0), num_layers, last, max_seq_len);
  check_cuda(workspace, "workspace");
  check_same_device(workspace, embed_weight, "workspace");
  QMK_CHECK(workspace.nbytes() >= qmk_workspace_bytes(), "workspace holds %lld bytes; needs %lld",
            (ll)workspace.nbytes(), (ll)qmk_workspace_bytes());
  check_dtype(first_tokens, torch::kInt32, "first_tokens", "int32");
  check_same_device(first_tokens, embed_weight, "first_tokens");
  QMK_CHECK(first_tokens.numel() >= QMK_BATCH_SEQS, "first_tokens must have %d elements", QMK_BATCH_SEQS);
  QmkBatchRunArgs a;
  memset(&a, 0, sizeof(a));
  if (output_log.has_value()) {
    check_dtype(*output_log, torch::kInt32, "output_log", "int32");
    check_same_device(*output_log, embed_weight, "output_log");
    QMK_CHECK(output_log->numel() >= num_steps * QMK_BATCH_SEQS, "output_log must have >= num_steps * %d elements",
              QMK_BATCH_SEQS);
    a.output_log = static_cast<int *>(output_log->data_ptr());
  }
  if (status.has_value()) {
    const auto &st = *status;
    QMK_CHECK(!st.is_cuda() && st.is_pinned(), "status must be a pinned CPU tensor");
    QMK_CHECK(st.nbytes() >= sizeof(QmkStatus), "status must hold >= %d bytes", (int)sizeof(QmkStatus));
    void *dev = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&dev, st.data_ptr(), 0);
    QMK_CHECK(e == cudaSuccess, "status: cudaHostGetDevicePointer: %s", cudaGetErrorString(e));
    a.status = static_cast<QmkStatus *>(dev);
  }
  a.embed_weight = embed_weight.data_ptr();
  a.layer_weights = reinterpret_cast<const LDGLayerWeights *>(layer_weights_packed.data_ptr());
  a.final_norm_weight = final_norm_weight.data_ptr();
  a.lm_head_weight = lm_head_weight.data_ptr();
  a.cos_table = cos_table.data_ptr();
  a.sin_table = sin_table.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.cache_seq_stride = k_cache.stride(0);
  a.workspace = workspace.data_ptr();
  a.workspace_bytes = workspace.nbytes();
  a.first_tokens = static_cast<const int *>(first_tokens.data_ptr());
  for (int b = 0; b < QMK_BATCH_SEQS; ++b) a.start_positions[b] = (int)start_positions[b];
  a.num_steps = (int)num_steps;
  a.num_layers = (int)num_layers;
  a.max_seq_len = (int)max_seq_len;
  a.attn_scale = (float)attn_scale;
  a.timeout_ns = (unsigned long long)std::max<int64_t>(timeout_ns, 0);
  c10::cuda::CUDAGuard guard(embed_weight.device());
  raise_if_error(qmk_run_batch(&a, c10::cuda::getCurrentCUDAStream().stream()));
}

// Token-parallel forward (prefill / batched decode): qmk_batch_forward.
// layer_ptrs: the num_layers * 11 device pointers in LDGLayerWeights order
// (the GEMMs are launched from the host, so the table is passed by value).
void batch_forward(torch::Tensor workspace, torch::Tensor embed_weight, std::vector<int64_t> layer_ptrs,
                   std::vector<int64_t> fused_ptrs, torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
                   torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache, int64_t kv_seq_stride,
                   int64_t num_seqs, int64_t num_layers, int64_t max_seq_len, double attn_scale,
                   torch::Tensor tokens, torch::Tensor row_seq, torch::Tensor row_pos,
                   std::optional<torch::Tensor> out_rows, std::optional<torch::Tensor> out_tokens,
                   std::optional<torch::Tensor> logits, std::optional<torch::Tensor> status, int64_t causal_run) {
  check_cuda(embed_weight, "embed_weight");
  for (const auto *t : {&workspace, &final_norm_weight, &lm_head_weight, &cos_table, &sin_table, &k_cache, &v_cache,
                        &tokens, &row_seq, &row_pos}) {
    QMK_CHECK(t->is_cuda() && t->device() == embed_weight.device(), "all tensors must be on the weights' device");
    QMK_CHECK(t->is_contiguous(), "tensors must be contiguous");
  }
  check_dtype(embed_weight, torch::kBFloat16, "embed_weight", "bfloat16");
  check_dtype(k_cache, torch::kBFloat16, "k_cache", "bfloat16");
  check_dtype(v_cache, torch::kBFloat16, "v_cache", "bfloat16");
  check_dtype(cos_table, torch::kBFloat16, "cos_table", "bfloat16");
  check_dtype(sin_table, torch::kBFloat16, "sin_table", "bfloat16");
  check_dtype(tokens, torch::kInt32, "tokens", "int32");
  check_dtype(row_seq, torch::kInt32, "row_seq", "int32");
  check_dtype(row_pos, torch::kInt32, "row_pos", "int32");
  const int64_t R = tokens.numel();
  QMK_CHECK(row_seq.numel() == R && row_pos.numel() == R, "tokens, row_seq and row_pos must have equal length");
  QMK_CHECK((int64_t)layer_ptrs.size() == num_layers * 11, "layer_ptrs must hold num_layers * 11 pointers");
  QMK_CHECK(fused_ptrs.empty() || (int64_t)fused_ptrs.size() == num_layers * 2,
            "fused_ptrs must be empty or hold num_layers * 2 pointers");
  QMK_CHECK(cos_table.size(0) >= max_seq_len && sin_table.size(0) >= max_seq_len,
            "RoPE tables need >= max_seq_len rows");
  const int64_t per_seq = num_layers * QMK_NUM_KV_HEADS * max_seq_len * QMK_HEAD_DIM;
  QMK_CHECK(k_cache.numel() >= (num_seqs - 1) * kv_seq_stride + per_seq && v_cache.numel() == k_cache.numel(),
            "caches too small for num_seqs sequences at kv_seq_stride");
  QmkBatchArgs a;
  memset(&a, 0, sizeof(a));
  int64_t O = 0;
  if (out_rows.has_value()) {
    check_dtype(*out_rows, torch::kInt32, "out_rows", "int32");
    check_same_device(*out_rows, embed_weight, "out_rows");
    O = out_rows->numel();
    a.out_rows = static_cast<const int *>(out_rows->data_ptr());
  }
  if (out_tokens.has_value()) {
    check_dtype(*out_tokens, torch::kInt32, "out_tokens", "int32");
    check_same_device(*out_tokens, embed_weight, "out_tokens");
    QMK_CHECK(out_tokens->numel() >= O, "out_tokens must have >= len(out_rows) elements");
    a.out_tokens = static_cast<int *>(out_tokens->data_ptr());
  }
  if (logits.has_value()) {
    check_dtype(*logits, torch::kFloat32, "logits", "float32");
    check_same_device(*logits, embed_weight, "logits");
    QMK_CHECK(logits->is_contiguous() && logits->numel() >= O * QMK_VOCAB,
              "logits must be contiguous with >= len(out_rows) * %d elements", QMK_VOCAB);
    a.logits = static_cast<float *>(logits->data_ptr());
  }
  if (status.has_value()) {
    check_dtype(*status, torch::kInt32, "status", "int32");
    check_same_device(*status, embed_weight, "status");
    a.status = reinterpret_cast<unsigned *>(status->data_ptr());
  }
  std::vector<const void *> ptrs(layer_ptrs.size());
  for (size_t i = 0; i < ptrs.size(); ++i) ptrs[i] = reinterpret_cast<const void *>(layer_ptrs[i]);
  std::vector<const void *> fptrs(fused_ptrs.size());
  for (size_t i = 0; i < fptrs.size(); ++i) fptrs[i] = reinterpret_cast<const void *>(fused_ptrs[i]);
  a.fused_ptrs = fptrs.empty() ? nullptr : fptrs.data();
  a.embed_weight = embed_weight.data_ptr();
  a.layer_ptrs = ptrs.data();
  a.final_norm_weight = final_norm_weight.data_ptr();
  a.lm_head_weight = lm_head_weight.data_ptr();
  a.cos_table = cos_table.data_ptr();
  a.sin_table = sin_table.data_ptr();
  a.k_cache = k_cache.data_ptr();
  a.v_cache = v_cache.data_ptr();
  a.kv_seq_stride = kv_seq_stride;
  a.num_seqs = (int)num_seqs;
  a.num_layers = (int)num_layers;
  a.max_seq_len = (int)max_seq_len;
  a.attn_scale = (float)attn_scale;
  a.num_rows = (int)R;
  a.tokens = static_cast<const int *>(tokens.data_ptr());
  a.row_seq = static_cast<const int *>(row_seq.data_ptr());
  a.row_pos = static_cast<const int *>(row_pos.data_ptr());
  a.num_out = (int)O;
  a.workspace = workspace.data_ptr();
  a.workspace_bytes = workspace.nbytes();
  a.causal_run = causal_run ? 1 : 0;
  c10::cuda::CUDAGuard guard(embed_weight.device());
  raise_if_error(qmk_batch_forward(&a, c10::cuda::getCurrentCUDAStream().stream()));
}

int64_t batch_workspace_bytes(int64_t num_rows, int64_t num_out) {
  const size_t n = qmk_batch_workspace_bytes((int)num_rows, (int)num_out);
  QMK_CHECK(n > 0, "batch_workspace_bytes: num_rows=%lld num_out=%lld out of range", (ll)num_rows, (ll)num_out);
  return (int64_t)n;
}

int64_t workspace_bytes() { return (int64_t)qmk_workspace_bytes(); }

void workspace_init(torch::Tensor workspace) {
  check_cuda(workspace, "workspace");
  c10::cuda::CUDAGuard guard(workspace.device());
  raise_if_error(qmk_workspace_init(workspace.data_ptr(), workspace.nbytes(),
                                    c10::cuda::getCurrentCUDAStream().stream()));
}

std::vector<int64_t> default_status() {
  QmkStatus st;
  raise_if_error(qmk_read_default_status(&st));
  return {(int64_t)st.error_code, (int64_t)st.error_info, (int64_t)st.launches, (int64_t)st.epoch};
}

int64_t num_ctas() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  QMK_CHECK(e == cudaSuccess, "cudaGetDevice: %s", cudaGetErrorString(e));
  const int n = qmk_num_ctas(dev);
  if (n < 0) raise_if_error(qmk_get_last_error());
  return n;
}

int64_t trace_words() { return qmk_trace_words(); }

TORCH_LIBRARY(qwen_megakernel_C, ops) {
  ops.def(
      "decode(Tensor output_token, int input_token_id, "
      "Tensor embed_weight, Tensor layer_weights_packed, "
      "Tensor final_norm_weight, Tensor lm_head_weight, "
      "Tensor cos_table, Tensor sin_table, "
      "Tensor k_cache, Tensor v_cache, "
      "Tensor hidden_buffer, Tensor activations, Tensor residual, "
      "Tensor q, Tensor k, Tensor v, Tensor attn_out, "
      "Tensor mlp_intermediate, Tensor normalized, "
      "Tensor block_max_vals, Tensor block_max_idxs, "
      "int num_layers, int position, int max_seq_len, "
      "float attn_scale) -> ()");
  ops.impl("decode", torch::kCUDA, &decode);

  ops.def(
      "generate_nosync(int first_token_id, int num_steps, "
      "Tensor embed_weight, Tensor layer_weights_packed, "
      "Tensor final_norm_weight, Tensor lm_head_weight, "
      "Tensor cos_table, Tensor sin_table, "
      "Tensor k_cache, Tensor v_cache, "
      "Tensor hidden_buffer, Tensor activations, Tensor residual, "
      "Tensor q, Tensor k, Tensor v, Tensor attn_out, "
      "Tensor mlp_intermediate, Tensor normalized, "
      "Tensor block_max_vals, Tensor block_max_idxs, "
      "int num_layers, int start_position, int max_seq_len, "
      "float attn_scale) -> Tensor");
  ops.impl("generate_nosync", torch::kCUDA, &generate_nosync);

  ops.def(
      "run(Tensor workspace, Tensor embed_weight, Tensor layer_weights_packed, "
      "Tensor final_norm_weight, Tensor lm_head_weight, Tensor cos_table, Tensor sin_table, "
      "Tensor k_cache, Tensor v_cache, Tensor? forced_tokens, int first_token, "
      "int start_position, int num_steps, int num_layers, int max_seq_len, float attn_scale, "
      "Tensor? output_log, Tensor? output_token, Tensor? logits, Tensor? final_hidden, "
      "Tensor? status, int timeout_ns=0, int debug_stall=0, Tensor? trace=None, "
      "int trace_step=0, int poll_backoff_ns=0, int tuning=0, float temperature=0.0, int seed=0, "
      "int stop_at_eos=0, int eos_token=0, Tensor? steps_done=None, int top_k=0) -> ()");
  ops.impl("run", torch::kCUDA, &run);

  ops.def(
      "run_batch(Tensor workspace, Tensor embed_weight, Tensor layer_weights_packed, "
      "Tensor final_norm_weight, Tensor lm_head_weight, Tensor cos_table, Tensor sin_table, "
      "Tensor k_cache, Tensor v_cache, Tensor first_tokens, int[] start_positions, int num_steps, "
      "int num_layers, int max_seq_len, float attn_scale, Tensor? output_log, Tensor? status, "
      "int timeout_ns=0) -> ()");
  ops.impl("run_batch", torch::kCUDA, &run_batch);

  ops.def(
      "batch_forward(Tensor workspace, Tensor embed_weight, int[] layer_ptrs, int[] fused_ptrs, "
      "Tensor final_norm_weight, "
      "Tensor lm_head_weight, Tensor cos_table, Tensor sin_table, Tensor k_cache, Tensor v_cache, "
      "int kv_seq_stride, int num_seqs, int num_layers, int max_seq_len, float attn_scale, "
      "Tensor tokens, Tensor row_seq, Tensor row_pos, Tensor? out_rows, Tensor? out_tokens, "
      "Tensor? logits, Tensor? status, int causal_run=0) -> ()");
  ops.impl("batch_forward", torch::kCUDA, &batch_forward);
  ops.def("batch_workspace_bytes(int num_rows, int num_out) -> int", &batch_workspace_bytes);

  ops.def("workspace_bytes() -> int", &workspace_bytes);
  ops.def("workspace_init(Tensor workspace) -> ()");
  ops.impl("workspace_init", torch::kCUDA, &workspace_init);
  ops.def("default_status() -> int[]", &default_status);
  ops.def("num_ctas() -> int", &num_ctas);
  ops.def("trace_words() -> int", &trace_words);
}

// Importable as a Python module too (mirrors the reference's REGISTER_EXTENSION,
// torch_bindings.cpp:14-19, 157); the ops are registered by loading the library.
static struct PyModuleDef qmk_module = {PyModuleDef_HEAD_INIT, "qwen_megakernel_C", nullptr, 0, nullptr};
PyMODINIT_FUNC PyInit_qwen_megakernel_C() { return PyModule_Create(&qmk_module); }
