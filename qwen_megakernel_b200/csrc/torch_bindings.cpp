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
//                           forced-token stream, fp32 logits, status block
//   workspace_bytes()    -> qmk_workspace_bytes
//   workspace_init(ws)   -> qmk_workspace_init
//   default_status()     -> qmk_read_default_status (after a synchronize)
//   num_ctas()           -> qmk_num_ctas(current device)
#include <Python.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <torch/all.h>
#include <torch/library.h>

#include "qwen_megakernel.h"

namespace {

void check_cuda(const torch::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

void check_bf16(const torch::Tensor &t, const char *name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16, got ", t.scalar_type());
}

void check_same_device(const torch::Tensor &t, const torch::Tensor &ref, const char *name) {
  TORCH_CHECK(t.device() == ref.device(), name, " is on ", t.device(), " but the weights are on ",
              ref.device());
}

// Shared checks of the model tensors of every operator.
void check_model(const torch::Tensor &embed_weight, const torch::Tensor &layer_weights_packed,
                 const torch::Tensor &final_norm_weight, const torch::Tensor &lm_head_weight,
                 const torch::Tensor &cos_table, const torch::Tensor &sin_table,
                 const torch::Tensor &k_cache, const torch::Tensor &v_cache, int64_t num_layers,
                 int64_t last_position, int64_t max_seq_len) {
  check_bf16(embed_weight, "embed_weight");
  TORCH_CHECK(embed_weight.dim() == 2 && embed_weight.size(0) == QMK_VOCAB &&
                  embed_weight.size(1) == QMK_HIDDEN,
              "embed_weight must be [", QMK_VOCAB, ", ", QMK_HIDDEN, "], got ", embed_weight.sizes());
  check_bf16(lm_head_weight, "lm_head_weight");
  TORCH_CHECK(lm_head_weight.sizes() == embed_weight.sizes(), "lm_head_weight must be [", QMK_VOCAB,
              ", ", QMK_HIDDEN, "]");
  check_bf16(final_norm_weight, "final_norm_weight");
  TORCH_CHECK(final_norm_weight.numel() == QMK_HIDDEN, "final_norm_weight must have ", QMK_HIDDEN,
              " elements");
  check_cuda(layer_weights_packed, "layer_weights_packed");
  TORCH_CHECK(num_layers >= 1 && num_layers <= QMK_MAX_LAYERS, "num_layers must be in [1, ",
              QMK_MAX_LAYERS, "], got ", num_layers);
  TORCH_CHECK(layer_weights_packed.nbytes() >= (size_t)num_layers * sizeof(LDGLayerWeights),
              "layer_weights_packed holds ", layer_weights_packed.nbytes(), " bytes; ", num_layers,
              " layers need ", (size_t)num_layers * sizeof(LDGLayerWeights));
  check_bf16(cos_table, "cos_table");
  check_bf16(sin_table, "sin_table");
  TORCH_CHECK(cos_table.dim() == 2 && cos_table.size(1) == QMK_HEAD_DIM,
              "cos_table must be [rows, 128], got ", cos_table.sizes());
  TORCH_CHECK(sin_table.sizes() == cos_table.sizes(), "sin_table must match cos_table");
  TORCH_CHECK(cos_table.size(0) > last_position, "cos/sin tables have ", cos_table.size(0),
              " rows; position ", last_position, " needs ", last_position + 1);
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(0) >= num_layers && k_cache.size(1) == QMK_NUM_KV_HEADS &&
                  k_cache.size(2) == max_seq_len && k_cache.size(3) == QMK_HEAD_DIM,
              "k_cache must be [>=num_layers, 8, max_seq_len=", max_seq_len, ", 128], got ",
              k_cache.sizes());
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes(), "v_cache must match k_cache");
  TORCH_CHECK(last_position < max_seq_len, "position ", last_position, " >= max_seq_len ", max_seq_len);
  for (const torch::Tensor *t : {&layer_weights_packed, &final_norm_weight, &lm_head_weight, &cos_table,
                                 &sin_table, &k_cache, &v_cache})
    check_same_device(*t, embed_weight, "tensor");
}

void raise_if_error(int rc) {
  if (rc != QMK_OK) {
    TORCH_CHECK(false, "qwen_megakernel: ", qmk_error_string(rc), ": ", qmk_get_last_error_message());
  }
}

void raise_if_status(const QmkStatus &st) {
  if (st.error_code != QMK_OK) {
    TORCH_CHECK(false, "qwen_megakernel: device error: ", qmk_error_string((int)st.error_code),
                " (cta ", (st.error_info >> 16), ", site ", ((st.error_info >> 8) & 0xff), ", layer ",
                (st.error_info & 0xff), ")");
  }
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
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, position, max_seq_len);
  TORCH_CHECK(position >= 0, "position must be >= 0");
  TORCH_CHECK(input_token_id >= 0 && input_token_id < QMK_VOCAB, "input_token_id ", input_token_id,
              " outside [0, ", QMK_VOCAB, ")");
  check_cuda(output_token, "output_token");
  TORCH_CHECK(output_token.scalar_type() == torch::kInt32 && output_token.numel() >= 1,
              "output_token must be int32 with >= 1 element");
  check_cuda(normalized, "normalized");
  TORCH_CHECK(normalized.scalar_type() == torch::kFloat32 && normalized.numel() >= QMK_HIDDEN,
              "normalized must be float32 with >= ", QMK_HIDDEN, " elements");
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
  TORCH_CHECK(num_steps >= 1, "num_steps must be >= 1");
  TORCH_CHECK(start_position >= 0, "start_position must be >= 0");
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, start_position + num_steps - 1, max_seq_len);
  TORCH_CHECK(first_token_id >= 0 && first_token_id < QMK_VOCAB, "first_token_id ", first_token_id,
              " outside [0, ", QMK_VOCAB, ")");
  check_cuda(normalized, "normalized");
  TORCH_CHECK(normalized.scalar_type() == torch::kFloat32 && normalized.numel() >= QMK_HIDDEN,
              "normalized must be float32 with >= ", QMK_HIDDEN, " elements");
  c10::cuda::CUDAGuard guard(embed_weight.device());
  auto stream = c10::cuda::getCurrentCUDAStream().stream();
  auto output_log =
      torch::empty({num_steps}, torch::dtype(torch::kInt32).device(embed_weight.device()));
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
  TORCH_CHECK(e == cudaSuccess, "qwen_megakernel: cudaStreamSynchronize: ", cudaGetErrorString(e));
  QmkStatus st;
  raise_if_error(qmk_read_default_status(&st));
  raise_if_status(st);
  return output_log;
}

// Extended operator: explicit workspace, forced tokens, logits, status.
void run(torch::Tensor workspace, torch::Tensor embed_weight, torch::Tensor layer_weights_packed,
         torch::Tensor final_norm_weight, torch::Tensor lm_head_weight, torch::Tensor cos_table,
         torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
         std::optional<torch::Tensor> forced_tokens, int64_t first_token, int64_t start_position,
         int64_t num_steps, int64_t num_layers, int64_t max_seq_len, double attn_scale,
         std::optional<torch::Tensor> output_log, std::optional<torch::Tensor> output_token,
         std::optional<torch::Tensor> logits, std::optional<torch::Tensor> final_hidden,
         std::optional<torch::Tensor> status, int64_t timeout_ns, int64_t debug_stall) {
  TORCH_CHECK(num_steps >= 1, "num_steps must be >= 1");
  TORCH_CHECK(start_position >= 0, "start_position must be >= 0");
  check_model(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
              sin_table, k_cache, v_cache, num_layers, start_position + num_steps - 1, max_seq_len);
  check_cuda(workspace, "workspace");
  check_same_device(workspace, embed_weight, "workspace");
  TORCH_CHECK(workspace.nbytes() >= qmk_workspace_bytes(), "workspace holds ", workspace.nbytes(),
              " bytes; needs ", qmk_workspace_bytes());
  QmkRunArgs a;
  memset(&a, 0, sizeof(a));
  int n_forced = 0;
  if (forced_tokens.has_value()) {
    const auto &f = *forced_tokens;
    check_cuda(f, "forced_tokens");
    check_same_device(f, embed_weight, "forced_tokens");
    TORCH_CHECK(f.scalar_type() == torch::kInt32, "forced_tokens must be int32");
    n_forced = (int)std::min<int64_t>(f.numel(), num_steps);
    a.forced_tokens = static_cast<const int *>(f.data_ptr());
  } else {
    TORCH_CHECK(first_token >= 0 && first_token < QMK_VOCAB, "first_token ", first_token,
                " outside [0, ", QMK_VOCAB, ")");
  }
  if (output_log.has_value()) {
    check_cuda(*output_log, "output_log");
    check_same_device(*output_log, embed_weight, "output_log");
    TORCH_CHECK(output_log->scalar_type() == torch::kInt32 && output_log->numel() >= num_steps,
                "output_log must be int32 with >= num_steps elements");
    a.output_log = static_cast<int *>(output_log->data_ptr());
  }
  if (output_token.has_value()) {
    check_cuda(*output_token, "output_token");
    check_same_device(*output_token, embed_weight, "output_token");
    TORCH_CHECK(output_token->scalar_type() == torch::kInt32 && output_token->numel() >= 1,
                "output_token must be int32 with >= 1 element");
    a.output_token = static_cast<int *>(output_token->data_ptr());
  }
  if (logits.has_value()) {
    check_cuda(*logits, "logits");
    check_same_device(*logits, embed_weight, "logits");
    TORCH_CHECK(logits->scalar_type() == torch::kFloat32 && logits->numel() >= num_steps * QMK_VOCAB,
                "logits must be float32 with >= num_steps * ", QMK_VOCAB, " elements");
    a.logits = static_cast<float *>(logits->data_ptr());
  }
  if (final_hidden.has_value()) {
    check_cuda(*final_hidden, "final_hidden");
    check_same_device(*final_hidden, embed_weight, "final_hidden");
    TORCH_CHECK(final_hidden->scalar_type() == torch::kFloat32 && final_hidden->numel() >= QMK_HIDDEN,
                "final_hidden must be float32 with >= ", QMK_HIDDEN, " elements");
    a.final_hidden = static_cast<float *>(final_hidden->data_ptr());
  }
  if (status.has_value()) {
    const auto &s = *status;
    TORCH_CHECK(!s.is_cuda() && s.is_pinned(), "status must be a pinned CPU tensor");
    TORCH_CHECK(s.nbytes() >= sizeof(QmkStatus), "status must hold >= ", sizeof(QmkStatus), " bytes");
    void *dev = nullptr;
    cudaError_t e = cudaHostGetDevicePointer(&dev, s.data_ptr(), 0);
    TORCH_CHECK(e == cudaSuccess, "status: cudaHostGetDevicePointer: ", cudaGetErrorString(e));
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
  c10::cuda::CUDAGuard guard(embed_weight.device());
  raise_if_error(qmk_run(&a, c10::cuda::getCurrentCUDAStream().stream()));
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
  TORCH_CHECK(e == cudaSuccess, "cudaGetDevice: ", cudaGetErrorString(e));
  const int n = qmk_num_ctas(dev);
  raise_if_error(n < 0 ? qmk_get_last_error() : QMK_OK);
  return n;
}

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
      "Tensor? status, int timeout_ns=0, int debug_stall=0) -> ()");
  ops.impl("run", torch::kCUDA, &run);

  ops.def("workspace_bytes() -> int", &workspace_bytes);
  ops.def("workspace_init(Tensor workspace) -> ()");
  ops.impl("workspace_init", torch::kCUDA, &workspace_init);
  ops.def("default_status() -> int[]", &default_status);
  ops.def("num_ctas() -> int", &num_ctas);
}

// Importable as a Python module too (mirrors the reference's REGISTER_EXTENSION,
// torch_bindings.cpp:14-19, 157); the ops are registered by loading the library.
static struct PyModuleDef qmk_module = {PyModuleDef_HEAD_INIT, "qwen_megakernel_C", nullptr, 0, nullptr};
PyMODINIT_FUNC PyInit_qwen_megakernel_C() { return PyModule_Create(&qmk_module); }
