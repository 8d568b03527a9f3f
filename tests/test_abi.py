"""The C-ABI library and the torch operator library (CPU only: no kernel runs).

Checks that libqwen_megakernel.so exports every function declared in
include/qwen_megakernel.h, that the host-side argument validation of qmk_run
rejects bad calls before touching a device, and that the torch operators keep
the reference's schemas (reference csrc/torch_bindings.cpp:129-155).
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "qwen_megakernel.h")

# Reference operator schemas, csrc/torch_bindings.cpp:130-140 and :143-153.
REF_DECODE = (
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
    "float attn_scale) -> ()"
)
REF_GENERATE = (
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
    "float attn_scale) -> Tensor"
)


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    src = re.sub(r"typedef struct .*?\}\s*\w+\s*;", "", src, flags=re.S)
    src = re.sub(r"#[^\n]*", "", src)
    names = re.findall(r"\b([A-Za-z_]\w*)\s*\(", src)
    skip = {"if", "sizeof"}
    return sorted({n for n in names if n not in skip})


@pytest.fixture(scope="module")
def lib():
    from qwen_megakernel_b200 import cdll

    return cdll()


def test_header_declares_reference_entry_points():
    names = declared_functions()
    for ref in ("launch_ldg_decode_direct", "launch_ldg_decode_persistent", "launch_ldg_generate_nosync"):
        assert ref in names
    assert "qmk_run" in names and "qmk_workspace_bytes" in names


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_host_queries(lib):
    assert lib.qmk_version().startswith(b"qwen_megakernel_b200")
    ws = lib.qmk_workspace_bytes()
    assert ws > 0 and ws % 4096 == 0
    assert lib.qmk_error_string(0) == b"ok"
    assert lib.qmk_error_string(4) == b"device-side wait timed out"
    # ~64 positions per split, capped by CTAs / 8 and by 18.
    assert lib.qmk_attention_splits(148, 0) == 1
    assert lib.qmk_attention_splits(148, 64) == 1
    assert lib.qmk_attention_splits(148, 65) == 2
    assert lib.qmk_attention_splits(148, 1535) == 18
    assert lib.qmk_attention_splits(148, 32768) == 18
    assert lib.qmk_attention_splits(64, 32768) == 8


def test_workspace_size_matches_torch_op(lib):
    from qwen_megakernel_b200 import ops

    assert ops().workspace_bytes() == lib.qmk_workspace_bytes()


class QmkRunArgs(ctypes.Structure):
    _fields_ = [
        ("embed_weight", ctypes.c_void_p),
        ("layer_weights", ctypes.c_void_p),
        ("final_norm_weight", ctypes.c_void_p),
        ("lm_head_weight", ctypes.c_void_p),
        ("cos_table", ctypes.c_void_p),
        ("sin_table", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("forced_tokens", ctypes.c_void_p),
        ("n_forced", ctypes.c_int),
        ("first_token", ctypes.c_int),
        ("start_position", ctypes.c_int),
        ("num_steps", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("max_seq_len", ctypes.c_int),
        ("attn_scale", ctypes.c_float),
        ("output_log", ctypes.c_void_p),
        ("output_token", ctypes.c_void_p),
        ("logits", ctypes.c_void_p),
        ("final_hidden", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_ulonglong),
        ("debug_stall", ctypes.c_int),
        ("trace", ctypes.c_void_p),
        ("trace_step", ctypes.c_int),
        ("poll_backoff_ns", ctypes.c_uint),
        ("tuning", ctypes.c_uint),
        ("temperature", ctypes.c_float),
        ("seed", ctypes.c_ulonglong),
        ("stop_at_eos", ctypes.c_int),
        ("eos_token", ctypes.c_int),
        ("steps_done", ctypes.c_void_p),
        ("top_k", ctypes.c_int),
    ]


def _valid_args(lib) -> QmkRunArgs:
    a = QmkRunArgs()
    fake = 0x10000  # never dereferenced: validation fails before any launch
    for f in ("embed_weight", "layer_weights", "final_norm_weight", "lm_head_weight", "cos_table",
              "sin_table", "k_cache", "v_cache", "workspace"):
        setattr(a, f, fake)
    a.workspace_bytes = lib.qmk_workspace_bytes()
    a.first_token = 1
    a.start_position = 0
    a.num_steps = 1
    a.num_layers = 28
    a.max_seq_len = 2048
    a.attn_scale = 0.088
    return a


@pytest.mark.parametrize(
    "field,value,code",
    [
        ("embed_weight", 0, 1),
        ("workspace", 0, 6),
        ("workspace_bytes", 16, 6),
        ("num_layers", 0, 1),
        ("num_layers", 65, 1),
        ("num_steps", 0, 1),
        ("start_position", 2048, 1),
        ("start_position", -1, 1),
        ("first_token", 151936, 1),
        ("first_token", -5, 1),
        ("attn_scale", 0.0, 1),
        ("n_forced", 3, 1),  # forced count without a pointer
        ("k_cache", 0x10001, 1),  # misaligned tensor
        ("temperature", -1.0, 1),
        ("temperature", float("nan"), 1),
        ("temperature", float("inf"), 1),
        ("top_k", -1, 1),
        ("top_k", 65, 1),
    ],
)
def test_qmk_run_rejects_bad_arguments(lib, field, value, code):
    a = _valid_args(lib)
    setattr(a, field, value)
    rc = lib.qmk_run(ctypes.byref(a), None)
    assert rc == code
    assert lib.qmk_get_last_error() == code
    assert len(lib.qmk_get_last_error_message()) > 0


def test_qmk_run_rejects_positions_past_max_seq_len(lib):
    a = _valid_args(lib)
    a.start_position = 2040
    a.num_steps = 9  # positions 2040..2048 > max_seq_len - 1
    assert lib.qmk_run(ctypes.byref(a), None) == 1


def test_qmk_run_rejects_bad_eos_token(lib):
    a = _valid_args(lib)
    a.stop_at_eos = 1
    for bad in (-1, 151936):
        a.eos_token = bad
        assert lib.qmk_run(ctypes.byref(a), None) == 1
        assert b"eos_token" in lib.qmk_get_last_error_message()


def test_workspace_init_rejects_small_buffer(lib):
    assert lib.qmk_workspace_init(None, 0, None) == 6


def test_torch_ops_keep_reference_schemas():
    from qwen_megakernel_b200 import ops

    o = ops()
    assert str(o.decode.default._schema) == "qwen_megakernel_C::" + REF_DECODE
    assert str(o.generate_nosync.default._schema) == "qwen_megakernel_C::" + REF_GENERATE
    run = str(o.run.default._schema)
    assert run.startswith("qwen_megakernel_C::run(Tensor workspace")


class QmkBatchRunArgs(ctypes.Structure):
    _fields_ = [
        ("embed_weight", ctypes.c_void_p),
        ("layer_weights", ctypes.c_void_p),
        ("final_norm_weight", ctypes.c_void_p),
        ("lm_head_weight", ctypes.c_void_p),
        ("cos_table", ctypes.c_void_p),
        ("sin_table", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("cache_seq_stride", ctypes.c_longlong),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("first_tokens", ctypes.c_void_p),
        ("start_positions", ctypes.c_int * 4),
        ("num_steps", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("max_seq_len", ctypes.c_int),
        ("attn_scale", ctypes.c_float),
        ("output_log", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_ulonglong),
    ]


def _valid_batch_args(lib) -> QmkBatchRunArgs:
    a = QmkBatchRunArgs()
    fake = 0x10000  # never dereferenced: validation fails before any launch
    for f in ("embed_weight", "layer_weights", "final_norm_weight", "lm_head_weight", "cos_table",
              "sin_table", "k_cache", "v_cache", "workspace", "first_tokens"):
        setattr(a, f, fake)
    a.workspace_bytes = lib.qmk_workspace_bytes()
    a.num_layers = 28
    a.max_seq_len = 2048
    a.cache_seq_stride = 28 * 8 * 2048 * 128
    a.num_steps = 4
    a.attn_scale = 0.088
    for s in range(4):
        a.start_positions[s] = 100 * s
    return a


@pytest.mark.parametrize(
    "field,value,code",
    [
        ("embed_weight", 0, 1),
        ("first_tokens", 0, 1),
        ("workspace", 0, 1),
        ("workspace_bytes", 16, 6),
        ("num_layers", 0, 1),
        ("num_steps", 0, 1),
        ("cache_seq_stride", 1024, 1),  # smaller than one sequence's cache
        ("cache_seq_stride", 28 * 8 * 2048 * 128 + 4, 1),  # not 16-byte aligned
        ("attn_scale", -1.0, 1),
        ("v_cache", 0x10008, 1),  # misaligned tensor
    ],
)
def test_qmk_run_batch_rejects_bad_arguments(lib, field, value, code):
    a = _valid_batch_args(lib)
    setattr(a, field, value)
    assert lib.qmk_run_batch(ctypes.byref(a), None) == code
    assert lib.qmk_get_last_error() == code


def test_qmk_run_batch_rejects_positions_past_max_seq_len(lib):
    a = _valid_batch_args(lib)
    a.start_positions[3] = 2045  # 2045 + 4 steps > 2048
    assert lib.qmk_run_batch(ctypes.byref(a), None) == 1
    assert b"sequence 3" in lib.qmk_get_last_error_message()
    a = _valid_batch_args(lib)
    a.start_positions[1] = -1
    assert lib.qmk_run_batch(ctypes.byref(a), None) == 1


def test_batch_decoder_megakernel_mode_needs_four_sequences():
    from qwen_megakernel_b200 import BatchDecoder
    from qwen_megakernel_b200.weights import random_weights

    w = random_weights(seed=1, device="cpu", max_seq_len=64, num_layers=1)
    with pytest.raises(ValueError, match="exactly 4"):
        BatchDecoder(w, 3, max_seq_len=64, decode="megakernel")
    with pytest.raises(ValueError, match="decode must be"):
        BatchDecoder(w, 4, max_seq_len=64, decode="fast")


def test_batch_status_bits_match_header():
    """The Python decoder of the token-parallel path's status word uses the
    bit values include/qwen_megakernel.h defines, and every bit has a
    message in BatchForward.check_status."""
    from qwen_megakernel_b200 import batch

    defines = dict(re.findall(r"#define\s+(QMK_BATCH_\w+)\s+(\d+)u?", open(HEADER).read()))
    pairs = {
        "QMK_BATCH_MAX_ROWS": batch.MAX_ROWS,
        "QMK_BATCH_BAD_TOKEN": batch.BAD_TOKEN,
        "QMK_BATCH_BAD_ROW": batch.BAD_ROW,
        "QMK_BATCH_TIMEOUT": batch.TIMEOUT,
        "QMK_BATCH_COPIES_PENDING": batch.COPIES_PENDING,
        "QMK_BATCH_SEQS": batch.MEGAKERNEL_SEQS,
    }
    for name, value in pairs.items():
        assert int(defines[name]) == value, name
    bits = [batch.BAD_TOKEN, batch.BAD_ROW, batch.TIMEOUT, batch.COPIES_PENDING]
    assert len(set(bits)) == len(bits) and all(b & (b - 1) == 0 for b in bits)
    src = open(batch.__file__).read()
    for name in ("BAD_TOKEN", "BAD_ROW", "TIMEOUT", "COPIES_PENDING"):
        assert f"code & {name}" in src, name
