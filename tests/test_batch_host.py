"""Host side of the token-parallel path (CPU only: no kernel runs).

qmk_batch_forward validates its arguments before it touches a device;
qmk_batch_workspace_bytes and the torch operator agree on the workspace size.
"""

import ctypes

import pytest

QMK_ERR_ARGS = 1
QMK_ERR_WORKSPACE = 6
MAX_ROWS = 4096


class QmkBatchArgs(ctypes.Structure):
    _fields_ = [
        ("embed_weight", ctypes.c_void_p),
        ("layer_ptrs", ctypes.c_void_p),
        ("fused_ptrs", ctypes.c_void_p),
        ("final_norm_weight", ctypes.c_void_p),
        ("lm_head_weight", ctypes.c_void_p),
        ("cos_table", ctypes.c_void_p),
        ("sin_table", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("kv_seq_stride", ctypes.c_longlong),
        ("num_seqs", ctypes.c_int),
        ("num_layers", ctypes.c_int),
        ("max_seq_len", ctypes.c_int),
        ("attn_scale", ctypes.c_float),
        ("num_rows", ctypes.c_int),
        ("tokens", ctypes.c_void_p),
        ("row_seq", ctypes.c_void_p),
        ("row_pos", ctypes.c_void_p),
        ("num_out", ctypes.c_int),
        ("out_rows", ctypes.c_void_p),
        ("out_tokens", ctypes.c_void_p),
        ("logits", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
        ("causal_run", ctypes.c_int),
    ]


@pytest.fixture(scope="module")
def lib():
    from qwen_megakernel_b200 import cdll

    lib = cdll()
    lib.qmk_batch_workspace_bytes.restype = ctypes.c_size_t
    lib.qmk_batch_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.qmk_batch_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    return lib


def test_workspace_bytes(lib):
    from qwen_megakernel_b200 import ops

    for rows, out in ((1, 1), (64, 64), (1024, 1), (MAX_ROWS, 0)):
        n = lib.qmk_batch_workspace_bytes(rows, out)
        assert n > 0 and n % 256 == 0
        assert ops().batch_workspace_bytes(rows, out) == n
    # grows with rows and outputs (a larger workspace serves smaller calls)
    assert lib.qmk_batch_workspace_bytes(65, 1) > lib.qmk_batch_workspace_bytes(64, 1)
    assert lib.qmk_batch_workspace_bytes(64, 2) > lib.qmk_batch_workspace_bytes(64, 1)
    for rows, out in ((0, 0), (MAX_ROWS + 1, 0), (4, 5), (4, -1)):
        assert lib.qmk_batch_workspace_bytes(rows, out) == 0


def test_workspace_bytes_monotone_in_rows(lib):
    """A workspace sized for R rows serves every smaller call (BatchForward
    grows its buffer only): the size never decreases with rows or outputs,
    across the split-K and split-attention thresholds (64 rows) and the
    tensor-core attention limit (2048 rows)."""
    prev = 0
    for rows in list(range(1, 300)) + [1000, 2047, 2048, 2049, 3000, MAX_ROWS]:
        n = lib.qmk_batch_workspace_bytes(rows, 1)
        assert n >= prev, f"workspace shrinks at {rows} rows"
        prev = n
        assert lib.qmk_batch_workspace_bytes(rows, rows) >= n


def _valid(lib, layers=28):
    fake = 0x10000  # never dereferenced: validation fails before any launch
    table = (ctypes.c_void_p * (layers * 11))(*([fake] * (layers * 11)))
    a = QmkBatchArgs()
    for f in ("embed_weight", "final_norm_weight", "lm_head_weight", "cos_table", "sin_table", "k_cache", "v_cache",
              "tokens", "row_seq", "row_pos", "out_rows", "workspace"):
        setattr(a, f, fake)
    a.layer_ptrs = ctypes.cast(table, ctypes.c_void_p)
    a.num_seqs = 1
    a.num_layers = layers
    a.max_seq_len = 2048
    a.attn_scale = 0.088
    a.num_rows = 16
    a.num_out = 1
    a.workspace_bytes = 1 << 20  # too small on purpose (see below)
    return a, table


@pytest.mark.parametrize(
    "field,value",
    [
        ("embed_weight", 0),
        ("layer_ptrs", 0),
        ("tokens", 0),
        ("row_pos", 0),
        ("num_rows", 0),
        ("num_rows", MAX_ROWS + 1),
        ("num_out", 17),
        ("num_out", -1),
        ("out_rows", 0),
        ("num_layers", 0),
        ("num_layers", 65),
        ("max_seq_len", 0),
        ("num_seqs", 0),
        ("num_seqs", 2),  # two sequences need a kv_seq_stride of at least one cache
    ],
)
def test_forward_rejects_bad_arguments(lib, field, value):
    a, table = _valid(lib)
    setattr(a, field, value)
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_ARGS
    assert len(lib.qmk_get_last_error_message()) > 0


def test_forward_rejects_unaligned_cache(lib):
    """Cache rows are copied with 16-byte-aligned bulk copies."""
    a, table = _valid(lib)
    a.k_cache = 0x10008
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_ARGS
    assert b"aligned" in lib.qmk_get_last_error_message()
    a, table = _valid(lib)
    a.num_seqs = 2
    a.kv_seq_stride = 28 * 8 * 2048 * 128 + 4
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_ARGS
    assert b"multiple of 8" in lib.qmk_get_last_error_message()


def test_forward_rejects_null_layer_pointer(lib):
    a, table = _valid(lib)
    table[5 * 11 + 6] = None  # o_proj of layer 5
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_ARGS
    assert b"layer pointer 61" in lib.qmk_get_last_error_message()


def test_forward_rejects_small_or_misaligned_workspace(lib):
    a, table = _valid(lib)
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_WORKSPACE
    a.workspace_bytes = lib.qmk_batch_workspace_bytes(16, 1)
    a.workspace = 0x10010  # not 256-byte aligned
    assert lib.qmk_batch_forward(ctypes.byref(a), None) == QMK_ERR_WORKSPACE
