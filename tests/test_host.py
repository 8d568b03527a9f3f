"""Host-side logic of the Python API (CPU only)."""

import struct

import pytest
import torch


def test_pack_layer_weights_is_the_reference_blob():
    """11 device pointers per layer, 8 bytes each, in the reference order
    (qwen_megakernel/model.py:97-108)."""
    from qwen_megakernel_b200.model import _pack_layer_weights

    ts = [torch.empty(16) for _ in range(22)]
    blob = _pack_layer_weights(ts, torch.device("cpu"))
    assert blob.dtype == torch.uint8 and blob.numel() == 22 * 8
    ptrs = struct.unpack("22Q", bytes(blob.tolist()))
    assert list(ptrs) == [t.data_ptr() for t in ts]


def test_random_weights_layout_and_determinism():
    from qwen_megakernel_b200.weights import LAYER_TENSORS, random_weights

    a = random_weights(seed=3, device="cpu", max_seq_len=32, num_layers=2)
    b = random_weights(seed=3, device="cpu", max_seq_len=32, num_layers=2)
    assert a["lm_head_weight"] is a["embed_weight"]
    assert a["embed_weight"].shape == (151936, 1024) and a["embed_weight"].dtype == torch.bfloat16
    assert len(a["layer_weights"]) == 22
    for i, (name, shape, kind) in enumerate(LAYER_TENSORS):
        t = a["layer_weights"][i]
        assert tuple(t.shape) == shape and t.dtype == torch.bfloat16, name
        if kind == "norm":
            assert torch.all(t == 1)
        else:
            assert abs(t.float().std().item() - 0.02) < 2e-3
    for x, y in zip(a["layer_weights"], b["layer_weights"]):
        assert torch.equal(x, y)
    assert torch.equal(a["embed_weight"], b["embed_weight"])
    assert a["cos_table"].shape == (32, 128) and a["cos_table"].dtype == torch.bfloat16


def test_decoder_refuses_cpu_weights():
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights

    w = random_weights(seed=1, device="cpu", max_seq_len=16, num_layers=1)
    with pytest.raises(RuntimeError, match="CUDA"):
        Decoder(w)


def _fake_decoder(status):
    from qwen_megakernel_b200 import Decoder

    d = object.__new__(Decoder)
    d._status = torch.tensor(status, dtype=torch.int32)
    return d


def test_status_block_decoding():
    from qwen_megakernel_b200 import DecodeError

    _fake_decoder([0, 0, 5, 100]).check_status()  # no error
    info = (17 << 16) | (6 << 8) | 3
    with pytest.raises(DecodeError, match=r"timed out.*cta 17, site 6, layer 3"):
        _fake_decoder([4, info, 6, 200]).check_status()
    with pytest.raises(DecodeError, match="token id out of range"):
        _fake_decoder([5, 0, 1, 1]).check_status()


def test_native_library_missing_fails_loudly(monkeypatch, tmp_path):
    from qwen_megakernel_b200 import _native

    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_native, "_cdll", None)
    with pytest.raises(_native.NativeLibraryMissing):
        _native.cdll()
