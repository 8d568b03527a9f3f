"""qmk_generate_static: the allocation-free entry point (no reference
counterpart).  It must give the same tokens and cache as the existing
reference entry point launch_ldg_generate_nosync on the same inputs, on two
calls in a row (the second continuing the first), and reject a step count
beyond the capacity of its static token log before touching a device.

Collected last on purpose: it must pass both alone and after every other
test of the suite (the static scratch array is shared by all calls of the
process on a device).
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, TOL_MAX_ABS

LIB = os.path.join(ROOT, "qwen_megakernel_b200", "libqwen_megakernel.so")
QMK_OK = 0
QMK_ERR_ARGS = 1
MAX_STEPS = 4096  # QMK_STATIC_MAX_STEPS in include/qwen_megakernel.h


def _lib():
    lib = ctypes.CDLL(LIB)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.qmk_generate_static.restype = i
    lib.qmk_generate_static.argtypes = [i, i, vp, vp, vp, vp, vp, vp, vp, vp, i, i, i, f, vp]
    lib.qmk_static_scratch_ptrs.restype = i
    lib.qmk_static_scratch_ptrs.argtypes = [ctypes.POINTER(vp), ctypes.POINTER(vp)]
    lib.qmk_get_last_error_message.restype = ctypes.c_char_p
    lib.launch_ldg_generate_nosync.restype = None
    lib.launch_ldg_generate_nosync.argtypes = [i, i] + [vp] * 20 + [i, i, i, f, vp]
    return lib


def test_static_entry_rejects_steps_beyond_capacity():
    lib = _lib()
    null = [None] * 8
    for steps in (0, MAX_STEPS + 1):
        rc = lib.qmk_generate_static(1, steps, *null, 2, 0, 64, 0.088, None)
        assert rc == QMK_ERR_ARGS
        msg = lib.qmk_get_last_error_message().decode()
        assert "num_steps" in msg and str(MAX_STEPS) in msg


def _copy_to_host(dev_ptr: int, nbytes: int) -> np.ndarray:
    from cuda.bindings import runtime as rt

    out = np.zeros(nbytes, dtype=np.uint8)
    (err,) = rt.cudaMemcpy(out.ctypes.data, dev_ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return out


@pytest.mark.gpu
def test_static_entry_matches_reference_entry_on_two_calls():
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights

    lib = _lib()
    w = random_weights(seed=11, device="cuda", max_seq_len=128, num_layers=2, norm_std=0.1)
    dec = Decoder(w, max_seq_len=128)  # owns the packed layer table used by both paths
    L, S = dec.num_layers, dec.max_seq_len
    scale = 1.0 / np.sqrt(128.0)
    k_ref, v_ref = torch.zeros_like(dec.k_cache), torch.zeros_like(dec.v_cache)
    k_st, v_st = torch.zeros_like(dec.k_cache), torch.zeros_like(dec.v_cache)
    scratch = [torch.zeros(4096, dtype=torch.float32, device="cuda") for _ in range(10)]
    log_ref = torch.zeros(MAX_STEPS, dtype=torch.int32, device="cuda")
    weights = [dec._embed_weight, dec._layer_weights_packed, dec._final_norm_weight, dec._lm_head_weight,
               dec._cos_table, dec._sin_table]
    wp = [t.data_ptr() for t in weights]
    stream = torch.cuda.current_stream().cuda_stream

    log_p, status_p = ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.qmk_static_scratch_ptrs(ctypes.byref(log_p), ctypes.byref(status_p)) == QMK_OK
    launches = int(_copy_to_host(status_p.value, 16).view(np.uint32)[2])
    first, start, steps = 42, 0, 8
    all_tokens = [first]
    for call in range(2):
        lib.launch_ldg_generate_nosync(first, steps, *wp, k_ref.data_ptr(), v_ref.data_ptr(),
                                       *[t.data_ptr() for t in scratch], None,
                                       log_ref.data_ptr(), L, start, S, scale, stream)
        rc = lib.qmk_generate_static(first, steps, *wp, k_st.data_ptr(), v_st.data_ptr(), L, start, S, scale,
                                     stream)
        assert rc == QMK_OK, lib.qmk_get_last_error_message().decode()
        torch.cuda.synchronize()
        assert lib.qmk_static_scratch_ptrs(ctypes.byref(log_p), ctypes.byref(status_p)) == QMK_OK
        status = _copy_to_host(status_p.value, 16).view(np.uint32)
        assert status[0] == 0, f"device error {status[0]:#x}, info {status[1]:#x}"
        # the static status block is written by the launch's last CTA: a
        # launch that never ran would leave the previous count in place
        assert int(status[2]) == launches + 1, f"call {call}: launches {status[2]} after {launches}"
        launches += 1
        toks_st = _copy_to_host(log_p.value, 4 * steps).view(np.int32)
        toks_ref = log_ref[:steps].cpu().numpy()
        assert np.array_equal(toks_st, toks_ref), f"call {call}: {toks_st} vs {toks_ref}"
        n = start + steps
        for a, b in ((k_st, k_ref), (v_st, v_ref)):
            d = (a[:, :, :n].float() - b[:, :, :n].float()).abs().max().item()
            assert d <= TOL_MAX_ABS, f"call {call}: cache differs by {d}"
        assert k_st[:, :, n:].abs().max().item() == 0.0
        all_tokens += [int(t) for t in toks_st]
        # the second call continues the first from its last token
        first, start = int(toks_st[-1]), start + steps

    # parity of the static entry's own output against the oracle: teacher
    # forced on the kernel's token stream, identical greedy tokens wherever
    # the oracle's top-2 gap exceeds the tolerance
    from oracle.qwen3_mirror import MirrorDecoder

    ref = MirrorDecoder(w, S, device="cuda").prefill(all_tokens[:-1], 0)
    top2 = ref.topk(2, dim=-1).values
    confident = ((top2[:, 0] - top2[:, 1]) > TOL_MAX_ABS).cpu().numpy()
    want = ref.argmax(-1).cpu().numpy()
    got = np.array(all_tokens[1:])
    assert confident.sum() >= 4
    assert np.array_equal(got[confident], want[confident])
