"""Failure detection on the GPU without faulting it (pytest -m gpu).

* A wait that can never be satisfied (test hook: one CTA polls for a flag
  value no CTA writes) must expire after the launch's short wait limit, report
  QMK_ERR_TIMEOUT through the host-visible status block, and leave the CUDA
  context usable: the next launches on the same and on a fresh decoder are
  correct.
* A bad token id inside a device-side forced-token stream is reported as
  QMK_ERR_TOKEN (the kernel substitutes id 0, so nothing is read out of range).
* Host-side validation rejects out-of-range positions before any launch.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from qwen_megakernel_b200.weights import random_weights

    return random_weights(seed=9, device="cuda", max_seq_len=64, num_layers=2, norm_std=0.1)


def test_expired_wait_reports_timeout_and_context_survives():
    from qwen_megakernel_b200 import DecodeError, Decoder

    w = _model()
    ref = Decoder(w, max_seq_len=64)
    want = [ref.step(t) for t in (5, 6, 7)]

    dec = Decoder(w, max_seq_len=64, timeout_ns=20_000_000)  # 20 ms per wait
    out = torch.full((1,), 1234, dtype=torch.int32, device="cuda")
    dec.decode_steps(1, first_token=5, output_token=out, debug_stall=1)
    torch.cuda.synchronize()
    with pytest.raises(DecodeError, match="timed out"):
        dec.check_status()
    assert int(out.item()) == -1  # no token is reported for an aborted launch
    # the same decoder (same workspace) and a fresh one keep working
    dec.reset()
    assert [dec.step(t) for t in (5, 6, 7)] == want
    again = Decoder(w, max_seq_len=64)
    assert [again.step(t) for t in (5, 6, 7)] == want


def test_stall_on_a_late_cta_is_also_reported():
    from qwen_megakernel_b200 import DecodeError, Decoder, ops

    w = _model()
    dec = Decoder(w, max_seq_len=64, timeout_ns=20_000_000)
    n = ops().num_ctas()
    dec.decode_steps(3, first_token=11, debug_stall=n)  # the last CTA stalls
    torch.cuda.synchronize()
    with pytest.raises(DecodeError, match=r"timed out.*cta %d" % (n - 1)):
        dec.check_status()
    dec.reset()
    assert 0 <= dec.step(11) < 151936


def test_bad_forced_token_is_reported():
    from qwen_megakernel_b200 import DecodeError, Decoder

    w = _model()
    dec = Decoder(w, max_seq_len=64)
    bad = torch.tensor([3, 151936 + 5, 4], dtype=torch.int32, device="cuda")
    dec.decode_steps(3, forced_tokens=bad)
    torch.cuda.synchronize()
    with pytest.raises(DecodeError, match="token id out of range"):
        dec.check_status()
    dec.reset()
    assert 0 <= dec.step(3) < 151936


def test_host_validation():
    from qwen_megakernel_b200 import Decoder, ops

    w = _model()
    dec = Decoder(w, max_seq_len=64)
    dec.position = 63
    assert 0 <= dec.step(1) < 151936  # last valid position
    with pytest.raises(ValueError):
        dec.decode_steps(1)  # position 64 == max_seq_len
    with pytest.raises(ValueError):
        dec.position = 65
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="outside"):
        dec.decode_steps(1, first_token=151936, output_token=out, start_position=0)
    with pytest.raises(RuntimeError):
        ops().run(dec._workspace[:16], w["embed_weight"], dec._layer_weights_packed, w["final_norm_weight"],
                  w["lm_head_weight"], w["cos_table"], w["sin_table"], dec.k_cache, dec.v_cache, None, 1, 0, 1, 2,
                  64, 0.088, None, None, None, None, None, 0, 0)
