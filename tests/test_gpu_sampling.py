"""On-device sampling (Gumbel-max, keyed by seed and position) and EOS stop of
the decode megakernel (run on a B200: pytest -m gpu).

No reference counterpart: the reference decodes greedily and truncates at EOS
on the host (qwen_megakernel/model.py:242-244).  The checker is
oracle/sampling.py: for every step, the token the kernel drew must be the
Gumbel-max draw over the kernel's own fp32 logits with the same noise.
"""

import numpy as np
import pytest
import torch

from test_gpu_parity import V, small_model

pytestmark = pytest.mark.gpu

T = 0.8
SEED = 2024


def _decoder(seed=7):
    from qwen_megakernel_b200 import Decoder

    return Decoder(small_model(2, seed=seed), max_seq_len=256)


def _sample_run(dec, first, start, n, seed=SEED, temperature=T, top_k=0):
    log = torch.empty(n, dtype=torch.int32, device="cuda")
    logits = torch.empty(n, V, device="cuda")
    dec.decode_steps(n, forced_tokens=torch.tensor([first], dtype=torch.int32, device="cuda"), start_position=start,
                     output_log=log, logits=logits, temperature=temperature, seed=seed, top_k=top_k)
    torch.cuda.synchronize()
    dec.check_status()
    return log.cpu().numpy(), logits.cpu().numpy()


def test_sampled_tokens_are_gumbel_max_draws_over_kernel_logits():
    from oracle.sampling import sample

    dec = _decoder()
    dec.prefill(list(range(100, 120)))
    toks, logits = _sample_run(dec, 5, 20, 24)
    checked = 0
    for t in range(len(toks)):
        want, gap = sample(logits[t], T, SEED, 20 + t)
        if gap > 1e-3:
            assert toks[t] == want, f"step {t}: kernel drew {toks[t]}, oracle {want} (gap {gap})"
            checked += 1
    assert checked >= len(toks) - 2
    # sampling is not greedy here (random logits have small margins)
    assert (toks != logits.argmax(-1)).any()


def test_sampling_reproducible_and_launch_split_invariant():
    a = _decoder()
    a.prefill(list(range(100, 120)))
    ta, _ = _sample_run(a, 5, 20, 16)
    b = _decoder()
    b.prefill(list(range(100, 120)))
    tb1, _ = _sample_run(b, 5, 20, 8)
    tb2, _ = _sample_run(b, int(tb1[-1]), 28, 8)
    assert np.array_equal(ta, np.concatenate([tb1, tb2]))
    c = _decoder()
    c.prefill(list(range(100, 120)))
    tc, _ = _sample_run(c, 5, 20, 16, seed=SEED + 1)
    assert not np.array_equal(ta, tc)


def test_zero_temperature_is_greedy():
    a = _decoder()
    b = _decoder()
    p = list(range(300, 310))
    assert a.generate_ids(p, 12) == b.generate_ids(p, 12, temperature=0.0, seed=5)


def test_eos_stops_the_launch_and_state_stays_consistent():
    prompt = list(range(500, 512))
    full = _decoder().generate_ids(prompt, 16)
    k = next((i for i in range(3, 12) if full[i] not in full[:i]), None)
    if k is None:
        pytest.skip("no token usable as EOS in this greedy run")
    eos = full[k]
    b = _decoder()
    got = b.generate_ids(prompt, 16, eos_token=eos)
    assert got == full[: k + 1]
    assert b.position == len(prompt) - 1 + k + 1
    # a later launch continues correctly from the stopped state
    more_b = b.generate_from(eos, 4)
    c = _decoder()
    c.generate_ids(prompt, k + 1)
    more_c = c.generate_from(eos, 4)
    assert more_b == more_c


def test_eos_in_forced_tokens_does_not_stop():
    prompt = [11, 12, 13, 14, 15, 16]
    a = _decoder()
    full = a.generate_ids(prompt, 6)
    b = _decoder()
    assert b.generate_ids(prompt, 6, eos_token=13) == full[: (full.index(13) + 1 if 13 in full else 6)]
    assert b.position >= len(prompt) - 1


@pytest.mark.parametrize("top_k", [1, 5, 40, 64])
def test_top_k_draws_match_oracle(top_k):
    """Top-k sampling: every drawn token is the oracle's Gumbel-max over the
    top_k largest of the kernel's own logits (top_k = 1: the greedy token)."""
    from oracle.sampling import sample

    dec = _decoder()
    dec.prefill(list(range(100, 120)))
    toks, logits = _sample_run(dec, 5, 20, 16, top_k=top_k)
    for t in range(len(toks)):
        want, gap = sample(logits[t], T, SEED, 20 + t, top_k=top_k)
        if top_k == 1:
            assert toks[t] == int(np.argmax(logits[t]))
        elif gap > 1e-3:
            assert toks[t] == want, f"step {t}: kernel {toks[t]}, oracle {want}"
        top = np.partition(logits[t], -top_k)[-top_k]
        assert logits[t][toks[t]] >= top, "drawn token outside the top-k set"
