"""Batched decode in the persistent kernel (qmk_run_batch, 4 sequences).

The batched instance runs every GEMV phase in one pass over the weight
tiles for all sequences (q|k|v, gate/up and the LM head on the tensor cores
with the 4 inputs as the MMA's N columns) and gives each sequence its own
attention items, so each sequence should decode as the single-sequence
kernel decodes it alone (the attention's position splits and the GEMV
summation order differ, hence the margin test), and as the oracle does."""

import pytest
import torch

from conftest import TOL_MAX_ABS
from test_gpu_parity import V, small_model

pytestmark = pytest.mark.gpu

SEQS = 4


def _prompts(lens, seed):
    g = torch.Generator().manual_seed(seed)
    return [[int(t) for t in torch.randint(0, V, (n,), generator=g)] for n in lens]


def test_megakernel_batch_matches_single_sequence_kernel():
    """4 sequences of different prompt lengths (token-parallel prefill), then
    24 greedy steps in one batched launch; each sequence against the
    single-sequence kernel decoding it alone: identical tokens wherever that
    decoder's top-2 logit gap is clear."""
    from qwen_megakernel_b200 import BatchDecoder, Decoder

    w = small_model(2, seed=31)
    prompts = _prompts([7, 40, 65, 130], 41)
    bd = BatchDecoder(w, SEQS, max_seq_len=256, decode="megakernel")
    assert bd.decode_mode == "megakernel"
    first = bd.prefill(prompts)
    log = bd.generate(first, 24)
    torch.cuda.synchronize()
    bd.check_status()
    log = log.cpu()
    assert bd.positions == [len(p) + 24 for p in prompts]
    for s in range(SEQS):
        dec = Decoder(w, max_seq_len=256)
        t0 = dec.prefill(prompts[s])
        assert t0 == first[s]
        lg = torch.empty(24, V, device="cuda")
        forced = torch.tensor([t0] + log[:-1, s].tolist(), dtype=torch.int32, device="cuda")
        dec.decode_steps(24, forced_tokens=forced, logits=lg)
        torch.cuda.synchronize()
        dec.check_status()
        top2 = lg.topk(2, dim=-1).values
        conf = ((top2[:, 0] - top2[:, 1]) > TOL_MAX_ABS).cpu()
        assert conf.sum() >= 12
        assert torch.equal(lg.argmax(-1).cpu()[conf], log[:, s].long()[conf]), f"sequence {s}"


def test_megakernel_batch_equals_token_parallel_tokens():
    """The same batch through the token-parallel decode (CUDA-graph steps)
    and through the persistent kernel: the confident greedy tokens agree."""
    from qwen_megakernel_b200 import BatchDecoder

    w = small_model(2, seed=37)
    prompts = _prompts([12, 12, 90, 3], 43)
    logs = {}
    for mode in ("token_parallel", "megakernel"):
        bd = BatchDecoder(w, SEQS, max_seq_len=256, decode=mode)
        first = bd.prefill(prompts)
        logs[mode] = (first, bd.generate(first, 16).cpu())
        torch.cuda.synchronize()
        bd.check_status()
    assert logs["megakernel"][0] == logs["token_parallel"][0]
    # same first disagreement-free prefix of at least 4 steps per sequence
    a, b = logs["megakernel"][1], logs["token_parallel"][1]
    for s in range(SEQS):
        assert torch.equal(a[:4, s], b[:4, s]), f"sequence {s}"


def test_megakernel_batch_full_depth_vs_oracle(cuda_weights):
    """BASELINE config 4 at B = 4 through the persistent kernel: the 28-layer
    model, 1024-token prompts, 8 greedy steps in one launch; every generated
    token equals the oracle's greedy token (teacher forced on the same
    prefix) wherever the oracle's top-2 gap is clear."""
    from oracle.qwen3_mirror import MirrorDecoder
    from qwen_megakernel_b200 import BatchDecoder

    P, steps = 1024, 8
    msl = P + steps + 8
    g = torch.Generator().manual_seed(500)
    prompts = [[int(t) for t in torch.randint(0, V, (P,), generator=g)] for _ in range(SEQS)]
    bd = BatchDecoder(cuda_weights, SEQS, max_seq_len=msl)
    assert bd.decode_mode == "megakernel"
    first = bd.prefill(prompts)
    log = bd.generate(first, steps).cpu()
    torch.cuda.synchronize()
    bd.check_status()
    m = MirrorDecoder(cuda_weights, msl, device="cuda")
    for s in range(SEQS):
        m.reset()
        seq = prompts[s] + [first[s]] + log[:-1, s].tolist()
        ref = m.prefill(seq, 0)[P:]  # logits after the first token and each generated one
        top2 = ref.topk(2, dim=-1).values
        conf = (top2[:, 0] - top2[:, 1]) > TOL_MAX_ABS
        assert torch.equal(ref.argmax(-1)[conf].cpu(), log[:, s].long()[conf.cpu()]), f"sequence {s}"


def test_megakernel_batch_rejects_bad_arguments():
    from qwen_megakernel_b200 import BatchDecoder

    w = small_model(1, seed=5)
    with pytest.raises(ValueError):
        BatchDecoder(w, 3, max_seq_len=64, decode="megakernel")
    bd = BatchDecoder(w, SEQS, max_seq_len=64, decode="megakernel")
    bd.prefill([[1, 2, 3]] * SEQS)
    with pytest.raises(ValueError):
        bd.generate([1, 2, 3, 4], 62)  # past max_seq_len


def test_megakernel_batch_reports_bad_token():
    """An out-of-range first token of one sequence: the launch completes
    (token 0 is used in its place, nothing is read out of bounds) and the
    status block reports QMK_ERR_TOKEN; the next launch on the same
    workspace is clean."""
    from qwen_megakernel_b200 import BatchDecoder, DecodeError

    w = small_model(1, seed=7)
    bd = BatchDecoder(w, SEQS, max_seq_len=64, decode="megakernel")
    first = bd.prefill([[1, 2, 3]] * SEQS)
    bd.generate([first[0], V, first[2], first[3]], 2)
    torch.cuda.synchronize()
    with pytest.raises(DecodeError, match="error 5"):
        bd.check_status()
    bd.generate(first, 2)
    torch.cuda.synchronize()
    bd.check_status()
