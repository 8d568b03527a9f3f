"""Generate the golden fixtures from the reference's own PyTorch path.

The reference checks its kernel against Hugging Face Qwen3ForCausalLM
(qwen_megakernel/bench.py:83-133) and ships no golden vectors, so these
fixtures are produced here from that path (transformers 5.5.0), evaluated in
fp32 on CPU over the seeded bf16 weights of qwen_megakernel_b200.weights:

  config1.npz  BASELINE config 0: 16-token uniform-random prompt (seed 1),
               128 greedy steps, all 28 layers, weights seed 0.
  config2.npz  BASELINE config 1 (shortened): 1024-token prompt (seed 2),
               512 greedy steps.

Each fixture holds, per generated step t: the greedy token, the top-2 gap,
top-8 (index, logit), logits at a fixed seeded sample of vocabulary indices,
summary stats of the full logit vector, full fp16 logits of a few steps, the
torch-fp32 mirror's error against HF on the full vector (teacher-forced on the
HF tokens) and the HF-bf16 path's error (information only).

    python tests/golden/make_golden.py [--config 1|2|all]
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.hf_reference import build_hf_model, hf_greedy  # noqa: E402
from oracle.qwen3_mirror import MirrorDecoder  # noqa: E402
from qwen_megakernel_b200.weights import VOCAB_SIZE, random_weights, weights_checksum  # noqa: E402

CONFIGS = {
    1: dict(prompt_len=16, n_new=128, prompt_seed=1, n_sample=512, full_steps=[0, 1, 63, 127]),
    2: dict(prompt_len=1024, n_new=512, prompt_seed=2, n_sample=256, full_steps=[0, 1, 255, 511]),
}
WEIGHT_SEED = 0
SAMPLE_SEED = 3


def prompt_ids(n: int, seed: int) -> list[int]:
    rng = np.random.Generator(np.random.PCG64(seed))
    return [int(x) for x in rng.integers(0, VOCAB_SIZE, size=n)]


def sample_indices(n: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(SAMPLE_SEED))
    return np.sort(rng.choice(VOCAB_SIZE, size=n, replace=False)).astype(np.int64)


def summarize(logits: torch.Tensor, idx: np.ndarray) -> dict:
    top = torch.topk(logits, 8, dim=-1)
    return dict(
        top_idx=top.indices.numpy().astype(np.int32),
        top_val=top.values.numpy().astype(np.float32),
        gap=(top.values[:, 0] - top.values[:, 1]).numpy().astype(np.float32),
        sample=logits[:, torch.from_numpy(idx)].numpy().astype(np.float32),
        stats=torch.stack(
            [logits.max(-1).values, logits.min(-1).values, logits.mean(-1), logits.norm(dim=-1)], -1
        )
        .numpy()
        .astype(np.float32),
    )


def make(cfg_id: int, weights: dict, out_dir: str) -> None:
    cfg = CONFIGS[cfg_id]
    prompt = prompt_ids(cfg["prompt_len"], cfg["prompt_seed"])
    idx = sample_indices(cfg["n_sample"])
    t0 = time.time()
    hf = build_hf_model(weights, torch.float32)
    toks, logits = hf_greedy(hf, prompt, cfg["n_new"])
    del hf
    t_hf = time.time() - t0
    s = summarize(logits, idx)

    # The mirror (kernel numerics), teacher-forced on the HF tokens.
    t0 = time.time()
    mir = MirrorDecoder(weights, cfg["prompt_len"] + cfg["n_new"] + 1)
    mtoks, mlogits = mir.greedy(prompt, cfg["n_new"], teacher=toks)
    del mir
    t_m = time.time() - t0
    d = (mlogits - logits).abs().max(-1).values
    rel = (mlogits - logits).norm(dim=-1) / logits.norm(dim=-1)

    # The literal reference path in bf16 (information only).
    hb = build_hf_model(weights, torch.bfloat16)
    _, blogits = hf_greedy(hb, prompt, cfg["n_new"], teacher=toks)
    del hb
    bd = (blogits.float() - logits).abs().max(-1).values

    full_steps = np.array(cfg["full_steps"], dtype=np.int32)
    np.savez_compressed(
        os.path.join(out_dir, f"config{cfg_id}.npz"),
        prompt=np.array(prompt, dtype=np.int32),
        tokens=np.array(toks, dtype=np.int32),
        sample_idx=idx.astype(np.int32),
        logits_sample=s["sample"],
        top_idx=s["top_idx"],
        top_val=s["top_val"],
        gap=s["gap"],
        stats=s["stats"],
        full_steps=full_steps,
        full_logits_f16=logits[torch.from_numpy(full_steps).long()].numpy().astype(np.float16),
        mirror_tokens=np.array(mtoks, dtype=np.int32),
        mirror_maxabs=d.numpy().astype(np.float32),
        mirror_rel_l2=rel.numpy().astype(np.float32),
        hf_bf16_maxabs=bd.numpy().astype(np.float32),
        meta=np.array(
            json.dumps(
                dict(
                    config=cfg_id,
                    weight_seed=WEIGHT_SEED,
                    prompt_seed=cfg["prompt_seed"],
                    sample_seed=SAMPLE_SEED,
                    num_layers=28,
                    rope_theta=1e6,
                    weights=weights_checksum(weights),
                    transformers=__import__("transformers").__version__,
                    torch=torch.__version__,
                    numpy=np.__version__,
                    seconds_hf=round(t_hf, 1),
                    seconds_mirror=round(t_m, 1),
                )
            )
        ),
    )
    print(
        f"config{cfg_id}: hf {t_hf:.0f}s mirror {t_m:.0f}s; mirror vs hf max|d| {d.max():.4f} "
        f"relL2 {rel.max():.5f}; hf-bf16 vs hf-fp32 max|d| {bd.max():.4f}; "
        f"min gap {s['gap'].min():.4f}; mirror tokens equal: {mtoks == toks}"
    )


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="all")
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    weights = random_weights(seed=WEIGHT_SEED, device="cpu", max_seq_len=2048)
    ids = [1, 2] if args.config == "all" else [int(args.config)]
    for i in ids:
        make(i, weights, HERE)
    return 0


if __name__ == "__main__":
    sys.exit(main())
