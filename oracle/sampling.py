"""numpy restatement of the kernel's on-device sampling (test infrastructure).

This module is a CHECKER: only tests/ import it; the product never does.

The reference decodes greedily only (csrc/kernel.cu:1020-1183, argmax) and
truncates at EOS on the host (qwen_megakernel/model.py:242-244); sampling is
an extension (on-device sampling).  Its defining semantics are the standard ones:
the next token is a draw from softmax(logits / T).  The kernel draws it with
the Gumbel-max trick (Gumbel 1954; e.g. Maddison, Tarlow and Minka 2014):
argmax_i(logit_i / T + g_i) with i.i.d. standard Gumbel g_i is distributed as
softmax(logits / T); top-k restricts the argmax to the logits >= the k-th
largest (an exact draw from the renormalized top-k softmax).  The noise is a deterministic function of
(seed, cache position, vocabulary index):

    z  = seed XOR (position << 20 | index)
    z  = splitmix64 finalizer of z (Steele, Lea and Flood 2014)
    u  = ((z >> 40) + 0.5) * 2^-24          (fp32, in (0, 1))
    g  = -log(-log(u))

restated here with numpy uint64 arithmetic (wrapping like the kernel's) and
float64 logarithms (the kernel uses fp32 logf: the two agree to ~1e-6).
"""

from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def uniform24(seed: int, position: int, index: np.ndarray) -> np.ndarray:
    """The kernel's u in (0, 1) for the given vocabulary indices (fp32 values)."""
    idx = np.asarray(index, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) ^ ((np.uint64(position) << np.uint64(20)) | idx)
        z = z + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    top = (z >> np.uint64(40)).astype(np.float32)
    return (top + np.float32(0.5)) * np.float32(1.0 / 16777216.0)


def gumbel(seed: int, position: int, index: np.ndarray) -> np.ndarray:
    u = uniform24(seed, position, index).astype(np.float64)
    return -np.log(-np.log(u))


def sample(logits: np.ndarray, temperature: float, seed: int, position: int, top_k: int = 0) -> tuple[int, float]:
    """Token the kernel draws from fp32 logits [vocab] at `position`, and the
    gap between the best and second-best perturbed keys (how robust the
    choice is to the kernel's fp32 rounding of the same keys).  With top_k
    > 0 only logits >= the top_k-th largest take part (ties at the threshold
    included, as in the kernel)."""
    v = logits.shape[-1]
    keys = logits.astype(np.float64) / temperature + gumbel(seed, position, np.arange(v))
    if top_k > 0:
        tau = np.partition(logits, -top_k)[-top_k]
        keys = np.where(logits >= tau, keys, -np.inf)
    top2 = np.partition(keys, -2)[-2:]
    return int(np.argmax(keys)), float(top2[1] - top2[0])
