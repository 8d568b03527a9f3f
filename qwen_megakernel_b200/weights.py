"""Weights in the reference's layout: seeded synthetic Qwen3-0.6B weights,
RoPE tables, and a local Hugging Face checkpoint loader.

The returned dict has the keys of the reference's ``load_weights``
(qwen_megakernel/model.py:83-90): ``embed_weight``, ``layer_weights`` (11
tensors per layer in the order of model.py:64-80), ``final_norm_weight``,
``lm_head_weight`` (tied to the embedding), ``cos_table``, ``sin_table``.
All weights are bf16 row-major ``[out, in]``; the tables are bf16
``[max_seq_len, 128]`` with the rotate-half halves duplicated
(model.py:53-60).  The RoPE base defaults to Qwen3's 1e6 (the reference
hard-codes 1e4 at model.py:55).
"""

from __future__ import annotations

import numpy as np
import torch

HIDDEN_SIZE = 1024
INTERMEDIATE_SIZE = 3072
NUM_LAYERS = 28
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
Q_SIZE = NUM_Q_HEADS * HEAD_DIM
KV_SIZE = NUM_KV_HEADS * HEAD_DIM
VOCAB_SIZE = 151936
RMS_EPS = 1e-6
ROPE_THETA = 1e6

# (HF state-dict suffix, shape, kind) in the reference's per-layer order
# (qwen_megakernel/model.py:64-80; csrc/kernel.cu:76-88).
LAYER_TENSORS = (
    ("input_layernorm.weight", (HIDDEN_SIZE,), "norm"),
    ("self_attn.q_proj.weight", (Q_SIZE, HIDDEN_SIZE), "linear"),
    ("self_attn.k_proj.weight", (KV_SIZE, HIDDEN_SIZE), "linear"),
    ("self_attn.v_proj.weight", (KV_SIZE, HIDDEN_SIZE), "linear"),
    ("self_attn.q_norm.weight", (HEAD_DIM,), "norm"),
    ("self_attn.k_norm.weight", (HEAD_DIM,), "norm"),
    ("self_attn.o_proj.weight", (HIDDEN_SIZE, Q_SIZE), "linear"),
    ("post_attention_layernorm.weight", (HIDDEN_SIZE,), "norm"),
    ("mlp.gate_proj.weight", (INTERMEDIATE_SIZE, HIDDEN_SIZE), "linear"),
    ("mlp.up_proj.weight", (INTERMEDIATE_SIZE, HIDDEN_SIZE), "linear"),
    ("mlp.down_proj.weight", (HIDDEN_SIZE, INTERMEDIATE_SIZE), "linear"),
)
TENSORS_PER_LAYER = len(LAYER_TENSORS)


def rope_tables(max_seq_len: int, theta: float = ROPE_THETA, device="cpu", dtype=torch.bfloat16):
    """cos/sin tables [max_seq_len, 128], computed in fp32 exactly as the HF
    Qwen3 rotary embedding does, then cast to ``dtype`` (bf16 is the
    reference's table format, model.py:59-60)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.int64).float() / HEAD_DIM))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos().to(dtype).contiguous().to(device)
    sin = emb.sin().to(dtype).contiguous().to(device)
    return cos, sin


def _normal_bf16(rng: np.random.Generator, shape, std: float) -> torch.Tensor:
    n = int(np.prod(shape))
    a = rng.standard_normal(size=n, dtype=np.float32)
    t = torch.from_numpy(a).view(*shape)
    t.mul_(std)
    return t.to(torch.bfloat16)


def random_weights(
    seed: int = 0,
    device="cuda",
    max_seq_len: int = 2048,
    num_layers: int = NUM_LAYERS,
    std: float = 0.02,
    norm_std: float = 0.0,
    rope_theta: float = ROPE_THETA,
) -> dict:
    """Seeded synthetic Qwen3-0.6B weights (bf16).

    Linear and embedding weights ~ N(0, std); norm weights are 1.0, or
    1 + N(0, norm_std) when ``norm_std > 0`` (tests use that to exercise the
    norm-weight paths).  Values come from numpy's PCG64 stream in a fixed
    order (embedding, then each layer's tensors in reference order, then the
    final norm), so they are identical on every machine with the same numpy.
    """
    rng = np.random.Generator(np.random.PCG64(seed))

    def norm(shape):
        if norm_std > 0:
            t = torch.from_numpy(rng.standard_normal(size=shape, dtype=np.float32))
            return (1.0 + norm_std * t).to(torch.bfloat16)
        return torch.ones(shape, dtype=torch.bfloat16)

    embed = _normal_bf16(rng, (VOCAB_SIZE, HIDDEN_SIZE), std).to(device)
    layers = []
    for _ in range(num_layers):
        for _name, shape, kind in LAYER_TENSORS:
            t = _normal_bf16(rng, shape, std) if kind == "linear" else norm(shape)
            layers.append(t.to(device).contiguous())
    final_norm = norm((HIDDEN_SIZE,)).to(device)
    cos, sin = rope_tables(max_seq_len, rope_theta, device=device)
    return dict(
        embed_weight=embed,
        layer_weights=layers,
        final_norm_weight=final_norm,
        lm_head_weight=embed,
        cos_table=cos,
        sin_table=sin,
    )


def weights_checksum(weights: dict) -> dict:
    """Cheap fingerprint of a weight dict (detects RNG drift between machines)."""
    e = weights["embed_weight"]
    out = {
        "embed_sum": float(e[:4096].float().sum().item()),
        "embed_first": [float(x) for x in e[0, :8].float().tolist()],
    }
    lw = weights["layer_weights"]
    if lw:
        q = lw[1]
        out["q0_sum"] = float(q[:64].float().sum().item())
        d = lw[-1]
        out["down_last_sum"] = float(d[:64].float().sum().item())
    return out


def load_hf_weights(model_name_or_path: str, device="cuda", max_seq_len: int = 2048, verbose: bool = True,
                    tokenizer: bool = True):
    """Load a local Qwen3-0.6B Hugging Face checkpoint into the reference's
    weight dict (mirrors qwen_megakernel/model.py:21-94, minus the network:
    the path must already be on disk).  Returns (weights, tokenizer).

    The RoPE base is read from the checkpoint's config (Qwen3: 1e6).  An
    untied ``lm_head.weight`` is used when the config does not tie it to the
    embedding (Qwen3-0.6B ties them).  With ``tokenizer=False`` the returned
    tokenizer is None: the token-id APIs need none."""
    from transformers import AutoModelForCausalLM, AutoTokenizer

    if verbose:
        print(f"Loading {model_name_or_path}...")
    model = AutoModelForCausalLM.from_pretrained(model_name_or_path, dtype=torch.bfloat16)
    tok = AutoTokenizer.from_pretrained(model_name_or_path) if tokenizer else None
    cfg = model.config
    rope = getattr(cfg, "rope_parameters", None) or {}
    theta = float(rope.get("rope_theta", getattr(cfg, "rope_theta", ROPE_THETA)))
    state = model.state_dict()
    layers = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        for name, _shape, _kind in LAYER_TENSORS:
            layers.append(state[p + name].to(device).contiguous())
    embed = state["model.embed_tokens.weight"].to(device).contiguous()
    lm_head = embed
    head = state.get("lm_head.weight")
    if head is not None and not getattr(cfg, "tie_word_embeddings", True):
        lm_head = head.to(device).contiguous()
    cos, sin = rope_tables(max_seq_len, theta, device=device)
    weights = dict(
        embed_weight=embed,
        layer_weights=layers,
        final_norm_weight=state["model.norm.weight"].to(device).contiguous(),
        lm_head_weight=lm_head,
        cos_table=cos,
        sin_table=sin,
    )
    del model
    return weights, tok
