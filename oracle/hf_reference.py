"""The reference's own PyTorch path, built on our seeded weights (test infrastructure).

The reference compares its kernel against Hugging Face
``Qwen3ForCausalLM`` (qwen_megakernel/bench.py:19-55 times it, :83-133 uses it
as the correctness comparator).  That model is a third-party dependency, not
part of the reference project: transformers (pinned only as ``>=4.40.0`` by the
reference's requirements.txt:2; this image has 5.5.0).  Here it is built from
an explicit Qwen3-0.6B config with the same bf16 weights the kernel uses and
evaluated either in fp32 (bf16 weights upcast exactly: the "after fp32
accumulation" parity target) or in bf16 (the literal reference path).

Only tests/, tests/golden/make_golden.py and bench.py's CPU-baseline /
reference legs may use this module.
"""

from __future__ import annotations

import torch

TENSORS_PER_LAYER = 11
_LAYER_NAMES = (
    "input_layernorm.weight",
    "self_attn.q_proj.weight",
    "self_attn.k_proj.weight",
    "self_attn.v_proj.weight",
    "self_attn.q_norm.weight",
    "self_attn.k_norm.weight",
    "self_attn.o_proj.weight",
    "post_attention_layernorm.weight",
    "mlp.gate_proj.weight",
    "mlp.up_proj.weight",
    "mlp.down_proj.weight",
)


def qwen3_config(num_layers: int = 28, rope_theta: float = 1e6):
    from transformers import Qwen3Config

    return Qwen3Config(
        hidden_size=1024,
        intermediate_size=3072,
        num_hidden_layers=num_layers,
        num_attention_heads=16,
        num_key_value_heads=8,
        head_dim=128,
        vocab_size=151936,
        rms_norm_eps=1e-6,
        tie_word_embeddings=True,
        max_position_embeddings=40960,
        rope_parameters={"rope_type": "default", "rope_theta": rope_theta},
        attention_bias=False,
        hidden_act="silu",
    )


def build_hf_model(weights: dict, dtype=torch.float32, num_layers: int | None = None, rope_theta: float = 1e6):
    """Qwen3ForCausalLM (eager attention) holding ``weights`` cast to ``dtype``."""
    from transformers import Qwen3ForCausalLM

    lw = weights["layer_weights"]
    L = num_layers if num_layers is not None else len(lw) // TENSORS_PER_LAYER
    cfg = qwen3_config(L, rope_theta)
    cfg._attn_implementation = "eager"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    sd = {"model.embed_tokens.weight": weights["embed_weight"], "model.norm.weight": weights["final_norm_weight"]}
    for i in range(L):
        for j, name in enumerate(_LAYER_NAMES):
            sd[f"model.layers.{i}.{name}"] = lw[i * TENSORS_PER_LAYER + j]
    sd = {k: v.detach().to("cpu").to(dtype).contiguous() for k, v in sd.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    model.load_state_dict(sd, assign=True, strict=False)
    model.lm_head.weight = model.model.embed_tokens.weight
    # Non-persistent buffers (rotary inv_freq) were created on meta: rebuild them.
    rot = model.model.rotary_emb
    inv_freq, scaling = rot.compute_default_rope_parameters(cfg, device="cpu")
    rot.inv_freq = inv_freq
    rot.original_inv_freq = inv_freq.clone()
    rot.attention_scaling = scaling
    model.eval()
    return model


@torch.no_grad()
def hf_greedy(model, prompt, n_new: int, teacher=None, keep_logits: bool = True):
    """Prefill ``prompt`` in one forward, then n_new greedy decode steps with a
    KV cache.  Returns (tokens, logits [n_new, V] fp32 or None).  With
    ``teacher`` the step after t consumes teacher[t] (teacher forcing)."""
    ids = torch.as_tensor([list(prompt)], dtype=torch.long)
    out = model(input_ids=ids, use_cache=True, logits_to_keep=1)
    logits = out.logits[0, -1].float()
    pkv = out.past_key_values
    toks, outs = [], []
    for t in range(n_new):
        if keep_logits:
            outs.append(logits.clone())
        tok = int(torch.argmax(logits).item())
        toks.append(tok)
        if t + 1 == n_new:
            break
        nxt = teacher[t] if teacher is not None else tok
        out = model(input_ids=torch.tensor([[nxt]]), past_key_values=pkv, use_cache=True)
        logits = out.logits[0, -1].float()
        pkv = out.past_key_values
    return toks, (torch.stack(outs) if keep_logits else None)
