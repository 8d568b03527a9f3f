"""load_hf_weights on a checkpoint written here (CPU, no network).

The reference loads Qwen3-0.6B from the hub (qwen_megakernel/model.py:21-94);
the loader here reads a local checkpoint.  A random 2-layer Qwen3 with the
0.6B dimensions is saved with ``save_pretrained`` and read back: the per-layer
tensor order must be the reference's (model.py:64-80), every value must be
the state dict's, the LM head must be tied to the embedding, and the RoPE
tables must use the checkpoint's rope_theta.
"""

import json
import os

import pytest
import torch

from oracle.hf_reference import qwen3_config
from qwen_megakernel_b200.weights import LAYER_TENSORS, load_hf_weights, rope_tables


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    """A random 2-layer Qwen3 (0.6B dimensions, rope_theta 1e6) saved once."""
    from transformers import Qwen3ForCausalLM

    torch.manual_seed(0)
    model = Qwen3ForCausalLM(qwen3_config(num_layers=2, rope_theta=1e6)).to(torch.bfloat16)
    with torch.no_grad():  # distinct norm weights so a swapped order shows
        for i, layer in enumerate(model.model.layers):
            layer.input_layernorm.weight.fill_(1.0 + 0.01 * i)
            layer.post_attention_layernorm.weight.fill_(1.5 + 0.01 * i)
            layer.self_attn.q_norm.weight.fill_(2.0 + 0.01 * i)
            layer.self_attn.k_norm.weight.fill_(2.5 + 0.01 * i)
    path = tmp_path_factory.mktemp("qwen3_2l")
    model.save_pretrained(path)
    return path, model.state_dict()


def test_loader_round_trip_order_values_and_rope(checkpoint):
    path, state = checkpoint
    w, tok = load_hf_weights(str(path), device="cpu", max_seq_len=64, verbose=False, tokenizer=False)
    assert tok is None
    lw = w["layer_weights"]
    assert len(lw) == 2 * len(LAYER_TENSORS)
    for i in range(2):
        for j, (name, shape, _kind) in enumerate(LAYER_TENSORS):
            t = lw[i * len(LAYER_TENSORS) + j]
            ref = state[f"model.layers.{i}.{name}"]
            assert tuple(t.shape) == shape, name
            assert t.dtype == torch.bfloat16 and t.is_contiguous()
            assert torch.equal(t, ref), f"layer {i} {name}"
    assert torch.equal(w["embed_weight"], state["model.embed_tokens.weight"])
    assert torch.equal(w["final_norm_weight"], state["model.norm.weight"])
    assert w["lm_head_weight"] is w["embed_weight"]  # tied, as Qwen3-0.6B
    cos, sin = rope_tables(64, 1e6)
    assert torch.equal(w["cos_table"], cos) and torch.equal(w["sin_table"], sin)


def test_loader_reads_rope_theta_from_config(checkpoint, tmp_path):
    """The same weights under a config with rope_theta 1e4 (the reference's
    hard-coded base, model.py:55) give that base's tables."""
    path, _ = checkpoint
    cfg = json.loads((path / "config.json").read_text())
    cfg["rope_parameters"] = {"rope_type": "default", "rope_theta": 1e4}
    cfg.pop("rope_theta", None)
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    for f in path.iterdir():
        if f.name != "config.json":
            os.symlink(f, tmp_path / f.name)
    w, _ = load_hf_weights(str(tmp_path), device="cpu", max_seq_len=32, verbose=False, tokenizer=False)
    cos, sin = rope_tables(32, 1e4)
    assert torch.equal(w["cos_table"], cos) and torch.equal(w["sin_table"], sin)
    assert not torch.equal(w["cos_table"], rope_tables(32, 1e6)[0])
