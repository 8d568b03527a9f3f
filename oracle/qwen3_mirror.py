"""Torch-fp32 restatement of the reference decode step (test infrastructure).

This module is the CHECKER for the CUDA kernel.  Only tests/, the smoke test
and bench.py's CPU-baseline leg may import it; the product never does.

It restates the algorithm of the reference megakernel
(AlpinDale/qwen_megakernel csrc/kernel.cu) with the reference's storage
formats, in plain torch fp32 (CPU or any device):

  embedding row (bf16 -> fp32)                         kernel.cu:1358-1371
  per layer:
    RMSNorm(x) * w_in, eps 1e-6                        kernel.cu:179-231
    q, k, v = W x (fp32 accumulate, bf16 weights)       kernel.cu:234-289
    per-head RMSNorm of q and k (q_norm / k_norm)       kernel.cu:346-412
    RoPE rotate-half with bf16 cos/sin tables           kernel.cu:366-377, model.py:53-60
    K, V appended to the cache as bf16 at `position`    kernel.cu:378-379
    GQA attention (2 q heads per KV head), fp32
      softmax over cache positions [0, position]         kernel.cu:488-585
    o = W_o attn + residual                             kernel.cu:663-707
    RMSNorm * w_post, gate/up, SiLU(gate) * up          kernel.cu:711-819
    x = W_down m + residual                             kernel.cu:823-862
  final RMSNorm * w_final, tied LM head, argmax         kernel.cu:1386-1423, 1020-1183

The residual stream between layers is kept in fp32 (the reference kernel
rounds it to bf16 at kernel.cu:859; the CUDA kernel of this repository keeps
fp32, which is closer to the fp32 evaluation of the HF path).  The same
formulas are the HF Qwen3 modules (transformers 5.5.0, models/qwen3/
modeling_qwen3.py: Qwen3RMSNorm :50-67, Qwen3MLP :70-83, rotate_half /
apply_rotary_pos_emb :151-181, Qwen3Attention :222-291), which is the
reference's own PyTorch comparator (qwen_megakernel/bench.py:19-55, 83-133).

Argmax ties resolve to the lowest index (torch.argmax).
"""

from __future__ import annotations

import math

import torch

HIDDEN = 1024
INTER = 3072
NQ = 16
NKV = 8
HD = 128
VOCAB = 151936
EPS = 1e-6
TENSORS_PER_LAYER = 11


def rms_norm(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) * w over the last dim (fp32)."""
    var = x.pow(2).mean(-1, keepdim=True)
    return (x * torch.rsqrt(var + EPS)) * w


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class MirrorDecoder:
    """Batch-1 decoder state: fp32 copies of the weights and a bf16 KV cache.

    ``step(token, position)`` returns the fp32 logits of one decode step;
    ``prefill(tokens, start)`` runs several positions at once (same math,
    causal attention) and returns the logits of every position.
    """

    def __init__(
        self,
        weights: dict,
        max_seq_len: int,
        device="cpu",
        num_layers: int | None = None,
        kv_dtype=torch.bfloat16,
    ):
        dev = torch.device(device)
        lw = weights["layer_weights"]
        self.num_layers = num_layers if num_layers is not None else len(lw) // TENSORS_PER_LAYER
        f = lambda t: t.to(dev).float()  # noqa: E731
        self.embed = f(weights["embed_weight"])
        self.lm_head = f(weights["lm_head_weight"]) if weights["lm_head_weight"] is not weights["embed_weight"] else self.embed
        self.final_norm = f(weights["final_norm_weight"])
        self.layers = []
        for i in range(self.num_layers):
            t = lw[i * TENSORS_PER_LAYER : (i + 1) * TENSORS_PER_LAYER]
            self.layers.append([f(x) for x in t])
        # The kernel reads bf16 tables; their fp32 values are what it uses.
        self.cos = f(weights["cos_table"])
        self.sin = f(weights["sin_table"])
        self.max_seq_len = max_seq_len
        self.device = dev
        shape = (self.num_layers, NKV, max_seq_len, HD)
        # bf16 is the reference cache format (kernel.cu:378-379); fp32 is for
        # measuring how much of the gap to the fp32 HF path it accounts for.
        self.k_cache = torch.zeros(shape, dtype=kv_dtype, device=dev)
        self.v_cache = torch.zeros(shape, dtype=kv_dtype, device=dev)
        self.scale = 1.0 / math.sqrt(HD)

    def reset(self):
        self.k_cache.zero_()
        self.v_cache.zero_()

    @torch.no_grad()
    def prefill(self, tokens, start: int = 0, return_hidden: bool = False) -> torch.Tensor:
        """Process tokens at positions [start, start + T); returns logits [T, V]."""
        toks = torch.as_tensor(tokens, dtype=torch.long, device=self.device).reshape(-1)
        T = toks.numel()
        pos = torch.arange(start, start + T, device=self.device)
        x = self.embed[toks]  # [T, H] fp32
        cos = self.cos[pos]  # [T, 128]
        sin = self.sin[pos]
        end = start + T
        for li, (w_in, wq, wk, wv, wqn, wkn, wo, w_post, wg, wu, wd) in enumerate(self.layers):
            h = rms_norm(x, w_in)
            q = (h @ wq.T).view(T, NQ, HD)
            k = (h @ wk.T).view(T, NKV, HD)
            v = (h @ wv.T).view(T, NKV, HD)
            q = rms_norm(q, wqn)
            k = rms_norm(k, wkn)
            q = q * cos[:, None, :] + rotate_half(q) * sin[:, None, :]
            k = k * cos[:, None, :] + rotate_half(k) * sin[:, None, :]
            self.k_cache[li, :, start:end] = k.transpose(0, 1).to(self.k_cache.dtype)
            self.v_cache[li, :, start:end] = v.transpose(0, 1).to(self.v_cache.dtype)
            K = self.k_cache[li, :, :end].float()  # [NKV, end, HD]
            V = self.v_cache[li, :, :end].float()
            qg = q.view(T, NKV, NQ // NKV, HD).permute(1, 2, 0, 3)  # [NKV, 2, T, HD]
            s = torch.einsum("gqtd,gpd->gqtp", qg, K) * self.scale
            # causal mask: query at position start+t sees cache positions <= start+t
            mask = torch.arange(end, device=self.device)[None, :] > pos[:, None]  # [T, end]
            s = s.masked_fill(mask[None, None], float("-inf"))
            p = torch.softmax(s, dim=-1)
            o = torch.einsum("gqtp,gpd->gqtd", p, V)  # [NKV, 2, T, HD]
            o = o.permute(2, 0, 1, 3).reshape(T, NQ * HD)
            a = o @ wo.T + x
            h2 = rms_norm(a, w_post)
            m = torch.nn.functional.silu(h2 @ wg.T) * (h2 @ wu.T)
            x = m @ wd.T + a
        xf = rms_norm(x, self.final_norm)
        logits = xf @ self.lm_head.T
        if return_hidden:
            return logits, xf
        return logits

    @torch.no_grad()
    def step(self, token: int, position: int) -> torch.Tensor:
        """One decode step; returns logits [V] (fp32)."""
        return self.prefill([int(token)], start=position)[0]

    @torch.no_grad()
    def greedy(self, prompt, n_new: int, teacher=None):
        """Prompt then n_new greedy steps.  Returns (tokens [n_new], logits [n_new, V]).
        With ``teacher`` (list of n_new tokens), step t+1 consumes teacher[t]
        instead of the argmax of step t (logits stay per-step)."""
        self.reset()
        prompt = list(prompt)
        logits = self.prefill(prompt, 0)[-1]
        toks, outs = [], []
        pos = len(prompt)
        for t in range(n_new):
            outs.append(logits)
            tok = int(torch.argmax(logits).item())
            toks.append(tok)
            if t + 1 == n_new:
                break
            nxt = teacher[t] if teacher is not None else tok
            logits = self.step(nxt, pos)
            pos += 1
        return toks, torch.stack(outs)
