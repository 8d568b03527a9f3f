"""High-level decode API, mirroring the reference's qwen_megakernel/model.py.

Same names and meaning as the reference: ``load_weights``, ``Decoder`` with
``step`` / ``reset`` / ``position`` / ``generate``, and ``generate``
(model.py:21-250).  Differences:
  * ``Decoder`` owns a private workspace, so several decoders can run on
    different streams (the reference shares process-global barrier state,
    csrc/kernel.cu:1446-1473);
  * ``generate`` runs the prompt and the generation in ONE kernel launch (the
    reference calls ``step`` per prompt token, model.py:210-211, then queues
    4 launches per generated token, csrc/kernel.cu:1582-1604);
  * ``max_seq_len`` is a constructor argument (the reference fixes 2048);
  * device-side errors (bounded-wait timeouts, bad token ids) and host-side
    argument errors raise RuntimeError.
Added: ``random_weights``, ``Decoder.step_logits``, ``Decoder.prefill``,
``Decoder.generate_ids`` (tokenizer-free), ``Decoder.decode_steps``.
"""

from __future__ import annotations

import math
import struct

import torch

from . import _native
from .weights import (
    HEAD_DIM,
    HIDDEN_SIZE,
    INTERMEDIATE_SIZE,
    KV_SIZE,
    NUM_KV_HEADS,
    NUM_LAYERS,
    Q_SIZE,
    TENSORS_PER_LAYER,
    VOCAB_SIZE,
    load_hf_weights,
    random_weights,
)

MAX_SEQ_LEN = 2048

__all__ = [
    "load_weights",
    "random_weights",
    "Decoder",
    "generate",
    "DecodeError",
    "NUM_LAYERS",
    "NUM_KV_HEADS",
    "HEAD_DIM",
    "HIDDEN_SIZE",
    "INTERMEDIATE_SIZE",
    "Q_SIZE",
    "KV_SIZE",
    "MAX_SEQ_LEN",
    "VOCAB_SIZE",
]

_ERROR_NAMES = {
    0: "ok",
    1: "invalid argument",
    2: "CUDA runtime error",
    3: "cooperative launch refused",
    4: "device-side wait timed out",
    5: "token id out of range",
    6: "workspace too small or misaligned",
}


class DecodeError(RuntimeError):
    """A device-side error reported by the kernel's status block."""


def load_weights(model_name="Qwen/Qwen3-0.6B", verbose: bool = True, max_seq_len: int = MAX_SEQ_LEN):
    """Load Qwen3-0.6B weights from a local Hugging Face checkpoint.

    Reference: qwen_megakernel/model.py:21-94 (which downloads from the hub;
    here the checkpoint must be on disk)."""
    return load_hf_weights(model_name, device="cuda", max_seq_len=max_seq_len, verbose=verbose)


def _pack_layer_weights(layer_weights: list[torch.Tensor], device) -> torch.Tensor:
    """Pack the 11-pointer-per-layer table (LDGLayerWeights[num_layers]) into a
    device byte tensor.  Reference: model.py:97-108."""
    n_layers = len(layer_weights) // TENSORS_PER_LAYER
    buf = bytearray(n_layers * TENSORS_PER_LAYER * 8)
    for i, t in enumerate(layer_weights[: n_layers * TENSORS_PER_LAYER]):
        struct.pack_into("Q", buf, i * 8, t.data_ptr())
    return torch.frombuffer(buf, dtype=torch.uint8).to(device)


class Decoder:
    """Stateful batch-1 decoder over the persistent sm_100a kernel."""

    def __init__(
        self,
        weights=None,
        tokenizer=None,
        model_name="Qwen/Qwen3-0.6B",
        verbose: bool = True,
        max_seq_len: int | None = None,
        timeout_ns: int = 0,
    ):
        if weights is None:
            weights, tokenizer = load_weights(model_name, verbose=verbose)
        self._ops = _native.ops()
        self.tokenizer = tokenizer
        self._position = 0
        self._weights = weights  # keeps the tensors behind the packed pointers alive
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm_head_weight = weights["lm_head_weight"]
        self._cos_table = weights["cos_table"]
        self._sin_table = weights["sin_table"]
        self.device = self._embed_weight.device
        if self.device.type != "cuda":
            raise RuntimeError("Decoder needs CUDA weights (there is no CPU path)")
        layer_weights = weights["layer_weights"]
        if len(layer_weights) % TENSORS_PER_LAYER:
            raise ValueError("layer_weights must hold 11 tensors per layer")
        self.num_layers = len(layer_weights) // TENSORS_PER_LAYER
        self._layer_weights_packed = _pack_layer_weights(layer_weights, self.device)
        self.max_seq_len = int(max_seq_len or self._cos_table.shape[0])
        if self._cos_table.shape[0] < self.max_seq_len:
            raise ValueError(
                f"RoPE tables have {self._cos_table.shape[0]} rows < max_seq_len {self.max_seq_len}"
            )
        self._attn_scale = 1.0 / math.sqrt(HEAD_DIM)
        self._timeout_ns = int(timeout_ns)
        self.poll_backoff_ns = 0  # tuning knob of the dataflow polls (ns, 0 = spin)
        self.tuning = 0  # QmkRunArgs.tuning flags

        kv_shape = (self.num_layers, NUM_KV_HEADS, self.max_seq_len, HEAD_DIM)
        self._k_cache = torch.zeros(kv_shape, dtype=torch.bfloat16, device=self.device)
        self._v_cache = torch.zeros_like(self._k_cache)
        self._workspace = torch.zeros(self._ops.workspace_bytes(), dtype=torch.uint8, device=self.device)
        self._status = torch.zeros(4, dtype=torch.int32).pin_memory()
        self._out_token = torch.empty(1, dtype=torch.int32, device=self.device)
        self._steps_done = torch.zeros(1, dtype=torch.int32, device=self.device)

    # ------------------------------------------------------------------ core
    @property
    def k_cache(self) -> torch.Tensor:
        return self._k_cache

    @property
    def v_cache(self) -> torch.Tensor:
        return self._v_cache

    @property
    def position(self) -> int:
        return self._position

    @position.setter
    def position(self, value: int) -> None:
        if not 0 <= value <= self.max_seq_len:
            raise ValueError(f"position {value} outside [0, {self.max_seq_len}]")
        self._position = int(value)

    def reset(self):
        self._position = 0
        self._k_cache.zero_()
        self._v_cache.zero_()

    def check_status(self) -> None:
        """Raise DecodeError if the last completed launch reported an error
        (call after the stream has been synchronized)."""
        code = int(self._status[0])
        if code != 0:
            info = int(self._status[1]) & 0xFFFFFFFF
            raise DecodeError(
                f"qwen_megakernel device error {code} ({_ERROR_NAMES.get(code, '?')}): "
                f"cta {info >> 16}, site {(info >> 8) & 0xFF}, layer {info & 0xFF}"
            )

    def decode_steps(
        self,
        num_steps: int,
        first_token: int = 0,
        forced_tokens: torch.Tensor | None = None,
        start_position: int | None = None,
        output_log: torch.Tensor | None = None,
        output_token: torch.Tensor | None = None,
        logits: torch.Tensor | None = None,
        final_hidden: torch.Tensor | None = None,
        debug_stall: int = 0,
        trace: torch.Tensor | None = None,
        trace_step: int = 0,
        poll_backoff_ns: int | None = None,
        tuning: int | None = None,
        temperature: float = 0.0,
        seed: int = 0,
        eos_token: int | None = None,
        steps_done: torch.Tensor | None = None,
        top_k: int = 0,
    ) -> None:
        """Queue one launch of ``num_steps`` decode steps (no host sync).

        Step t consumes ``forced_tokens[t]`` while t < len(forced_tokens),
        else ``first_token`` (t == 0) or the previous step's argmax, at
        position ``start_position + t``; it writes its argmax to
        ``output_log[t]`` and its fp32 logits to ``logits[t]`` if given.
        ``temperature`` > 0 samples instead of taking the argmax (Gumbel-max,
        reproducible per (seed, position)), among the ``top_k`` largest logits
        if ``top_k`` > 0; with ``eos_token`` the launch ends
        after the first generated token equal to it, and ``steps_done``
        (device int32 [1]) receives the number of steps run."""
        start = self._position if start_position is None else int(start_position)
        if start < 0 or start + num_steps > self.max_seq_len:
            raise ValueError(f"positions [{start}, {start + num_steps}) exceed max_seq_len {self.max_seq_len}")
        if forced_tokens is not None and forced_tokens.dtype != torch.int32:
            forced_tokens = forced_tokens.to(torch.int32)
        self._ops.run(
            self._workspace,
            self._embed_weight,
            self._layer_weights_packed,
            self._final_norm_weight,
            self._lm_head_weight,
            self._cos_table,
            self._sin_table,
            self._k_cache,
            self._v_cache,
            forced_tokens,
            int(first_token),
            start,
            int(num_steps),
            self.num_layers,
            self.max_seq_len,
            self._attn_scale,
            output_log,
            output_token,
            logits,
            final_hidden,
            self._status,
            self._timeout_ns,
            int(debug_stall),
            trace,
            int(trace_step),
            int(self.poll_backoff_ns if poll_backoff_ns is None else poll_backoff_ns),
            int(self.tuning if tuning is None else tuning),
            float(temperature),
            int(seed),
            0 if eos_token is None else 1,
            0 if eos_token is None else int(eos_token),
            steps_done,
            int(top_k),
        )

    # ------------------------------------------------------- reference API
    def step(self, token_id: int) -> int:
        """Decode one token. Returns the next token id (reference model.py:166-196)."""
        self.decode_steps(1, first_token=token_id, output_token=self._out_token)
        tok = int(self._out_token.item())
        self.check_status()
        self._position += 1
        return tok

    def generate(self, prompt: str, max_tokens: int = 100) -> str:
        """Reference model.py:207-245: reset, prompt, greedy generation, EOS
        truncation, detokenize."""
        if self.tokenizer is None:
            raise RuntimeError("generate(prompt) needs a tokenizer; use generate_ids for token ids")
        ids = self.tokenizer.encode(prompt, add_special_tokens=True)
        eos = self.tokenizer.eos_token_id
        # the kernel stops at EOS (the reference generates max_tokens and
        # truncates on the host, model.py:242-244: same text)
        out = self.generate_ids(ids, max_tokens, eos_token=eos)
        if eos in out:
            out = out[: out.index(eos)]
        return self.tokenizer.decode(out, skip_special_tokens=True)

    # ------------------------------------------------------------ additions
    def step_logits(self, token_id: int) -> tuple[int, torch.Tensor]:
        """Like step(), also returning the fp32 logits [151936]."""
        logits = torch.empty(VOCAB_SIZE, dtype=torch.float32, device=self.device)
        self.decode_steps(1, first_token=token_id, output_token=self._out_token, logits=logits)
        tok = int(self._out_token.item())
        self.check_status()
        self._position += 1
        return tok, logits

    def prefill(self, token_ids, logits: torch.Tensor | None = None) -> int:
        """Consume ``token_ids`` at positions [position, position + n) in one
        launch (sequential decode, as the reference's per-token prompt loop);
        returns the argmax after the last token."""
        ids = torch.as_tensor(list(token_ids), dtype=torch.int32).to(self.device)
        n = int(ids.numel())
        if n == 0:
            raise ValueError("prefill needs at least one token")
        self.decode_steps(n, forced_tokens=ids, output_token=self._out_token, logits=logits)
        tok = int(self._out_token.item())
        self.check_status()
        self._position += n
        return tok

    def prefill_batched(self, token_ids, logits: torch.Tensor | None = None) -> int:
        """Like prefill(), but token-parallel: the prompt runs as rows of one
        causal forward pass (tensor-core GEMMs over all tokens at once,
        ``qmk_batch_forward``) instead of one decode step per token.  Same
        cache contents and logits within the parity tolerance; returns the
        argmax after the last token (its fp32 logits into ``logits`` [vocab]
        if given)."""
        from .batch import MAX_ROWS, BatchForward, _int32

        ids = [int(t) for t in token_ids]
        n = len(ids)
        if n == 0:
            raise ValueError("prefill needs at least one token")
        start = self._position
        if start + n > self.max_seq_len:
            raise ValueError(f"positions [{start}, {start + n}) exceed max_seq_len {self.max_seq_len}")
        if getattr(self, "_batch_fw", None) is None:
            self._batch_fw = BatchForward(self._weights, self.max_seq_len)
        fw = self._batch_fw
        for c0 in range(0, n, MAX_ROWS):
            c1 = min(n, c0 + MAX_ROWS)
            last = c1 == n
            tokens = _int32(ids[c0:c1], self.device)
            row_pos = torch.arange(start + c0, start + c1, dtype=torch.int32, device=self.device)
            row_seq = torch.zeros(c1 - c0, dtype=torch.int32, device=self.device)
            out_rows = torch.full((1,), c1 - c0 - 1, dtype=torch.int32, device=self.device) if last else None
            fw.forward(self._k_cache, self._v_cache, 1, tokens, row_seq, row_pos, out_rows,
                       self._out_token if last else None, logits if last else None,
                       causal_run=(start + c0 == 0))
        tok = int(self._out_token.item())
        fw.check_status()
        self._position += n
        return tok

    def generate_from(self, token_id: int, max_tokens: int, position: int | None = None,
                      temperature: float = 0.0, seed: int = 0, eos_token: int | None = None,
                      top_k: int = 0) -> list[int]:
        """Continuation from the current KV cache: consume ``token_id`` at
        ``position`` (default: the decoder's position) and return ``max_tokens``
        generated ids -- the semantics of the reference's ``generate_nosync``
        operator (csrc/torch_bindings.cpp:93-127), with host ids in and out.
        Additions: ``temperature`` > 0 samples on the device; with
        ``eos_token`` the launch stops after generating it (the returned list
        ends with it and may be shorter)."""
        pos = self._position if position is None else int(position)
        n = int(max_tokens)
        host_tok = torch.tensor([int(token_id)], dtype=torch.int32).pin_memory()
        dev_tok = host_tok.to(self.device, non_blocking=True)
        log = torch.empty(n, dtype=torch.int32, device=self.device)
        done = self._steps_done
        self.decode_steps(n, forced_tokens=dev_tok, start_position=pos, output_log=log, temperature=temperature,
                          seed=seed, eos_token=eos_token, steps_done=done, top_k=top_k)
        host = torch.empty(n + 1, dtype=torch.int32).pin_memory()
        host[:n].copy_(log, non_blocking=True)
        host[n:].copy_(done, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.check_status()
        ran = int(host[n])
        self._position = pos + ran
        return host[:ran].tolist()

    def generate_ids(self, prompt_ids, max_tokens: int = 100, reset: bool = True, temperature: float = 0.0,
                     seed: int = 0, eos_token: int | None = None, top_k: int = 0) -> list[int]:
        """Token-id version of generate(): one launch runs the prompt (forced
        tokens) and ``max_tokens`` greedy (or, with ``temperature`` > 0,
        sampled) steps with on-device feedback, stopping after ``eos_token``
        if given."""
        if reset:
            self.reset()
        ids = [int(t) for t in prompt_ids]
        if not ids:
            raise ValueError("prompt must hold at least one token")
        n_steps = len(ids) - 1 + int(max_tokens)
        forced = torch.tensor(ids, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
        log = torch.empty(n_steps, dtype=torch.int32, device=self.device)
        self.decode_steps(n_steps, forced_tokens=forced, output_log=log, temperature=temperature, seed=seed,
                          eos_token=eos_token, steps_done=self._steps_done, top_k=top_k)
        ran = int(self._steps_done.item())
        out = log[len(ids) - 1 : ran].cpu().tolist()
        self.check_status()
        self._position += ran
        return out


def generate(prompt: str, max_tokens: int = 100, verbose: bool = True) -> str:
    """One-shot convenience: load model, generate, return text (model.py:248-250)."""
    return Decoder(verbose=verbose).generate(prompt, max_tokens)
