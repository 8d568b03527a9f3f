"""Token-parallel path: batched prompt prefill and batched decode.

Host side of ``qmk_batch_forward`` (``include/qwen_megakernel.h``): one call
runs the model over many rows at once (row = token of a sequence at a
position).  No counterpart in the reference, which feeds a prompt through one
decode step per token (qwen_megakernel/model.py:210-211) and decodes a single
sequence; these are the "batched prefill" and "batch > 1" extensions of its
``Decoder``.

* ``BatchForward``      owns the per-model arguments (pointer table, workspace)
* ``Decoder.prefill_batched`` (model.py) uses it for a prompt
* ``BatchDecoder``      B independent sequences, one row each per step; the
                        step is captured in a CUDA graph (device-side token
                        feedback, no host round trip per step).  With B =
                        MEGAKERNEL_SEQS its decode steps run instead in the
                        persistent decode kernel (``qmk_run_batch``): one
                        launch for all steps, every weight tile streamed
                        once per step for all sequences.
"""

from __future__ import annotations

import math

import torch

from . import _native
from .weights import HEAD_DIM, NUM_KV_HEADS, TENSORS_PER_LAYER, VOCAB_SIZE

MAX_ROWS = 4096  # QMK_BATCH_MAX_ROWS
BAD_TOKEN = 1  # QMK_BATCH_BAD_TOKEN
BAD_ROW = 2  # QMK_BATCH_BAD_ROW
TIMEOUT = 4  # QMK_BATCH_TIMEOUT
COPIES_PENDING = 8  # QMK_BATCH_COPIES_PENDING
MEGAKERNEL_SEQS = 4  # QMK_BATCH_SEQS: sequences of the persistent kernel's batched instance


class BatchError(RuntimeError):
    pass


class BatchForward:
    """Arguments of ``qmk_batch_forward`` that belong to one model."""

    def __init__(self, weights, max_seq_len: int, fuse: bool = True):
        self._ops = _native.ops()
        self._weights = weights  # keeps the tensors behind the raw pointers alive
        lw = weights["layer_weights"]
        if len(lw) % TENSORS_PER_LAYER:
            raise ValueError("layer_weights must hold 11 tensors per layer")
        self.num_layers = len(lw) // TENSORS_PER_LAYER
        self.layer_ptrs = [int(t.data_ptr()) for t in lw]
        # One GEMM for q|k|v and one for gate|up: concatenated copies of the
        # reference-layout matrices (bf16 [4096, 1024] and [6144, 1024] per
        # layer, 20 MB each; the originals stay the source of truth).
        self._fused = []
        if fuse:
            for layer in range(self.num_layers):
                t = lw[layer * TENSORS_PER_LAYER:(layer + 1) * TENSORS_PER_LAYER]
                self._fused.append(torch.cat([t[1], t[2], t[3]], 0).contiguous())
                self._fused.append(torch.cat([t[8], t[9]], 0).contiguous())
        self.fused_ptrs = [int(t.data_ptr()) for t in self._fused]
        self.embed = weights["embed_weight"]
        self.final_norm = weights["final_norm_weight"]
        self.lm_head = weights["lm_head_weight"]
        self.cos = weights["cos_table"]
        self.sin = weights["sin_table"]
        self.device = self.embed.device
        self.max_seq_len = int(max_seq_len)
        if self.cos.shape[0] < self.max_seq_len:
            raise ValueError(f"RoPE tables have {self.cos.shape[0]} rows < max_seq_len {self.max_seq_len}")
        self.attn_scale = 1.0 / math.sqrt(HEAD_DIM)
        self._ws = torch.empty(0, dtype=torch.uint8, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def workspace(self, rows: int, out: int) -> torch.Tensor:
        need = int(self._ops.batch_workspace_bytes(rows, out))
        if self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def cache_shape(self) -> tuple[int, int, int, int]:
        return (self.num_layers, NUM_KV_HEADS, self.max_seq_len, HEAD_DIM)

    def forward(self, k_cache, v_cache, num_seqs, tokens, row_seq, row_pos, out_rows=None, out_tokens=None,
                logits=None, workspace=None, causal_run: bool = False) -> None:
        """Queue one forward pass (no host sync).  Caches: [num_seqs, L, 8, S, 128]
        or, for one sequence, [L, 8, S, 128].  ``causal_run``: the caller
        guarantees row r is position r of sequence 0 (a fresh prompt), which
        lets the attention run as tensor-core GEMMs."""
        rows = int(tokens.numel())
        out = 0 if out_rows is None else int(out_rows.numel())
        ws = self.workspace(rows, out) if workspace is None else workspace
        stride = 0 if num_seqs == 1 else int(math.prod(self.cache_shape()))
        self._ops.batch_forward(
            ws, self.embed, self.layer_ptrs, self.fused_ptrs, self.final_norm, self.lm_head, self.cos, self.sin, k_cache, v_cache,
            stride, int(num_seqs), self.num_layers, self.max_seq_len, self.attn_scale, tokens, row_seq, row_pos,
            out_rows, out_tokens, logits, self.status, 1 if causal_run else 0)

    def check_status(self) -> None:
        """Raise BatchError if a device-side check fired (after a sync)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            what = []
            if code & BAD_TOKEN:
                what.append("token id outside the vocabulary (token 0 used)")
            if code & BAD_ROW:
                what.append("row with a sequence or position out of range (skipped)")
            if code & TIMEOUT:
                what.append("attention K/V copy did not complete within 1 s (outputs invalid)")
            if code & COPIES_PENDING:
                what.append("K/V copies still in flight after the drain limit (context suspect: recreate it)")
            raise BatchError("qmk_batch_forward: " + "; ".join(what))


def _int32(values, device) -> torch.Tensor:
    return torch.tensor([int(v) for v in values], dtype=torch.int32).pin_memory().to(device, non_blocking=True)


class BatchDecoder:
    """``batch_size`` independent greedy sequences decoded together.

    Each sequence has its own KV cache (``k_cache[s]``, the reference layout
    [L, 8, max_seq_len, 128]) and position.  ``prefill`` runs prompts as
    token-parallel rows (all sequences' prompts in one pass), ``step`` one
    row per sequence."""

    def __init__(self, weights, batch_size: int, max_seq_len: int | None = None, use_graphs: bool = True,
                 decode: str = "auto"):
        """decode: "token_parallel" (one row per sequence through the
        token-parallel kernels), "megakernel" (the persistent decode kernel's
        batched instance, B == MEGAKERNEL_SEQS only) or "auto" (the persistent
        kernel when B == MEGAKERNEL_SEQS)."""
        if batch_size < 1 or batch_size > MAX_ROWS:
            raise ValueError(f"batch_size must be in [1, {MAX_ROWS}]")
        if decode not in ("auto", "token_parallel", "megakernel"):
            raise ValueError("decode must be 'auto', 'token_parallel' or 'megakernel'")
        if decode == "megakernel" and batch_size != MEGAKERNEL_SEQS:
            raise ValueError(f"the persistent kernel decodes exactly {MEGAKERNEL_SEQS} sequences")
        self.B = int(batch_size)
        self.fw = BatchForward(weights, int(max_seq_len or weights["cos_table"].shape[0]))
        self.device = self.fw.device
        self.max_seq_len = self.fw.max_seq_len
        shape = (self.B,) + self.fw.cache_shape()
        self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.positions = [0] * self.B
        self.use_graphs = bool(use_graphs)
        # Static step inputs/outputs (graph-captured addresses).
        self._tok = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self._pos = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self._seq = torch.arange(self.B, dtype=torch.int32, device=self.device)
        self._out = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self._ws_step = torch.empty(int(self.fw._ops.batch_workspace_bytes(self.B, self.B)), dtype=torch.uint8,
                                    device=self.device)
        self._graph = None
        self.decode_mode = "megakernel" if (decode == "megakernel" or (decode == "auto" and self.B == MEGAKERNEL_SEQS)) \
            else "token_parallel"
        if self.decode_mode == "megakernel":
            from .model import _pack_layer_weights

            self._mk_layers = _pack_layer_weights(weights["layer_weights"], self.device)
            self._mk_ws = torch.zeros(int(self.fw._ops.workspace_bytes()), dtype=torch.uint8, device=self.device)
            self._mk_status = torch.zeros(4, dtype=torch.int32).pin_memory()
            self._mk_first = torch.zeros(self.B, dtype=torch.int32, device=self.device)

    def check_status(self) -> None:
        """Raise if the last completed step (token-parallel) or launch
        (persistent kernel) reported a device error; call after a stream
        synchronize."""
        self.fw.check_status()
        if self.decode_mode == "megakernel":
            from .model import _ERROR_NAMES, DecodeError

            code = int(self._mk_status[0])
            if code != 0:
                info = int(self._mk_status[1]) & 0xFFFFFFFF
                raise DecodeError(f"qwen_megakernel device error {code} ({_ERROR_NAMES.get(code, '?')}): "
                                  f"cta {info >> 16}, site {(info >> 8) & 0xFF}, layer {info & 0xFF}")

    def reset(self) -> None:
        self.k_cache.zero_()
        self.v_cache.zero_()
        self.positions = [0] * self.B

    def prefill(self, prompts: list[list[int]], logits: torch.Tensor | None = None) -> list[int]:
        """Consume prompts[s] for every sequence s at its current position
        (token-parallel, causal); returns the greedy token after each prompt."""
        if len(prompts) != self.B or any(len(p) == 0 for p in prompts):
            raise ValueError(f"need {self.B} non-empty prompts")
        for s, p in enumerate(prompts):
            if self.positions[s] + len(p) > self.max_seq_len:
                raise ValueError(f"sequence {s}: prompt exceeds max_seq_len {self.max_seq_len}")
        # Rows in chunks of <= MAX_ROWS; a sequence's last prompt row is an output row.
        rows = [(s, self.positions[s] + i, int(t)) for s, p in enumerate(prompts) for i, t in enumerate(p)]
        last_row = {}
        idx = 0
        for s, p in enumerate(prompts):
            idx += len(p)
            last_row[idx - 1] = s
        next_tok = [0] * self.B
        for c0 in range(0, len(rows), MAX_ROWS):
            chunk = rows[c0:c0 + MAX_ROWS]
            outs = [(i - c0, s) for i, s in sorted(last_row.items()) if c0 <= i < c0 + len(chunk)]
            tokens = _int32([r[2] for r in chunk], self.device)
            row_seq = _int32([r[0] for r in chunk], self.device)
            row_pos = _int32([r[1] for r in chunk], self.device)
            out_rows = _int32([o[0] for o in outs], self.device) if outs else None
            out_tok = torch.empty(len(outs), dtype=torch.int32, device=self.device) if outs else None
            lg = None
            if logits is not None and outs:
                lg = torch.empty(len(outs), VOCAB_SIZE, dtype=torch.float32, device=self.device)
            self.fw.forward(self.k_cache, self.v_cache, self.B, tokens, row_seq, row_pos, out_rows, out_tok, lg)
            if outs:
                got = out_tok.cpu().tolist()
                for (_, s), t in zip(outs, got):
                    next_tok[s] = t
                if lg is not None:
                    for k, (_, s) in enumerate(outs):
                        logits[s].copy_(lg[k])
        torch.cuda.current_stream(self.device).synchronize()
        self.fw.check_status()
        for s, p in enumerate(prompts):
            self.positions[s] += len(p)
        return next_tok

    def _launch_step(self, logits=None) -> None:
        self.fw.forward(self.k_cache, self.v_cache, self.B, self._tok, self._seq, self._pos, self._seq, self._out,
                        logits, workspace=self._ws_step)

    def step(self, tokens, logits: torch.Tensor | None = None) -> torch.Tensor:
        """One decode row per sequence: tokens[s] at positions[s].  Returns the
        greedy next tokens (device int32 [B]); ``logits`` [B, vocab] if given."""
        if any(p >= self.max_seq_len for p in self.positions):
            raise ValueError("a sequence is at max_seq_len")
        self._tok.copy_(torch.as_tensor(tokens, dtype=torch.int32).to(self.device, non_blocking=True))
        self._pos.copy_(_int32(self.positions, self.device))
        self._launch_step(logits)
        self.positions = [p + 1 for p in self.positions]
        return self._out.clone()

    def _capture(self) -> None:
        """CUDA graph of one greedy step: forward, then feed the argmax back as
        the next token and advance every position on the device."""
        self._launch_step()  # warm-up outside capture: cuBLAS handle, workspace
        torch.cuda.current_stream(self.device).synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._launch_step()
            self._tok.copy_(self._out)
            self._pos.add_(1)
        self._graph = g

    def generate(self, first_tokens, max_tokens: int) -> torch.Tensor:
        """Greedy continuation of every sequence from first_tokens[s] at its
        current position; returns the generated ids, device int32
        [max_tokens, B] (row t = step t's argmax)."""
        n = int(max_tokens)
        if n < 1:
            raise ValueError("max_tokens must be >= 1")
        if any(p + n > self.max_seq_len for p in self.positions):
            raise ValueError("generation would exceed max_seq_len")
        log = torch.empty(n, self.B, dtype=torch.int32, device=self.device)
        if self.decode_mode == "megakernel":
            # one launch of the persistent kernel for all n steps
            fw = self.fw
            self._mk_first.copy_(torch.as_tensor(first_tokens, dtype=torch.int32).to(self.device, non_blocking=True))
            fw._ops.run_batch(self._mk_ws, fw.embed, self._mk_layers, fw.final_norm, fw.lm_head, fw.cos, fw.sin,
                              self.k_cache, self.v_cache, self._mk_first, [int(p) for p in self.positions], n,
                              fw.num_layers, self.max_seq_len, fw.attn_scale, log, self._mk_status, 0)
            self.positions = [p + n for p in self.positions]
            return log
        self._tok.copy_(torch.as_tensor(first_tokens, dtype=torch.int32).to(self.device, non_blocking=True))
        self._pos.copy_(_int32(self.positions, self.device))
        if not self.use_graphs:
            for t in range(n):
                self._launch_step()
                log[t].copy_(self._out)
                self._tok.copy_(self._out)
                self._pos.add_(1)
        else:
            if self._graph is None:
                # capture at the current positions, then restore the inputs
                tok0, pos0 = self._tok.clone(), self._pos.clone()
                self._capture()
                self._tok.copy_(tok0)
                self._pos.copy_(pos0)
                # the warm-up and captured steps wrote K/V at the current
                # positions; the replays below rewrite the same rows
            for t in range(n):
                self._graph.replay()
                log[t].copy_(self._out)
        self.positions = [p + n for p in self.positions]
        return log
