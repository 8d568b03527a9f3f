"""Benchmark: batch-1 greedy decode tok/s of Qwen3-0.6B (bf16) at ~1k context.

Workload: seeded random-init Qwen3-0.6B weights; a
1024-token uniform-random prompt is prefilled (untimed, forced decode steps),
then every bench step is ONE kernel launch that greedily generates 512 tokens
from position 1023 (the reference's generate_nosync semantics), i.e. cache
positions 1023..1534.  Weights (1.19 GB) are streamed from HBM every token, so
the inputs are far larger than the 126 MB L2 and no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own PyTorch path (HF Qwen3ForCausalLM,
bf16, qwen_megakernel/bench.py:19-55) on the host CPU cores, on the same
workload, bounded to a few decode tokens per step.

Multi-GPU (torchrun, one process per GPU): every rank runs an independent
replica with its own prompt seed; no collective on the data path.  Rank 0
prints one JSON line with the whole-job throughput (tokens of all ranks over
the max device time of the ranks).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s (Qwen3-0.6B bf16, ctx 1k)"
PROMPT_LEN = 1024
GEN_TOKENS = 512
WEIGHT_BYTES = 1_192_101_888  # per token: 28 layers' linears + norms + embed row + LM head
KV_BYTES_PER_POS = 114_688  # 28 layers x 8 KV heads x 128 dims x (K, V) x 2 B
WORKLOAD = (
    "configs[1]: Qwen3-0.6B (random init, seed 0) batch-1 greedy decode of 512 tokens after a "
    "1024-token random-id prompt (cache positions 1023..1534), one launch per 512 tokens"
)


def kv_bytes(first_pos: int, n: int) -> int:
    """Algorithmic KV bytes of n tokens at positions first_pos..first_pos+n-1:
    a token at position p reads p cached positions and writes one."""
    return KV_BYTES_PER_POS * sum(p + 1 for p in range(first_pos, first_pos + n))


def launch_bytes() -> int:
    return GEN_TOKENS * WEIGHT_BYTES + kv_bytes(PROMPT_LEN - 1, GEN_TOKENS)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic_per_token():
    """DRAM bytes per decoded token from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "decode_kernel_traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_token"])
    except Exception:
        return None


def smi_gpu_id(local: int) -> str:
    """nvidia-smi's id of CUDA device `local`: with CUDA_VISIBLE_DEVICES set,
    its local-th entry (a physical index or a UUID, both accepted by
    `nvidia-smi -i`), else the index itself."""
    ids = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return ids[local] if local < len(ids) else str(local)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = (
        "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu = smi_gpu_id(gpu_index)
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except OSError:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t:
            self._t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws: int, local: int):
    if ws <= 1:
        return False
    import datetime

    import torch.distributed as dist

    backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120), **kw)
    return True


def reduce_max(x: float, distributed: bool) -> float:
    if not distributed:
        return x
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(distributed: bool):
    if distributed:
        import torch.distributed as dist

        dist.barrier()


def prompt_for_rank(rank: int) -> list[int]:
    rng = np.random.Generator(np.random.PCG64(2 + rank))
    return [int(x) for x in rng.integers(0, 151936, size=PROMPT_LEN)]


# ------------------------------------------------------------------ CPU legs
def cpu_reference_rate(weights_cpu: dict, prompt: list[int], tokens_per_step: int, steps: int, warmup: int):
    """HF Qwen3ForCausalLM bf16 (the reference's PyTorch path) on the host CPU:
    prefill the prompt once (untimed), then time greedy decode of
    `tokens_per_step` tokens per step from the prompt's KV cache."""
    from oracle.hf_reference import build_hf_model

    torch.set_num_threads(os.cpu_count() or 1)
    model = build_hf_model(weights_cpu, torch.bfloat16)
    with torch.no_grad():
        out = model(input_ids=torch.tensor([prompt[:-1]]), use_cache=True, logits_to_keep=1)
        base_cache = out.past_key_values

        def one_step():
            import copy

            cache = copy.deepcopy(base_cache)
            tok = prompt[-1]
            for _ in range(tokens_per_step):
                o = model(input_ids=torch.tensor([[tok]]), past_key_values=cache, use_cache=True)
                cache = o.past_key_values
                tok = int(o.logits[0, -1].argmax())

        for _ in range(warmup):
            one_step()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            one_step()
            times.append(time.perf_counter() - t0)
    total = sum(times)
    return tokens_per_step * steps / total, total * 1000.0 / steps, torch.get_num_threads()


def run_reference_arm(args):
    ws, rank, local = dist_env()
    if rank != 0:
        return 0
    from qwen_megakernel_b200.weights import random_weights

    t0 = time.time()
    weights = random_weights(seed=0, device="cpu", max_seq_len=2048)
    prompt = prompt_for_rank(0)
    tps = 4
    value, ms, cores = cpu_reference_rate(weights, prompt, tps, args.steps, max(1, min(args.warmup, 1)))
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
        "config": {
            "workload": WORKLOAD,
            "sample": f"{tps} greedy tokens per step from position {PROMPT_LEN - 1} after an untimed prefill",
        },
        "cpu_baseline": {
            "value": round(value, 3),
            "unit": "tok/s",
            "cores": cores,
            "kind": "reference",
            "sample": f"HF Qwen3ForCausalLM bf16 on CPU, {tps} decode tokens x {args.steps} steps at ctx ~1k",
        },
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_seconds": round(time.time() - t0, 1),
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm
def run_ours(args):
    ws, rank, local = dist_env()
    distributed = init_dist(ws, local)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200._native import loaded_library_paths
    from qwen_megakernel_b200.weights import random_weights

    weights_cpu = random_weights(seed=0, device="cpu", max_seq_len=2048)
    weights = {
        k: ([t.to(dev) for t in v] if isinstance(v, list) else v.to(dev)) for k, v in weights_cpu.items()
    }
    weights["lm_head_weight"] = weights["embed_weight"]
    dec = Decoder(weights, max_seq_len=2048)
    prompt = prompt_for_rank(rank)
    dec.prefill(prompt[:-1])  # positions 0..1022
    start = PROMPT_LEN - 1
    log = torch.empty(GEN_TOKENS, dtype=torch.int32, device=dev)
    first = torch.tensor([prompt[-1]], dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        dec.decode_steps(GEN_TOKENS, forced_tokens=first, start_position=start, output_log=log)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dec.check_status()

    sampler = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(distributed)
    torch.cuda.synchronize(dev)
    sampler.start()
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    t_all0.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t_all1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier(distributed)
    dec.check_status()
    local_ms = t_all0.elapsed_time(t_all1)
    per_launch_ms = [a.elapsed_time(b) for a, b in ev]
    max_ms = reduce_max(local_ms, distributed)

    # end to end through the public API (host token in, host tokens out)
    e2e_ev0, e2e_ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dec.generate_from(prompt[-1], GEN_TOKENS, position=start)  # warm
    barrier(distributed)
    torch.cuda.synchronize(dev)
    e2e_ev0.record(stream)
    t_host0 = time.perf_counter()
    for _ in range(args.steps):
        dec.generate_from(prompt[-1], GEN_TOKENS, position=start)
    e2e_ev1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_host_ms = (time.perf_counter() - t_host0) * 1000.0
    e2e_ms = max(e2e_ev0.elapsed_time(e2e_ev1), e2e_host_ms)
    e2e_max = reduce_max(e2e_ms, distributed)
    barrier(distributed)

    tokens_total = args.steps * GEN_TOKENS * ws
    value = tokens_total / (max_ms / 1000.0)
    e2e_value = tokens_total / (e2e_max / 1000.0)

    cpu_baseline = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        try:
            v, ms, cores = cpu_reference_rate(weights_cpu, prompt, 8, 2, 1)
            cpu_baseline = {
                "value": round(v, 3),
                "unit": "tok/s",
                "cores": cores,
                "kind": "reference",
                "sample": "HF Qwen3ForCausalLM bf16 on the host CPU (the reference's PyTorch path): "
                "1023-token prefill untimed, then 2 x 8 greedy decode tokens at ctx ~1k",
            }
        except Exception as e:  # the baseline is informative; never fail the bench on it
            cpu_baseline = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                            "sample": f"failed: {type(e).__name__}: {e}"}

    extras = {}
    if not args.no_extras:
        try:
            extras = measure_extras(args, rank, ws, distributed)
        except Exception as e:  # secondary configs are informative; never lose the headline line
            extras = {"error": f"{type(e).__name__}: {e}"}

    if rank == 0:
        peak, peak_kind = measured_peak()
        lb = launch_bytes()
        mean_launch_ms = statistics.mean(per_launch_ms)
        achieved = lb / (mean_launch_ms / 1000.0) / 1e9
        tpt = profiled_traffic_per_token()
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "tok/s",
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(max_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
            "config": {
                "workload": WORKLOAD,
                "batch": 1,
                "prompt_len": PROMPT_LEN,
                "gen_tokens_per_step": GEN_TOKENS,
                "accumulate": "fp32",
                "parallelism": f"replicas x{ws} (independent decode stream per GPU, no collective)",
                "l2": "no flush: 1.19 GB of weights streamed per token >> 126 MB L2",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": (round(tpt * GEN_TOKENS) if tpt else None),
                "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": lb,
                "kernel": "qmk::decode_kernel",
            },
            "e2e": {
                "value": round(e2e_value, 2),
                "unit": "tok/s",
                "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * GEN_TOKENS,
            },
            "gpu_launches": args.steps,
            "clocks": clocks,
            "per_token_us": round(max_ms / args.steps / GEN_TOKENS * 1000.0, 2),
            "native_libraries": [os.path.basename(p) for p in loaded_library_paths()],
        }
        if cpu_baseline is not None:
            line["cpu_baseline"] = cpu_baseline
        if extras:
            line["extra"] = extras
        print(json.dumps(line), flush=True)

    if distributed:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def run_profile_case(steps: int) -> int:
    """Small case for ncu captures: the bench model and prompt, one prefill
    launch (positions 0..1022), then ONE decode launch of `steps` tokens at
    ctx ~1k (the launch to capture: ncu -k regex:decode_kernel -s 1 -c 1)."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device="cuda", max_seq_len=2048)
    dec = Decoder(weights, max_seq_len=2048)
    prompt = prompt_for_rank(0)
    dec.prefill(prompt[:-1])
    first = torch.tensor([prompt[-1]], dtype=torch.int32, device=dev)
    log = torch.empty(steps, dtype=torch.int32, device=dev)
    dec.decode_steps(steps, forced_tokens=first, start_position=PROMPT_LEN - 1, output_log=log)
    torch.cuda.synchronize(dev)
    dec.check_status()
    print(json.dumps({"profile_case": {"steps": steps, "tokens": log[:4].tolist(),
                                       "max_memory_gb": round(torch.cuda.max_memory_allocated() / 1e9, 3)}}))
    return 0


def run_profile_ctx(L: int, steps: int = 4) -> int:
    """Small long-context case for ncu captures: K/V cache of bf16 N(0, 1)
    at positions [0, L) (as `--ctx L`), one warm-up launch, then ONE launch
    of `steps` tokens (capture with ncu -k regex:decode_kernel -s 1 -c 1)."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights, rope_tables

    msl = L + steps + 8
    weights = random_weights(seed=0, device=dev, max_seq_len=2048)
    weights["cos_table"], weights["sin_table"] = rope_tables(msl, device=dev)
    dec = Decoder(weights, max_seq_len=msl)
    gen = torch.Generator(device=dev).manual_seed(2)
    dec.k_cache[:, :, :L].normal_(generator=gen)
    dec.v_cache[:, :, :L].normal_(generator=gen)
    first = torch.tensor([17], dtype=torch.int32, device=dev)
    log = torch.empty(steps, dtype=torch.int32, device=dev)
    for _ in range(2):
        dec.decode_steps(steps, forced_tokens=first, start_position=L, output_log=log)
    torch.cuda.synchronize(dev)
    dec.check_status()
    print(json.dumps({"profile_ctx": {"ctx": L, "steps": steps, "tokens": log.tolist(),
                                      "max_memory_gb": round(torch.cuda.max_memory_allocated() / 1e9, 3)}}))
    return 0


def run_trace(steps: int) -> int:
    """Per-phase critical path of the decode kernel: the bench model and
    prompt, then launches of `steps` greedy tokens at ctx ~1k whose middle
    step is traced (the feature instance of the kernel carries the trace
    stamps).  Three global-timer traces (the fastest step is tabulated) and
    one clock64 trace (inside the phases).  Prints markdown tables and one
    JSON line."""
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    from qwen_megakernel_b200 import Decoder, cdll
    from qwen_megakernel_b200.trace import TUNE_TRACE_CLOCK, format_detail, format_table, phase_detail, phase_table
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device="cuda", max_seq_len=2048)
    dec = Decoder(weights, max_seq_len=2048)
    prompt = prompt_for_rank(0)
    dec.prefill(prompt[:-1])
    lib = cdll()
    ncta = lib.qmk_num_ctas(0)
    words = lib.qmk_trace_words()
    first = torch.tensor([prompt[-1]], dtype=torch.int32, device=dev)
    log = torch.empty(steps, dtype=torch.int32, device=dev)

    def traced(tuning: int):
        trace = torch.zeros(ncta * words, dtype=torch.int64, device=dev)
        dec.decode_steps(steps, forced_tokens=first, start_position=PROMPT_LEN - 1, output_log=log,
                         trace=trace, trace_step=steps // 2, tuning=tuning)
        torch.cuda.synchronize(dev)
        dec.check_status()
        return trace.view(ncta, words).cpu().numpy()

    tabs = [phase_table(traced(0), dec.num_layers) for _ in range(3)]
    best = min(tabs, key=lambda t: t["step_us"])
    pos = PROMPT_LEN - 1 + steps // 2
    splits = lib.qmk_attention_splits(ncta, PROMPT_LEN - 1 + steps - 1)
    detail = phase_detail(traced(TUNE_TRACE_CLOCK), dec.num_layers, splits, pos)
    print(format_table(best))
    print()
    print("inside the phases (SM cycles, clock64):")
    print(format_detail(detail))
    print(json.dumps({"trace": {"steps": steps, "traced_step": steps // 2, "position": pos, "ctas": ncta,
                                "step_us": [round(t["step_us"], 2) for t in tabs], "phases": best["phases"],
                                "lm_head": best["lm_head"], "layer_us": best["layer_us"],
                                "detail_cycles": detail}}), flush=True)
    return 0


def measure_batch(B: int, steps: int, warmup: int, seed_base: int = 100, distributed: bool = False,
                  clock_gpu: int = 0) -> dict:
    """BASELINE config 4 (and config 5's batch-16 replicas): B independent
    sequences, 1024-token random prompts (token-parallel prefill, untimed),
    then `steps` batched greedy decode steps (CUDA-graph replays, B tokens
    each) through BatchDecoder.generate.  Device time with CUDA events,
    max over ranks when distributed."""
    dev = torch.device("cuda", torch.cuda.current_device())
    from qwen_megakernel_b200 import BatchDecoder
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device=dev, max_seq_len=2048)
    bd = BatchDecoder(weights, B, max_seq_len=2048)
    prompts = [prompt_for_rank(seed_base + s) for s in range(B)]
    first = bd.prefill(prompts)
    pos0 = bd.positions[0]
    bd.generate(first, max(1, warmup))  # capture + warm-up (advances positions)
    torch.cuda.synchronize(dev)
    p_start = bd.positions[0]
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(clock_gpu)
    barrier(distributed)
    torch.cuda.synchronize(dev)
    sampler.start()
    e0.record(stream)
    log = bd.generate(first, steps)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier(distributed)
    ms = reduce_max(e0.elapsed_time(e1), distributed)
    # end to end: host tokens in, host token log out
    t0 = time.perf_counter()
    out = bd.generate(first, steps).cpu()
    e2e_ms = reduce_max((time.perf_counter() - t0) * 1000.0, distributed)
    bd.check_status()
    step_bytes = [WEIGHT_BYTES + B * KV_BYTES_PER_POS * (p + 1) for p in range(p_start, p_start + steps)]
    achieved = sum(step_bytes) / (ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    del log
    return {
        "metric": f"batched decode tok/s (Qwen3-0.6B bf16, ctx 1k, B={B})",
        "value": round(B * steps / (ms / 1000.0), 1), "unit": "tok/s", "steps": steps, "warmup": warmup,
        "ms_per_step": round(ms / steps, 4), "batch": B,
        "workload": f"configs[3]-style: {B} sequences, 1024-token prompts, {steps} greedy steps "
                    f"(cache positions {p_start}..{p_start + steps - 1}), "
                    + ("one launch of the persistent decode kernel (batched instance)" if bd.decode_mode == "megakernel"
                       else "token-parallel kernels, CUDA-graph step"),
        "decode_path": bd.decode_mode,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_step": int(sum(step_bytes) / steps)},
        "e2e": {"value": round(B * steps / (e2e_ms / 1000.0), 1), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * B},
        "prefill_positions": pos0, "clocks": clocks, "tokens_sample": out[:2, :4].tolist(),
    }


def run_batch(args) -> int:
    """BASELINE config 4 as its own JSON line: `bench.py --batch B`."""
    torch.cuda.set_device(0)
    from qwen_megakernel_b200._native import loaded_library_paths

    r = measure_batch(args.batch, args.steps, args.warmup)
    line = {k: v for k, v in r.items() if k not in ("workload", "batch")}
    line.update({"n_gpus": 1, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                 "data": "synthetic (seeded random-init weights, uniform random prompt ids)",
                 "config": {"workload": r["workload"], "batch": r["batch"],
                            "path": "token-parallel (qmk_batch_forward), CUDA-graph step"},
                 "native_libraries": [os.path.basename(p) for p in loaded_library_paths()]})
    print(json.dumps(line), flush=True)
    return 0


def run_profile_batch(B: int) -> int:
    """Small case for ncu launch lists of the token-parallel path: B
    sequences prefilled with 1024-token prompts, 2 warm-up steps, then ONE
    eager batched decode step between cudaProfilerStart/Stop (capture with
    ncu --profile-from-start off)."""
    torch.cuda.set_device(0)
    from qwen_megakernel_b200 import BatchDecoder
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device="cuda", max_seq_len=2048)
    bd = BatchDecoder(weights, B, max_seq_len=2048, use_graphs=False)
    first = bd.prefill([prompt_for_rank(100 + s) for s in range(B)])
    bd.generate(first, 2)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    bd.generate(first, 1)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    bd.fw.check_status()
    print(json.dumps({"profile_batch": {"batch": B, "positions": bd.positions[:2]}}))
    return 0


def measure_long_context(L: int, steps: int, warmup: int, reps: int = 3) -> dict:
    """the K/V cache holds bf16 N(0, 1) at positions
    [0, L) (seed 2), then launches of `steps` greedy decode steps at
    positions L, L+1, ... through the megakernel (mean of `reps` launches)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights, rope_tables

    msl = L + steps + 8
    weights = random_weights(seed=0, device=dev, max_seq_len=2048)
    weights["cos_table"], weights["sin_table"] = rope_tables(msl, device=dev)
    dec = Decoder(weights, max_seq_len=msl)
    gen = torch.Generator(device=dev).manual_seed(2)
    dec.k_cache[:, :, :L].normal_(generator=gen)
    dec.v_cache[:, :, :L].normal_(generator=gen)
    first = torch.tensor([17], dtype=torch.int32, device=dev)
    log = torch.empty(steps, dtype=torch.int32, device=dev)

    def launch():
        dec.decode_steps(steps, forced_tokens=first, start_position=L, output_log=log)

    for _ in range(max(1, warmup)):
        launch()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        launch()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    dec.check_status()
    ms = e0.elapsed_time(e1) / reps
    launch_b = steps * WEIGHT_BYTES + kv_bytes(L, steps)
    achieved = launch_b / (ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    return {
        "metric": f"batch-1 decode tok/s (Qwen3-0.6B bf16, ctx {L})", "value": round(steps / (ms / 1000.0), 2),
        "unit": "tok/s", "steps": steps, "reps": reps, "ms_per_launch": round(ms, 4),
        "per_token_us": round(ms / steps * 1000.0, 2),
        "workload": f"configs[2]: {steps} greedy steps at positions {L}..{L + steps - 1}, one launch; "
                    f"K/V cache N(0,1) at positions [0, {L})",
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": launch_b},
        "clocks": clocks,
    }


def run_long_context(args) -> int:
    """BASELINE config 3 as its own JSON line: `bench.py --ctx L`."""
    torch.cuda.set_device(0)
    r = measure_long_context(args.ctx, args.steps, args.warmup)
    line = {k: v for k, v in r.items() if k != "workload"}
    line.update({"n_gpus": 1, "higher_is_better": True, "dtype": "bf16",
                 "data": "synthetic (seeded random-init weights, K/V cache N(0,1) at positions [0, L))",
                 "config": {"workload": r["workload"], "ctx": args.ctx}})
    print(json.dumps(line), flush=True)
    return 0


def measure_prefill(steps: int, warmup: int) -> dict:
    """Token-parallel prompt prefill: a 1024-token prompt through
    Decoder.prefill_batched, median of `steps` timed repetitions."""
    dev = torch.device("cuda", torch.cuda.current_device())
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device=dev, max_seq_len=2048)
    dec = Decoder(weights, max_seq_len=2048)
    prompt = prompt_for_rank(0)
    for _ in range(max(1, warmup)):
        dec.reset()
        dec.prefill_batched(prompt)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    times = []
    for _ in range(steps):
        dec.reset()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tok = dec.prefill_batched(prompt)
        e1.record()
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1))
    clocks = sampler.stop()
    ms = statistics.median(times)
    flops = 2 * 2 * 595_984_384 * PROMPT_LEN  # stacked hi/lo GEMMs: twice the model's 2 N flops per token
    peak_tf, kind = 1590.0, "fallback"
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak_tf, kind = float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, ValueError, KeyError):
        pass
    return {
        "metric": "prefill tok/s (Qwen3-0.6B bf16, 1024-token prompt, token-parallel)",
        "value": round(PROMPT_LEN / (ms / 1000.0), 1), "unit": "tok/s", "ms_per_prompt": round(ms, 3),
        "steps": steps, "warmup": warmup,
        "roofline": {"bound": "tensor", "achieved": round(flops / (ms / 1000.0) / 1e12, 1), "peak": peak_tf,
                     "unit": "TFLOP/s", "frac": round(flops / (ms / 1000.0) / 1e12 / peak_tf, 4),
                     "flops_per_prompt": flops, "peak_kind": kind},
        "next_token": tok, "clocks": clocks,
    }


def run_prefill(args) -> int:
    torch.cuda.set_device(0)
    r = measure_prefill(args.steps, args.warmup)
    r["dtype"] = "bf16"
    print(json.dumps(r), flush=True)
    return 0


def run_profile_prefill() -> int:
    """Small case for ncu launch lists of the token-parallel prefill: one
    warm 1024-token prefill, then ONE more between cudaProfilerStart/Stop
    (capture with ncu --profile-from-start off)."""
    torch.cuda.set_device(0)
    from qwen_megakernel_b200 import Decoder
    from qwen_megakernel_b200.weights import random_weights

    weights = random_weights(seed=0, device="cuda", max_seq_len=2048)
    dec = Decoder(weights, max_seq_len=2048)
    prompt = prompt_for_rank(0)
    dec.prefill_batched(prompt)
    dec.reset()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    tok = dec.prefill_batched(prompt)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"profile_prefill": {"tokens": PROMPT_LEN, "next_token": tok}}))
    return 0


def run_profile_gemm(n: int, rows: int, k: int, reps: int = 8) -> int:
    """The token-parallel path's tensor-core GEMM alone (qmk_gemm_bf16_nt,
    C[rows, n] = A[rows, k] W[n, k]^T, bf16 in, fp32 out) on random operands:
    `reps` launches timed with CUDA events, checked against torch fp32.  For
    ncu: -k regex:gemm_kernel -s 2 -c 1."""
    import ctypes

    torch.cuda.set_device(0)
    from qwen_megakernel_b200 import cdll

    lib = cdll()
    vp, i, ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
    lib.qmk_gemm_bf16_nt.restype = i
    lib.qmk_gemm_bf16_nt.argtypes = [vp, ll, ll, i, vp, ll, ll, i, i, i, i, vp, ll, ll, ll, vp, vp]
    g = torch.Generator(device="cuda").manual_seed(0)
    W = torch.randn(n, k, generator=g, device="cuda").to(torch.bfloat16)
    A = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    C = torch.empty(rows, n, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def run():
        rc = lib.qmk_gemm_bf16_nt(W.data_ptr(), k, 0, n, A.data_ptr(), k, 0, rows, k, 1, 1, C.data_ptr(), n, 0, 0,
                                  None, stream)
        if rc != 0:
            raise RuntimeError(lib.qmk_get_last_error_message())

    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1000.0
    err = (C - A.float() @ W.float().T).abs().max().item()
    print(json.dumps({"profile_gemm": {"n": n, "rows": rows, "k": k, "us": round(us, 2),
                                       "tflops": round(2 * n * rows * k / (us * 1e-6) / 1e12, 1),
                                       "bytes_gbs": round((n * k + rows * k) * 2 / (us * 1e-6) / 1e9, 1),
                                       "max_err": err}}))
    return 0


def measure_extras(args, rank: int, ws: int, distributed: bool) -> dict:
    """The secondary BASELINE configs as extra keys of the headline line.
    One GPU: configs[2] (ctx 8192 and 32768, 64 steps), configs[3] (B = 4,
    16, 64; 64 batched steps) and the 1024-token prefill.  N GPUs (config
    5): every rank also decodes a batch of 16 of its own sequences; the
    whole-job rate is all ranks' tokens over the slowest rank's time."""
    extras = {}
    torch.cuda.empty_cache()
    if ws == 1:
        for L in (8192, 32768):
            extras[f"ctx{L}"] = measure_long_context(L, 64, 1, reps=2)
            torch.cuda.empty_cache()
        for B in (4, 16, 64):
            extras[f"batch{B}"] = measure_batch(B, 64, 3)
            torch.cuda.empty_cache()
        extras["prefill1024"] = measure_prefill(5, 2)
    else:
        r = measure_batch(16, 64, 3, seed_base=1000 * (rank + 1), distributed=distributed,
                          clock_gpu=torch.cuda.current_device())
        total = 16 * 64 * ws
        r["value"] = round(total / (r["ms_per_step"] * 64 / 1000.0), 1)
        r["e2e"]["value"] = round(r["e2e"]["value"] * ws, 1)  # per-rank rate over the slowest rank's time
        r["metric"] = "batched decode tok/s, batch-16 replicas (whole job)"
        r["n_gpus"] = ws
        extras["batch16_replicas"] = r
    return extras


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the secondary configs (ctx 8k/32k, batches 4/16/64, prefill; N>1: batch-16 replicas)")
    ap.add_argument("--profile-case", type=int, default=0, metavar="STEPS",
                    help="run only the small ncu case: one decode launch of STEPS tokens")
    ap.add_argument("--batch", type=int, default=0, metavar="B",
                    help="config 4 instead of the headline: B sequences decoded together (B = 4: the decode kernel's "
                         "batched instance; otherwise the token-parallel kernels)")
    ap.add_argument("--prefill", action="store_true", help="time the token-parallel 1024-token prefill instead")
    ap.add_argument("--ctx", type=int, default=0, metavar="L",
                    help="config 3 instead of the headline: batch-1 decode after L cached positions of random K/V")
    ap.add_argument("--profile-batch", type=int, default=0, metavar="B",
                    help="run only the small ncu case of the token-parallel path: one batched step of B rows")
    ap.add_argument("--trace", type=int, default=0, metavar="STEPS",
                    help="print the per-phase critical path of one traced step of a STEPS-token launch")
    ap.add_argument("--profile-ctx", type=int, default=0, metavar="L",
                    help="run only the small ncu case of a long context: 4-token launches after L random K/V positions")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="run only the small ncu case of the token-parallel prefill")
    ap.add_argument("--profile-gemm", type=int, nargs=3, default=None, metavar=("N", "ROWS", "K"),
                    help="run only the tensor-core GEMM C[ROWS, N] = A[ROWS, K] W[N, K]^T")
    args = ap.parse_args(argv)
    if args.profile_prefill:
        return run_profile_prefill()
    if args.profile_ctx:
        return run_profile_ctx(args.profile_ctx)
    if args.profile_gemm:
        return run_profile_gemm(*args.profile_gemm)
    if args.trace:
        return run_trace(args.trace)
    if args.profile_batch:
        return run_profile_batch(args.profile_batch)
    if args.batch:
        return run_batch(args)
    if args.ctx:
        return run_long_context(args)
    if args.prefill:
        return run_prefill(args)
    if args.profile_case:
        return run_profile_case(args.profile_case)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
