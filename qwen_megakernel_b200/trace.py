"""Per-phase critical path of one decode step from the kernel's timeline trace.

The feature instance of the decode kernel stamps %globaltimer (ns) into an
optional buffer (``QmkRunArgs.trace``, ``Decoder.decode_steps(trace=...)``):
per CTA a row of ``qmk_trace_words()`` uint64 words; per layer 16 slots
(phase input ready / phase done, producer issue window) and, after the last
layer, the LM-head slots; then per ring tile six stamps.  Slot meaning is
fixed by the kernel source (``csrc/megakernel.cu``, "Optional timeline
trace").  With ``tuning`` bit 4 (TUNE_TRACE_CLOCK) the stamps are SM clock
cycles (%clock64) instead: the global timer ticks in 256 ns steps on B200,
too coarse inside a phase, while clock64 resolves single cycles but is per
SM, so only differences within one CTA mean something.

``phase_table`` (global-timer trace) gives, per phase and layer:
  * ``span``: max over CTAs of the phase's done stamp minus the same for the
    phase before it -- the phase's share of the step's critical path;
  * ``wait``: the input-ready stamp of a CTA minus the moment the last CTA of
    the previous phase finished (the exchange latency: dataflow word store ->
    L2 -> poll), median over the CTAs of the phase;
  * ``work``: done minus input-ready of a CTA (median and max over CTAs).
``phase_detail`` (clock trace) splits the inside of each phase.
Rows are aggregated over layers (median), so one table describes a step.
"""

from __future__ import annotations

import statistics

import numpy as np

SLOTS_PER_LAYER = 16
# (name, input-ready slot, done slot) in dependency order within a layer
PHASES = (
    ("P1 rmsnorm+qkv", 0, 1),
    ("P2 attention", 2, 3),
    ("P2.5 split merge", 4, 5),
    ("P3 o_proj+residual", 6, 7),
    ("P4 rmsnorm+gate/up+silu", 8, 9),
    ("P5 down+residual", 10, 11),
)
LM_READY, LM_DONE, STEP_START = 0, 1, 5  # slots after the last layer
TRACE_TILES = 512
TILE_BASE = (64 + 1) * SLOTS_PER_LAYER  # after the per-layer slots of kMaxLayers = 64 layers
TUNE_TRACE_CLOCK = 16  # QmkRunArgs.tuning bit: stamps in SM cycles


def _stamps(tr: np.ndarray, slot: int) -> np.ndarray:
    """Column `slot` of the trace as float64, NaN where a CTA did not stamp."""
    col = tr[:, slot].astype(np.int64).astype(np.float64)
    col[col == 0] = np.nan
    return col


def phase_table(trace, num_layers: int) -> dict:
    """Critical-path breakdown of one traced step (global-timer stamps).

    trace: array-like [num_ctas, words_per_cta] of uint64/int64 stamps.
    Returns {"phases": [{name, span_us, wait_us, work_med_us, work_max_us,
    ctas}], "lm_head": {...}, "layer_us": median layer time, "layers_us":
    per-layer spans, "step_us": step time}."""
    tr = np.asarray(trace)
    base_lm = num_layers * SLOTS_PER_LAYER
    start = _stamps(tr, base_lm + STEP_START)
    t0 = np.nanmin(start)
    per_phase = {name: {"span": [], "wait": [], "work_med": [], "work_max": [], "ctas": 0} for name, _, _ in PHASES}
    layer_spans = []
    prev_done_max = np.nanmax(start)
    for layer in range(num_layers):
        b = layer * SLOTS_PER_LAYER
        layer_start = prev_done_max
        for name, rs, ds in PHASES:
            ready = _stamps(tr, b + rs)
            done = _stamps(tr, b + ds)
            ok = ~np.isnan(ready) & ~np.isnan(done)
            if not ok.any():
                continue
            dmax = np.nanmax(done[ok])
            work = done[ok] - ready[ok]
            rec = per_phase[name]
            rec["span"].append(dmax - prev_done_max)
            rec["wait"].append(float(np.median(ready[ok] - prev_done_max)))
            rec["work_med"].append(float(np.median(work)))
            rec["work_max"].append(float(np.max(work)))
            rec["ctas"] = int(ok.sum())
            prev_done_max = dmax
        layer_spans.append(prev_done_max - layer_start)
    lm_ready = _stamps(tr, base_lm + LM_READY)
    lm_done = _stamps(tr, base_lm + LM_DONE)
    ok = ~np.isnan(lm_ready) & ~np.isnan(lm_done)
    lm = {
        "span_us": (np.nanmax(lm_done[ok]) - prev_done_max) / 1e3 if ok.any() else None,
        "wait_us": float(np.median(lm_ready[ok] - prev_done_max)) / 1e3 if ok.any() else None,
        "work_med_us": float(np.median(lm_done[ok] - lm_ready[ok])) / 1e3 if ok.any() else None,
        "work_max_us": float(np.max(lm_done[ok] - lm_ready[ok])) / 1e3 if ok.any() else None,
    }
    rows = []
    for name, _, _ in PHASES:
        rec = per_phase[name]
        if not rec["span"]:
            continue
        rows.append({
            "name": name,
            "span_us": statistics.median(rec["span"]) / 1e3,
            "wait_us": statistics.median(rec["wait"]) / 1e3,
            "work_med_us": statistics.median(rec["work_med"]) / 1e3,
            "work_max_us": statistics.median(rec["work_max"]) / 1e3,
            "ctas": rec["ctas"],
        })
    step_end = np.nanmax(lm_done) if ok.any() else prev_done_max
    return {
        "phases": rows,
        "lm_head": lm,
        "layer_us": statistics.median(layer_spans) / 1e3 if layer_spans else None,
        "layers_us": [s / 1e3 for s in layer_spans],
        "step_us": (step_end - t0) / 1e3,
    }


def _split(n: int, cta: int, ncta: int) -> tuple[int, int]:
    return (n * cta) // ncta, (n * (cta + 1)) // ncta


def _ntiles(r: tuple[int, int], per: int) -> int:
    return max(0, (r[1] - r[0] + per - 1) // per)


def cta_tiles(cta: int, ncta: int, splits: int, position: int, num_layers: int) -> list[tuple[int, str]]:
    """(layer, phase) of every ring tile CTA `cta` consumes in one step, in
    stream order: per layer the q|k|v rows (16 per tile), the attention
    item's K/V positions (64 per tile), O rows (8), gate/up rows (8), down
    rows (4); then the LM-head rows (16).  Mirrors the static partition of
    csrc/qmk_schedule.h."""
    out = []
    item = cta if cta < 8 * splits else -1
    for layer in range(num_layers):
        out += [(layer, "qkv")] * _ntiles(_split(4096, cta, ncta), 16)
        if item >= 0:
            s = item % splits
            ch = ((position * s) // splits, (position * (s + 1)) // splits)
            out += [(layer, "attn")] * _ntiles(ch, 64)
        out += [(layer, "o")] * _ntiles(_split(1024, cta, ncta), 8)
        out += [(layer, "gu")] * _ntiles(_split(3072, cta, ncta), 8)
        out += [(layer, "down")] * _ntiles(_split(1024, cta, ncta), 4)
    out += [(num_layers, "lm")] * _ntiles(_split(151936, cta, ncta), 16)
    return out


_PHASE_SLOTS = {"qkv": (0, 1), "attn": (2, 3), "o": (6, 7), "gu": (8, 9), "down": (10, 11)}


def phase_detail(trace_clk, num_layers: int, splits: int, position: int) -> list[dict]:
    """Inside-the-phase breakdown from a clock64 trace, per phase, medians
    over CTAs and layers, in SM cycles:
      entry_to_ready  this CTA's previous phase done -> this phase's input
                      ready (dataflow wait + staging, as this CTA sees it);
      ready_to_acc    input ready -> first tile's accumulator read (tensor-
                      core phases: issue + MMA + commit + TMEM load);
      per_tile        accumulator read -> the tile's rows emitted;
      gap             one tile's rows emitted -> the next tile's accumulator;
      tail            last rows emitted -> phase done stamp;
      first_release   input ready -> the phase's first tile released (all
                      phases: the ring slot's last reader finished);
      last_release    input ready -> the phase's last tile released;
      absorb          attention: a K/V tile landed -> released;
      late            share of the phase's tiles whose waiter found them not
                      yet landed (waited > 300 cycles: the weight stream was
                      behind)."""
    tr = np.asarray(trace_clk).astype(np.int64)
    ncta = tr.shape[0]
    base = TILE_BASE
    T = TRACE_TILES
    keys = ("entry_to_ready", "ready_to_acc", "per_tile", "gap", "tail", "first_release", "last_release",
            "absorb", "late")
    acc = {k: {q: [] for q in keys} for k in _PHASE_SLOTS}
    order = ["qkv", "attn", "o", "gu", "down"]
    for cta in range(ncta):
        row = tr[cta]
        tiles = cta_tiles(cta, ncta, splits, position, num_layers)
        by = {}
        for k, (layer, ph) in enumerate(tiles[:T]):
            by.setdefault((layer, ph), []).append(k)
        prev_done = None
        for layer in range(num_layers):
            b = layer * SLOTS_PER_LAYER
            for ph in order:
                rs, ds = _PHASE_SLOTS[ph]
                ready, done = int(row[b + rs]), int(row[b + ds])
                if ready == 0 or done == 0:
                    continue
                rec = acc[ph]
                pd = prev_done
                if ph == "o" and int(row[b + 5]) != 0:  # this CTA also merged
                    pd = int(row[b + 5])
                if pd is not None:
                    rec["entry_to_ready"].append(ready - pd)
                ks = by.get((layer, ph), [])
                if ks:
                    waited = [int(row[base + 2 * k + 1]) - int(row[base + 2 * k]) for k in ks]
                    rec["late"].append(sum(1 for x in waited if x > 300) / len(ks))
                    rel = [int(row[base + 3 * T + k]) for k in ks]
                    if all(rel):
                        rec["first_release"].append(rel[0] - ready)
                        rec["last_release"].append(rel[-1] - ready)
                    if ph == "attn":
                        for k in ks:
                            r_, ld = int(row[base + 3 * T + k]), int(row[base + 2 * k + 1])
                            if r_ and ld:
                                rec["absorb"].append(r_ - max(ld, ready))
                    else:
                        a = [int(row[base + 4 * T + k]) for k in ks]
                        d = [int(row[base + 5 * T + k]) for k in ks]
                        if all(a) and all(d):
                            rec["ready_to_acc"].append(a[0] - ready)
                            rec["per_tile"] += [d[i] - a[i] for i in range(len(ks))]
                            rec["gap"] += [a[i + 1] - d[i] for i in range(len(ks) - 1)]
                            rec["tail"].append(done - d[-1])
                prev_done = done

    def med(v):
        return float(np.median(v)) if v else None

    return [{"phase": ph, **{k: med(v) for k, v in acc[ph].items()}} for ph in order]


def format_detail(rows: list[dict]) -> str:
    cols = ["entry_to_ready", "ready_to_acc", "per_tile", "gap", "tail", "first_release", "last_release",
            "absorb", "late"]
    out = ["| phase | " + " | ".join(cols) + " |", "|---|" + "---:|" * len(cols)]
    for r in rows:
        cells = []
        for c in cols:
            v = r.get(c)
            cells.append("" if v is None else (f"{v:.2f}" if c == "late" else f"{v:.0f}"))
        out.append(f"| {r['phase']} | " + " | ".join(cells) + " |")
    return "\n".join(out)


def format_table(tab: dict) -> str:
    """Markdown table of phase_table()'s result."""
    out = ["| phase | span (critical path) us | wait (exchange) us | work median us | work max us | CTAs |",
           "|---|---:|---:|---:|---:|---:|"]
    for r in tab["phases"]:
        out.append(f"| {r['name']} | {r['span_us']:.2f} | {r['wait_us']:.2f} | {r['work_med_us']:.2f} | "
                   f"{r['work_max_us']:.2f} | {r['ctas']} |")
    lm = tab["lm_head"]
    if lm["span_us"] is not None:
        out.append(f"| LM head + argmax | {lm['span_us']:.2f} | {lm['wait_us']:.2f} | {lm['work_med_us']:.2f} | "
                   f"{lm['work_max_us']:.2f} | all |")
    out.append("")
    out.append(f"median layer: {tab['layer_us']:.2f} us; traced step: {tab['step_us']:.2f} us")
    return "\n".join(out)
