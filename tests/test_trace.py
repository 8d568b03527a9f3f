"""Host logic of the timeline-trace analysis (qwen_megakernel_b200/trace.py),
on synthetic stamps: no GPU."""

import numpy as np

from qwen_megakernel_b200.trace import (SLOTS_PER_LAYER, TILE_BASE, TRACE_TILES, cta_tiles, phase_detail,
                                        phase_table)


def test_cta_tiles_follow_the_partition():
    # 148 CTAs, 18 splits at position 1027: CTA 0 holds 28 q|k|v rows (2
    # tiles), one 57-position K/V tile, 6 O rows (1), 20 gate/up rows (3),
    # 6 down rows (2); CTA 147 is no attention item.
    t0 = cta_tiles(0, 148, 18, 1027, 2)
    assert [p for _, p in t0[:9]] == ["qkv", "qkv", "attn", "o", "gu", "gu", "gu", "down", "down"]
    assert t0[-1] == (2, "lm")
    t147 = cta_tiles(147, 148, 18, 1027, 2)
    assert "attn" not in [p for _, p in t147]
    # every CTA's LM rows: 1026 or 1027 of 151936 -> 65 tiles
    assert sum(1 for _, p in t0 if p == "lm") == 65


def _synthetic(ncta=4, layers=2, words=TILE_BASE + 6 * TRACE_TILES):
    """Each CTA: layer l phase k ready at 1000*(6l+k) + 100*cta, done 50 later."""
    tr = np.zeros((ncta, words), dtype=np.int64)
    for c in range(ncta):
        tr[c, layers * SLOTS_PER_LAYER + 5] = 1  # step start
        for l in range(layers):
            for k, (rs, ds) in enumerate(((0, 1), (2, 3), (4, 5), (6, 7), (8, 9), (10, 11))):
                t = 1000 * (6 * l + k + 1) + 100 * c
                tr[c, l * SLOTS_PER_LAYER + rs] = t
                tr[c, l * SLOTS_PER_LAYER + ds] = t + 50
        tr[c, layers * SLOTS_PER_LAYER + 0] = 20000 + c
        tr[c, layers * SLOTS_PER_LAYER + 1] = 30000 + c
    return tr


def test_phase_table_spans_and_waits():
    tab = phase_table(_synthetic(), 2)
    names = [r["name"] for r in tab["phases"]]
    assert names[0].startswith("P1") and names[-1].startswith("P5")
    for r in tab["phases"][1:]:
        # last CTA done at base + 350; next phase ready 1000 later at base+1000+c*100
        assert abs(r["span_us"] * 1e3 - 1000) < 1e-6
        assert abs(r["wait_us"] * 1e3 - (1000 - 350 + 150)) < 1e-6  # median CTA (c = 1.5)
        assert abs(r["work_med_us"] * 1e3 - 50) < 1e-6
    assert abs(tab["layers_us"][1] * 1e3 - 6000) < 1e-6  # layer 0 also holds the wait from the step start


def test_phase_detail_entry_to_ready():
    rows = {r["phase"]: r for r in phase_detail(_synthetic(ncta=148), 2, 18, 1027)}
    # attention follows P1 of the same CTA: ready 1000 after... 950 after P1 done
    assert rows["attn"]["entry_to_ready"] == 950
    # O follows the merge slot (4, 5) when the CTA stamped it: 950 again
    assert rows["o"]["entry_to_ready"] == 950
