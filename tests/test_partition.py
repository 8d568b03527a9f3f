"""The static work partition (qmk_schedule.h), queried through the C ABI.

Every phase's output rows must be covered exactly once by the CTAs, every
(KV head, split) attention item and every merge task must have exactly one
owner, and the KV chunks of a head must tile [0, position) -- for the B200's
148 CTAs and for other grid sizes the library accepts.
"""

import ctypes

import pytest

N_QKV, N_O, N_GU, N_D, N_LM = 4096, 1024, 3072, 1024, 151936


@pytest.fixture(scope="module")
def lib():
    from qwen_megakernel_b200 import cdll

    return cdll()


def partition(lib, ncta, splits):
    out = (ctypes.c_int * 12)()
    rows = []
    for c in range(ncta):
        assert lib.qmk_describe_partition(ncta, splits, c, out, 12) == 0
        rows.append(list(out))
    return rows


@pytest.mark.parametrize("ncta", [148, 132, 64, 160])
@pytest.mark.parametrize("splits", [1, 7, 8, 18])
def test_rows_items_merges_cover_exactly_once(lib, ncta, splits):
    if 8 * splits > ncta:
        pytest.skip("more items than CTAs")
    rows = partition(lib, ncta, splits)
    for k, n in enumerate((N_QKV, N_O, N_GU, N_D, N_LM)):
        covered = []
        for r in rows:
            b, e = r[2 * k], r[2 * k + 1]
            assert 0 <= b <= e <= n
            covered.extend(range(b, e))
        assert covered == list(range(n)), f"phase {k} not tiled"
        sizes = [r[2 * k + 1] - r[2 * k] for r in rows]
        assert max(sizes) - min(sizes) <= 1, "row split not balanced"
    items = sorted(r[10] for r in rows if r[10] >= 0)
    assert items == list(range(8 * splits))
    merges = sorted(r[11] for r in rows if r[11] >= 0)
    assert merges == list(range(32))
    # Every CTA owns QKV rows: each phase's output then depends on every CTA,
    # which is what makes the flag-word dataflow safe to reuse per layer.
    assert all(r[1] > r[0] for r in rows)


def test_bad_partition_arguments(lib):
    out = (ctypes.c_int * 12)()
    assert lib.qmk_describe_partition(148, 19, 0, out, 12) != 0  # > 18 splits
    assert lib.qmk_describe_partition(148, 1, 148, out, 12) != 0  # CTA out of range
    assert lib.qmk_describe_partition(32, 1, 0, out, 12) != 0  # too few CTAs
    assert lib.qmk_describe_partition(148, 1, 0, out, 11) != 0  # short buffer


def kv_chunk(prev, s, splits):
    return prev * s // splits, prev * (s + 1) // splits


@pytest.mark.parametrize("prev", [0, 1, 17, 1023, 1535, 8192, 32768])
@pytest.mark.parametrize("splits", [1, 5, 18])
def test_kv_chunks_tile_previous_positions(prev, splits):
    covered = []
    for s in range(splits):
        b, e = kv_chunk(prev, s, splits)
        covered.extend(range(b, e))
    assert covered == list(range(prev))
