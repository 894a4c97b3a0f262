"""The attention's split plan and the prefill attention's position groups: host logic, no GPU.

The decode step splits the attention over T positions into `nsplit` runs of `chunk` positions; the
prefill groups prompt positions that share a plan so that one item loads each K/V batch once for all of
them.  These checks go through the C ABI (dk_attn_split_plan, dk_prefill_attn_plan)."""
import ctypes as C

import numpy as np
import pytest

from diolkos_b200._native import lib


def split_plan(T, max_splits, min_chunk):
    ns, ch = C.c_int(), C.c_int()
    assert lib().dk_attn_split_plan(T, max_splits, min_chunk, C.byref(ns), C.byref(ch)) == 0
    return ns.value, ch.value


@pytest.mark.parametrize("max_splits", [1, 5, 16, 24, 93])
def test_split_plan_covers_every_position_without_an_empty_split(max_splits):
    for T in range(1, 4097):
        ns, ch = split_plan(T, max_splits, 16)
        assert 1 <= ns <= max_splits
        assert (ns - 1) * ch < T <= ns * ch, (T, ns, ch)  # the last split holds at least one position
        assert ns <= (T + 15) // 16  # never more splits than runs of 16 positions


def test_split_plan_capped_example():
    # 385 positions over at most 24 splits: chunk 17, so 23 splits (a 24th would start at 391)
    assert split_plan(385, 24, 16) == (23, 17)
    assert split_plan(384, 24, 16) == (24, 16)


def prefill_plan(n_heads, n_kv_heads, max_splits, pos0, ntok):
    out = np.zeros(5 * ntok, np.int32)
    items = C.c_longlong()
    n = lib().dk_prefill_attn_plan(n_heads, n_kv_heads, max_splits, 16, pos0, ntok, out.ctypes.data, C.byref(items))
    assert n > 0
    return out[: 5 * n].reshape(n, 5), items.value


@pytest.mark.parametrize(
    "n_heads,n_kv_heads,max_splits,pos0,ntok",
    [
        (32, 32, 24, 0, 256),      # 7B shape on 148 SMs, first chunk
        (32, 32, 24, 1792, 256),   # 7B, the last chunk of a 2048-token prompt
        (32, 32, 24, 256, 200),    # through the capped positions 385-529
        (64, 8, 93, 1000, 256),    # 70B shape: 8 query heads per KV head
        (8, 1, 32, 256, 44),       # one KV head
    ],
)
def test_prefill_groups_cover_each_item_once_with_the_decode_plan(n_heads, n_kv_heads, max_splits, pos0, ntok):
    g, items = prefill_plan(n_heads, n_kv_heads, max_splits, pos0, ntok)
    kv_mul = n_heads // n_kv_heads
    rows_max = 8  # kPrefillRows
    seen = set()
    expect_item0 = 0
    for first, count, nsplit, chunk, item0 in g:
        assert item0 == expect_item0
        expect_item0 += n_kv_heads * nsplit
        assert 1 <= count and count * kv_mul <= rows_max
        for q in range(count):
            pos = first + q
            ns, ch = split_plan(pos + 1, max_splits, 16)
            assert ns == nsplit and (ns == 1 or ch == chunk)
            for s in range(nsplit):
                t0 = s * chunk
                t1 = min(pos + 1, t0 + chunk)
                # the same positions as the decode step's split s at this position
                assert (t0, t1) == (s * ch, min(pos + 1, (s + 1) * ch)) and t1 > t0
                for h in range(n_kv_heads):
                    key = (pos, h, s)
                    assert key not in seen
                    seen.add(key)
    assert items == expect_item0
    want = sum(n_kv_heads * split_plan(p + 1, max_splits, 16)[0] for p in range(pos0, pos0 + ntok))
    assert len(seen) == want
    assert g[0][0] == pos0 and g[-1][0] + g[-1][1] == pos0 + ntok
