"""The attention's split plan and the prefill attention's position groups: host logic, no GPU.

The decode step splits the attention over T positions into `nsplit` runs of `chunk` positions; the
prefill groups prompt positions that share a plan so that one item loads each K/V batch once for all of
them.  These checks go through the C ABI (dk_attn_split_plan, dk_step_attn_plan, dk_prefill_attn_plan)."""
import ctypes as C

import numpy as np
import pytest

from diolkos_b200._native import lib


def split_plan(T, max_splits, min_chunk):
    ns, ch = C.c_int(), C.c_int()
    assert lib().dk_attn_split_plan(T, max_splits, min_chunk, C.byref(ns), C.byref(ch)) == 0
    return ns.value, ch.value


@pytest.mark.parametrize("min_chunk", [16, 40, 320])
@pytest.mark.parametrize("max_splits", [1, 4, 5, 16, 18, 24, 93])
def test_split_plan_covers_every_position_without_an_empty_split(max_splits, min_chunk):
    for T in range(1, 4097):
        ns, ch = split_plan(T, max_splits, min_chunk)
        assert 1 <= ns <= max_splits
        assert (ns - 1) * ch < T <= ns * ch, (T, ns, ch)  # the last split holds at least one position
        assert ns <= (T + min_chunk - 1) // min_chunk  # never more splits than runs of min_chunk positions


def test_split_plan_capped_example():
    # 385 positions over at most 24 splits: chunk 17, so 23 splits (a 24th would start at 391)
    assert split_plan(385, 24, 16) == (23, 17)
    assert split_plan(384, 24, 16) == (24, 16)


NEVER = 0x7FFFFFFF


def step_plan_args(n_kv_heads, kv_mul, seq_len, num_sms=148, wide_from=None):
    """The persistent step's plan as dk_model_create sets it (engine.cu): narrow items of 2 warps, 5 per
    SM, splits of at least 16 positions, at most one wave of items; wide items of 10 warps, one per SM,
    splits of at least step_min_chunk(kv_mul) = max(80, 320 / kv_mul) positions, from 384 positions on
    unless the wide items would leave more than a tenth of the SMs idle (wide_from given: the
    DIOLKOS_ATTN_WIDE_FROM override)."""
    narrow = max(1, min(5 * num_sms // n_kv_heads, -(-seq_len // 16)))
    wide_chunk = max(80, 320 // kv_mul)
    wide = max(1, min(num_sms // n_kv_heads, -(-seq_len // wide_chunk)))
    if wide_from is None:
        wide_from = NEVER if wide * n_kv_heads * 10 < num_sms * 9 else 384
    return np.array([narrow, 16, wide, wide_chunk, wide_from], np.int32)


@pytest.mark.parametrize("n_kv_heads,num_sms", [(32, 148), (16, 148), (8, 148), (4, 148), (6, 148), (32, 132)])
def test_narrow_items_fit_one_wave(n_kv_heads, num_sms):
    """Every narrow item of a position has a 2-warp group of its own (5 per SM): no second wave."""
    plan = step_plan_args(n_kv_heads, 1, 4096, num_sms=num_sms, wide_from=NEVER)
    for T in range(1, 4097):
        warps, ns, ch = step_plan(T, plan)
        assert warps == 2 and ns * n_kv_heads <= 5 * num_sms, (T, ns)


def test_default_form_choice():
    """The 7B shape on one GPU (32 KV heads: 4 wide splits = 128 items on 148 SMs) keeps the narrow form;
    with 16 KV heads per rank (2 GPUs, 144 items) or the 70B shape's 8 (144 items) the wide form starts at
    384 positions."""
    assert step_plan_args(32, 1, 4096)[4] == NEVER
    assert step_plan_args(16, 1, 4096)[4] == 384
    assert step_plan_args(8, 8, 4096)[4] == 384


def step_plan(T, plan):
    ns, ch = C.c_int(), C.c_int()
    warps = lib().dk_step_attn_plan(T, plan.ctypes.data, C.byref(ns), C.byref(ch))
    assert warps in (2, 10)
    return warps, ns.value, ch.value


@pytest.mark.parametrize("n_kv_heads,kv_mul,wide_from", [(32, 1, 384), (8, 8, 384), (1, 8, 0), (32, 1, 0), (4, 1, 100)])
def test_step_plan_forms(n_kv_heads, kv_mul, wide_from):
    """Narrow up to wide_from positions, wide beyond; no empty split; the wide chunk is whole 8-position
    batches (one split: the run [0, T)) and never more splits than one wave of CTAs."""
    plan = step_plan_args(n_kv_heads, kv_mul, 4096, wide_from=wide_from)
    for T in range(1, 4097):
        warps, ns, ch = step_plan(T, plan)
        assert warps == (2 if T <= wide_from else 10)
        assert (ns - 1) * ch < T <= ns * ch, (T, ns, ch)
        if warps == 2:
            assert (ns, ch) == split_plan(T, plan[0], plan[1])
        else:
            assert 1 <= ns <= plan[2] and ns * n_kv_heads <= 148
            assert ns == 1 and ch == T or ch % 8 == 0, (T, ns, ch)
            assert ns <= -(-T // plan[3])  # never more splits than runs of the shortest split


def prefill_plan(n_heads, n_kv_heads, plan, pos0, ntok):
    out = np.zeros(6 * ntok, np.int32)
    items, narrow = C.c_longlong(), C.c_longlong()
    n = lib().dk_prefill_attn_plan(n_heads, n_kv_heads, plan.ctypes.data, pos0, ntok, out.ctypes.data,
                                   C.byref(items), C.byref(narrow))
    assert n > 0
    return out[: 6 * n].reshape(n, 6), items.value, narrow.value


@pytest.mark.parametrize(
    "n_heads,n_kv_heads,pos0,ntok,wide_from",
    [
        (32, 32, 0, 256, 384),      # 7B shape on 148 SMs, first chunk (narrow)
        (32, 32, 1792, 256, 384),   # 7B, the last chunk of a 2048-token prompt (wide)
        (32, 32, 256, 200, 384),    # through the capped narrow positions 385-529 and the switch at 384
        (32, 32, 256, 200, 100000),  # the narrow form only
        (64, 8, 1000, 256, 384),    # 70B shape: 8 query heads per KV head
        (64, 8, 256, 256, 384),     # 70B through the switch
        (8, 1, 256, 44, 0),         # one KV head, wide throughout
        (8, 1, 256, 44, 384),
    ],
)
def test_prefill_groups_cover_each_item_once_with_the_decode_plan(n_heads, n_kv_heads, pos0, ntok, wide_from):
    kv_mul = n_heads // n_kv_heads
    plan = step_plan_args(n_kv_heads, kv_mul, 4096, wide_from=wide_from)
    g, items, narrow_items = prefill_plan(n_heads, n_kv_heads, plan, pos0, ntok)
    rows_max = 8  # kPrefillRows
    seen = set()
    expect_item0 = 0
    last_warps = 2
    for first, count, nsplit, chunk, item0, warps in g:
        assert item0 == expect_item0
        if warps == 10 and last_warps == 2:
            assert narrow_items == item0  # the narrow groups' items come first
        last_warps = warps
        expect_item0 += n_kv_heads * nsplit
        assert 1 <= count and count * kv_mul <= rows_max
        for q in range(count):
            pos = first + q
            w, ns, ch = step_plan(pos + 1, plan)
            assert w == warps and ns == nsplit and (ns == 1 or ch == chunk)
            for s in range(nsplit):
                t0 = s * chunk
                t1 = min(pos + 1, t0 + chunk)
                # the same positions as the decode step's split s at this position
                assert (t0, t1) == (s * ch, min(pos + 1, (s + 1) * ch)) and t1 > t0
                for h in range(n_kv_heads):
                    key = (pos, h, s)
                    assert key not in seen
                    seen.add(key)
    if last_warps == 2:
        assert narrow_items == items
    assert items == expect_item0
    want = sum(n_kv_heads * step_plan(p + 1, plan)[1] for p in range(pos0, pos0 + ntok))
    assert len(seen) == want
    assert g[0][0] == pos0 and g[-1][0] + g[-1][1] == pos0 + ntok


def test_wide_prefill_groups_hold_eight_positions():
    """Past the split cap the wide chunk changes only every 8 x nsplit positions: 7B groups are full
    (the 7B shape with the wide form forced from 384 positions)."""
    plan = step_plan_args(32, 1, 4096, wide_from=384)
    g, _, _ = prefill_plan(32, 32, plan, 1792, 256)
    assert (g[:, 5] == 10).all()
    assert np.mean(g[:, 1]) > 7.0, g[:, 1]
