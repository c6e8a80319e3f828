"""GPU parity of the group index (tbgb_group_index_build) and of first-seen int64 codes
(tbgb_factorize_i64) against the oracle's restatements of GroupIndex::build and
Dictionary::encode (exact: every output is an integer)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def dev(x):
    import torch

    return torch.as_tensor(np.ascontiguousarray(x)).cuda()


def u32(t):
    return t.cpu().numpy().view(np.uint32)


def check_index(ctx, keys, max_key):
    got = ctx.group_index_build(dev(np.asarray(keys, np.int32)), max_key)
    want = oracle.group_index_build(keys, max_key)
    for f in ("row_to_group", "group_counts", "group_offsets", "rows_by_group"):
        assert np.array_equal(u32(got[f]), want[f]), f
    assert got["n_active"] == want["n_active"]


def test_hand_case(ctx):
    check_index(ctx, [2, 0, 2, 1, 0], 3)


@pytest.mark.parametrize("max_key", [0, 999, 12287, 12288, 70000])
def test_random_columns(ctx, max_key):
    rng = np.random.default_rng(max_key)
    n = 1_000_003
    hi = max(1, (max_key + 1) // 2) if max_key > 10 else max_key + 1  # leave groups empty too
    keys = rng.integers(0, hi, n).astype(np.int32)
    check_index(ctx, keys, max_key)


def test_sorted_and_skewed_columns(ctx):
    keys = np.sort(np.random.default_rng(1).integers(0, 300, 200_000)).astype(np.int32)
    check_index(ctx, keys, 299)
    skew = np.where(np.random.default_rng(2).random(300_000) < 0.9, 7, 11).astype(np.int32)
    check_index(ctx, skew, 20)


def test_errors(ctx):
    import torch

    import winrapids_b200 as wb

    with pytest.raises(wb.InvalidArgument):
        ctx.group_index_build(torch.empty(0, dtype=torch.int32, device="cuda"), 5)
    with pytest.raises(wb.KeyOutOfRange):
        ctx.group_index_build(dev(np.array([0, 6, 1], np.int32)), 5)
    check_index(ctx, [0, 5, 1], 5)  # usable afterwards


def test_group_index_class(ctx):
    import winrapids_b200 as wb

    keys = dev(np.array([3, 1, 3, 0], np.int32))
    gi = wb.GroupIndex.build(ctx, keys, 3)
    assert gi.accumulator_size == 4 and gi.n_rows == 4 and gi.n_active == 3 and gi.is_valid_for(keys)
    assert u32(gi.rows_by_group).tolist() == [3, 1, 0, 2]


@pytest.mark.parametrize("n,ids", [(1, 1), (1000, 10), (1_000_000, 100_000), (2_000_000, 1_500_000)])
def test_factorize(ctx, n, ids):
    rng = np.random.default_rng(n)
    pool = rng.integers(-2**63, 2**63 - 1, ids, dtype=np.int64)
    pool[0] = np.iinfo(np.int64).min
    keys = pool[rng.integers(0, ids, n)]
    codes, uniq = ctx.factorize_i64(dev(keys), ids)
    want_codes, want_uniq = oracle.factorize_first_seen(keys)
    assert np.array_equal(codes.cpu().numpy(), want_codes)
    assert np.array_equal(uniq.cpu().numpy(), want_uniq)


def test_factorize_table_full(ctx):
    import winrapids_b200 as wb

    with pytest.raises(wb.TableFull):
        ctx.factorize_i64(dev(np.arange(10_000, dtype=np.int64)), 100)
    codes, uniq = ctx.factorize_i64(dev(np.array([4, 4, 2], np.int64)), 100)
    assert codes.cpu().tolist() == [0, 0, 1] and uniq.cpu().tolist() == [4, 2]
