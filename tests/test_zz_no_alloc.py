"""tbgb_groupby_dense_noalloc: the context-free entry point that allocates no device
memory (its scratch is a fixed device array inside the library).

It serves callers that cannot let a library allocate while they run: a host engine
that already reserved nearly all device memory for its own buffer store, or a
latency-critical loop that cannot take cudaMalloc's implicit synchronisation.  Each
case calls it twice in a row (the second call reuses the scratch the first left
behind) and checks it against both the allocating entry point and the oracle.  This
file is collected last so that, if it fails, a stop-at-first-failure run has already
run every other test; it passes both alone and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from parity import abs_sums, bits, check, to_host

pytestmark = pytest.mark.gpu

FIELDS = ("count", "sum", "min", "max", "mean", "m2", "var_pop", "var_samp", "m3", "m4")
M34_TOL = 1e-9  # |got - want| <= 1e-9 * sum |v - r|^k over the group's finite selected values


def _noalloc(keys, vals, G, out, mask=None):
    import torch

    import winrapids_b200 as wb
    from winrapids_b200._lib import lib

    m = wb.Context.moments_struct(out)
    st = lib().tbgb_groupby_dense_noalloc(C.c_void_p(keys.data_ptr()), C.c_void_p(vals.data_ptr()),
                                          None if mask is None else C.c_void_p(mask.data_ptr()),
                                          int(vals.numel()), int(G), C.byref(m),
                                          C.c_void_p(int(torch.cuda.current_stream().cuda_stream)))
    return st


def _inputs(ctx, n, G, seed):
    import torch

    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    dv = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, G, seed)
    ctx.gen_values_normal(dv, 10.0, 2.0, seed)
    dv[::1001] = float("nan")
    dv[7::4999] = float("inf")
    dv[9::6007] = float("-inf")
    dv[11::7001] = 0.0
    dv[13::7919] = -0.0
    return dk, dv


def _check_m34(got, want, keys, vals, G, live, label):
    c = want["counts"]
    r = np.where(c > 0, want["sums"] / np.where(c > 0, c, 1.0), 0.0)
    ok = np.isfinite(vals) & live
    for f, w, k in (("m3", want["m3s"], 3), ("m4", want["m4s"], 4)):
        scale = np.bincount(keys[ok], weights=np.abs(vals[ok] - r[keys[ok]]) ** k, minlength=G)
        assert np.all(np.abs(got[f] - w) <= M34_TOL * scale), f"{label} {f}"


def _same_as_allocating(got, want, absum, label):
    for f in ("count", "min", "max"):
        assert np.array_equal(bits(got[f]), bits(want[f])), (label, f)
    assert np.all(np.abs(got["sum"] - want["sum"]) <= 1e-12 * absum), label
    for f in ("m2", "var_pop", "var_samp", "m3", "m4"):
        assert np.array_equal(np.isnan(got[f]), np.isnan(want[f])), (label, f)
        ok = ~np.isnan(want[f])
        assert np.all(np.abs(got[f][ok] - want[f][ok]) <= 1e-9 * np.abs(want[f][ok]) + 1e-300), (label, f)


@pytest.mark.parametrize("masked", [False, True])
def test_noalloc_matches_the_allocating_entry_point_and_the_oracle_on_two_calls(masked):
    import torch

    import winrapids_b200 as wb

    ctx = wb.Context(0)
    n, G = 3_000_001, 256
    dk, dv = _inputs(ctx, n, G, 123 + masked)
    keys, vals = dk.cpu().numpy(), dv.cpu().numpy()
    live = np.ones(n, dtype=bool)
    dmask = None
    if masked:
        # a selection over many 4096-row tiles: whole tiles off, runs, and single rows
        rng = np.random.default_rng(5)
        live = rng.random(n) < 0.3
        live[100_000:400_000] = False
        live[1_000_000:1_020_000] = True
        words = np.zeros((n + 63) // 64, dtype=np.uint64)
        idx = np.nonzero(live)[0]
        np.bitwise_or.at(words, idx // 64, np.left_shift(np.uint64(1), (idx % 64).astype(np.uint64)))
        dmask = torch.as_tensor(words.view(np.int64)).cuda()
    want_gpu = to_host(ctx.groupby_dense(dk, dv, G, mask=dmask, out=ctx.alloc_moments(G, FIELDS)))
    want = oracle.moments_grouped_mt(vals, keys, G, threads=8, m34=True,
                                     mask=None if dmask is None else dmask.cpu().numpy().view(np.uint64))
    absum = abs_sums(keys, vals, G, live)
    outs = [ctx.alloc_moments(G, FIELDS) for _ in range(2)]
    torch.cuda.synchronize()
    for call in range(2):  # the second call reuses the scratch left by the first
        for t in outs[call].values():
            t.fill_(-12345.0)
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        assert _noalloc(dk, dv, G, outs[call], dmask) == 0, f"call {call}"
        free1 = torch.cuda.mem_get_info()[0]
        if call == 1:  # the first call on a device may map the library's array; later calls take nothing
            assert free1 == free0, f"device memory changed by {free0 - free1} bytes"
        got = to_host(outs[call])
        label = f"masked={masked} call {call}"
        _same_as_allocating(got, want_gpu, absum, label)
        check(got, want, absum, label)
        _check_m34(got, want, keys, vals, G, live, label)
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch_and_bad_keys():
    import torch

    import winrapids_b200 as wb

    out = {f: torch.empty(300, dtype=torch.float64, device="cuda") for f in wb.MOMENT_FIELDS}
    dk = torch.zeros(10, dtype=torch.int32, device="cuda")
    dv = torch.ones(10, dtype=torch.float64, device="cuda")
    assert _noalloc(dk, dv, 257, out) == 7   # TBGB_ERR_INVALID_ARGUMENT: n_groups above the 256 limit
    assert _noalloc(dk, dv, 0, out) == 7     # and below 1
    dk[3] = 5
    assert _noalloc(dk, dv, 4, out) == 8     # TBGB_ERR_KEY_OUT_OF_RANGE
    dk[3] = 1
    assert _noalloc(dk, dv, 4, out) == 0     # the error does not stick to the next call
    assert out["count"][:4].cpu().tolist() == [9.0, 1.0, 0.0, 0.0]
    empty = torch.empty(0, dtype=torch.int32, device="cuda")
    assert _noalloc(empty, torch.empty(0, dtype=torch.float64, device="cuda"), 4, out) == 0  # n = 0
    assert out["count"][:4].cpu().tolist() == [0.0, 0.0, 0.0, 0.0]
