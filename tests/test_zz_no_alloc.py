"""tbgb_groupby_dense_noalloc: the context-free entry point that allocates no device
memory (its scratch is a fixed device array inside the library).

It serves callers that must not have the library allocate at call time, such as a
host engine that already reserved nearly all device memory for its own buffers or a
latency-critical loop that cannot take cudaMalloc's implicit synchronisation.  This
file is collected last so that, if it fails, a stop-at-first-failure run has already
run every other test; it passes both alone and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float64).view(np.uint64)


def _noalloc(keys, vals, G, out):
    import torch

    import winrapids_b200 as wb
    from winrapids_b200._lib import lib

    m = wb.Context.moments_struct(out)
    st = lib().tbgb_groupby_dense_noalloc(C.c_void_p(keys.data_ptr()), C.c_void_p(vals.data_ptr()), None,
                                          int(vals.numel()), int(G), C.byref(m),
                                          C.c_void_p(int(torch.cuda.current_stream().cuda_stream)))
    return st


def test_noalloc_matches_the_allocating_entry_point_on_two_calls():
    import torch

    import winrapids_b200 as wb

    ctx = wb.Context(0)
    n, G = 3_000_001, 256
    dk = torch.empty(n, dtype=torch.int32, device="cuda")
    dv = torch.empty(n, dtype=torch.float64, device="cuda")
    ctx.gen_keys_uniform(dk, G, 123)
    ctx.gen_values_normal(dv, 10.0, 2.0, 123)
    dv[::1001] = float("nan")
    dv[7::4999] = float("inf")
    dv[11::7001] = 0.0
    want = {k: v.cpu().numpy() for k, v in ctx.groupby_dense(dk, dv, G).items()}
    absum = torch.zeros(G, dtype=torch.float64, device="cuda").index_add_(
        0, dk.long(), torch.where(torch.isfinite(dv), dv.abs(), torch.zeros_like(dv))).cpu().numpy()
    for call in range(2):  # the second call reuses the scratch left by the first
        out = ctx.alloc_moments(G)
        for t in out.values():
            t.fill_(-12345.0)
        assert _noalloc(dk, dv, G, out) == 0, f"call {call}"
        got = {k: v.cpu().numpy() for k, v in out.items()}
        for f in ("count", "min", "max"):
            assert np.array_equal(_bits(got[f]), _bits(want[f])), (call, f)
        assert np.all(np.abs(got["sum"] - want["sum"]) <= 1e-12 * absum), call
        for f in ("m2", "var_pop", "var_samp"):
            assert np.array_equal(np.isnan(got[f]), np.isnan(want[f])), (call, f)
            ok = ~np.isnan(want[f])
            assert np.all(np.abs(got[f][ok] - want[f][ok]) <= 1e-9 * np.abs(want[f][ok])), (call, f)
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch_and_bad_keys():
    import torch

    import winrapids_b200 as wb

    out = {f: torch.empty(300, dtype=torch.float64, device="cuda") for f in wb.MOMENT_FIELDS}
    dk = torch.zeros(10, dtype=torch.int32, device="cuda")
    dv = torch.ones(10, dtype=torch.float64, device="cuda")
    assert _noalloc(dk, dv, 257, out) == 7   # TBGB_ERR_INVALID_ARGUMENT: n_groups above the 256 limit
    dk[3] = 5
    assert _noalloc(dk, dv, 4, out) == 8     # TBGB_ERR_KEY_OUT_OF_RANGE
    dk[3] = 1
    assert _noalloc(dk, dv, 4, out) == 0     # the error does not stick to the next call
    assert out["count"][:4].cpu().tolist() == [9.0, 1.0, 0.0, 0.0]
