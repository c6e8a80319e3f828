"""The reference's own GPU groupby kernels (scatter_stats / scatter_stats_smem /
scatter_stats_warp, the SCATTER_CUDA_SOURCE string of crates/tambear/src/hash_scatter.rs,
built from the reference tree into oracle/_ref by oracle/build.py) run beside
tbgb_groupby_dense on the same device arrays of NaN-free data (the reference's GPU kernels do
not skip NaN): counts equal, sums within 1e-12 * sum|x| of each other, and the reference's
sum of squares within 1e-9 relative of the oracle's exact sum of v*v."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

import oracle
from parity import abs_sums

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_hash_scatter.so"


@pytest.fixture(scope="module")
def ref():
    if not LIB.exists():
        pytest.skip("oracle/_ref/libref_hash_scatter.so was not built (reference tree absent at build time)")
    return C.CDLL(str(LIB))


@pytest.mark.parametrize("kind,G", [(0, 256), (1, 256), (2, 256), (1, 1000), (2, 7)])
def test_reference_kernels_agree_with_ours(ctx, ref, kind, G):
    import torch

    n = 2_000_003
    keys = oracle.gen_keys_uniform(n, G, 11)
    vals = oracle.gen_values_uniform(n, -1.0, 1.0, 11)
    dk = torch.as_tensor(keys).cuda()
    dv = torch.as_tensor(vals).cuda()
    outs = [torch.empty(G, dtype=torch.float64, device="cuda") for _ in range(3)]
    st = ref.ref_scatter_stats(C.c_int(kind), C.c_void_p(dk.data_ptr()), C.c_void_p(dv.data_ptr()),
                               *[C.c_void_p(o.data_ptr()) for o in outs], C.c_longlong(n), C.c_int(G),
                               C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    r_sum, r_sq, r_cnt = (o.cpu().numpy() for o in outs)
    mine = {k: v.cpu().numpy() for k, v in ctx.groupby_dense(dk, dv, G).items()}
    absum = abs_sums(keys, vals, G)
    assert np.array_equal(r_cnt, mine["count"])
    assert np.all(np.abs(r_sum - mine["sum"]) <= 2e-12 * absum)
    sq = oracle.scatter_phi("v * v", keys, vals, None, G)
    assert np.all(np.abs(r_sq - sq) <= 1e-9 * sq)
