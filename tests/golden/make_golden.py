"""Write tests/golden/reference_vectors.json: the reference's own golden vectors.

The reference is Rust and cannot be built here, so its known-answer tests are
transcribed: each case records its inputs and the expected values asserted by
the cited reference test (paths relative to the reference project root).  For
the adversarial corpora, whose reference tests compare against the Kulisch
oracle rather than literals, the expected correctly-rounded sums are computed
independently with Python's math.fsum (Shewchuk's exact summation), which
pins the oracle's Kulisch restatement without trusting it.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import math
import struct
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_vectors.json"

TINY = struct.unpack("<d", struct.pack("<Q", 1))[0]  # f64::from_bits(1)


def enc(x: float):
    """JSON-safe float: non-finite and -0.0 as strings, everything else as hex for bit-exactness."""
    return float.hex(x) if math.isfinite(x) else ("nan" if math.isnan(x) else ("inf" if x > 0 else "-inf"))


def encl(xs):
    return [enc(float(x)) for x in xs]


def exact(xs):
    return math.fsum([x for x in xs if math.isfinite(x) and x != 0.0])


# ---- determinism_contract.rs corpora (crates/tambear/tests/determinism_contract.rs:49-101)
def corpus_small():
    return [1.0, 2.0, 3.0, 4.0, 5.0]


def corpus_signed():
    return [3.7, -0.25, 1e10, -0.5, 1.25, -1e10, 42.0, -6.0]


def corpus_cancellation():
    xs = []
    for _ in range(1000):
        xs += [1e17, 1.0, -1e17]
    return xs


def corpus_kahan_trap():
    return [1.0] + [1e-10] * 10000


def corpus_mixed_scale():
    out = []
    for i in range(500):
        m = i % 4
        if m == 0:
            out.append(i * 1e50)
        elif m == 1:
            out.append(-float(i))
        elif m == 2:
            out.append(i * 1e-50)
        else:
            out.append(math.sin(float(i)) * 1e10)
    return out


def corpus_subnormal():
    return [TINY] * 2000


CORPORA = {
    "small": corpus_small(), "signed": corpus_signed(), "cancellation": corpus_cancellation(),
    "kahan_trap": corpus_kahan_trap(), "mixed_scale": corpus_mixed_scale(), "subnormal": corpus_subnormal(),
}
# extra recipes used only by the Kulisch unit-test cases
RECIPES = dict(CORPORA)
RECIPES["cancellation_1e100"] = [1e100, 1.0, -1e100] * 1000
RECIPES["subnormal_1000"] = [TINY] * 1000


def case_inputs(case):
    """(keys, values) of a case; corpus-based cases are rebuilt from their recipe."""
    if "corpus" in case:
        xs = RECIPES[case["corpus"]]
        mod = case.get("keys_mod", 1)
        return [i % mod for i in range(len(xs))], list(xs)
    vals = [float.fromhex(v) if v not in ("nan", "inf", "-inf") else float(v) for v in case["values"]]
    return case.get("keys", [0] * len(vals)), vals


def main():
    g = {"source": "transcribed from the reference's tests; see `cite` of each case", "cases": []}
    add = g["cases"].append

    # ---- KulischAccumulator unit tests (kulisch_accumulator.rs:443-778)
    for x in [1.0, 3.14, -2.71, 1e100, 1e-100, 1024.0, 0.125, -7.5]:
        add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:449-460 single_value_roundtrip",
             "values": encl([x]), "expect": enc(x)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:463-471 ignores_zero_nan_inf",
         "values": encl([0.0, -0.0, math.nan, math.inf, -math.inf]), "expect": enc(0.0)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:474-480 integer_sum_is_exact",
         "values": encl([float(i) for i in range(1, 101)]), "expect": enc(5050.0)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:483-491 cancellation_recovery",
         "values": encl([1e17, 1.0, -1e17]), "expect": enc(1.0)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:494-503 large_cancellation_chain",
         "corpus": "cancellation_1e100", "expect": enc(1000.0)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:506-514 subnormal_accumulation",
         "corpus": "subnormal_1000", "expect": enc(1000.0 * TINY)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:517-525 sign_handling",
         "values": encl([5.0, -3.0, -10.0]), "expect": enc(-8.0)})
    add({"kind": "exact_sum", "cite": "kulisch_accumulator.rs:528-533 zero_result_from_exact_cancellation",
         "values": encl([1e50, -1e50]), "expect": enc(0.0)})
    add({"kind": "exact_sum_tol", "cite": "kulisch_accumulator.rs:561-574 beats_naive_sum_on_stress_input",
         "corpus": "kahan_trap", "expect": enc(1.0 + 10000 * 1e-10), "tol": 1e-15})

    # ---- determinism corpora: Kulisch oracle == correctly rounded exact sum
    for name, xs in CORPORA.items():
        add({"kind": "exact_sum", "cite": f"determinism_contract.rs:49-101 corpus_{name} (expect = fsum)",
             "corpus": name, "expect": enc(exact(xs))})
    xs = corpus_mixed_scale()
    keys7 = [i % 7 for i in range(len(xs))]
    keys8 = [i % 8 for i in range(len(xs))]
    for G, keys, cite in ((7, keys7, "determinism_contract.rs:219-245 run_to_run_stable_add_bykey"),
                          (8, keys8, "determinism_contract.rs:310-335 op_add_bykey_matches_kulisch_oracle")):
        want = [exact([x for x, k in zip(xs, keys) if k == gi]) for gi in range(G)]
        add({"kind": "scatter_phi", "cite": cite + " (expect = fsum per group)", "phi": "v", "keys_mod": G,
             "corpus": "mixed_scale", "n_groups": G, "expect": encl(want)})
    mask_rows = [i for i in range(len(xs)) if i % 3 == 0]
    mask = [0] * ((len(xs) + 63) // 64)
    for i in mask_rows:
        mask[i // 64] |= 1 << (i % 64)
    add({"kind": "scatter_phi_masked", "cite": "determinism_contract.rs:420-447 cpu_scatter_phi_masked_matches_kulisch_oracle",
         "phi": "v", "keys_mod": 1, "corpus": "mixed_scale", "mask": [str(w) for w in mask], "n_groups": 1,
         "expect": encl([exact([xs[i] for i in mask_rows])])})
    # idempotent ops: Max/Min over the corpora (determinism_contract.rs:223-262)
    for name, xs in CORPORA.items():
        fin = [x for x in xs if math.isfinite(x)]
        add({"kind": "extremum", "cite": f"determinism_contract.rs:252-278 Max/Min on corpus_{name}",
             "keys_mod": 1, "corpus": name, "n_groups": 1,
             "expect_min": encl([min(fin)]), "expect_max": encl([max(fin)])})

    # ---- ComputeEngine CPU tests (compute_engine.rs:866-1091)
    add({"kind": "scatter_phi", "cite": "compute_engine.rs:868-874 scatter_sum_cpu", "phi": "v",
         "keys": [0, 0, 1, 1, 2], "values": encl([1, 2, 3, 4, 5]), "n_groups": 3, "expect": encl([3, 7, 5])})
    add({"kind": "scatter_phi", "cite": "compute_engine.rs:877-883 scatter_sum_sq_cpu", "phi": "v * v",
         "keys": [0, 0, 1], "values": encl([3, 4, 5]), "n_groups": 2, "expect": encl([25, 25])})
    add({"kind": "scatter_phi", "cite": "compute_engine.rs:886-892 scatter_count_cpu", "phi": "1.0",
         "keys": [0, 0, 1, 2, 2, 2], "values": encl([0] * 6), "n_groups": 3, "expect": encl([2, 1, 3])})
    add({"kind": "scatter_phi", "cite": "compute_engine.rs:895-905 scatter_centered_cpu",
         "phi": "(v - r) * (v - r)", "keys": [0, 0, 1, 1], "values": encl([10, 20, 30, 40]),
         "refs": encl([15, 35]), "n_groups": 2, "expect": encl([50, 50])})
    add({"kind": "scatter_multi_phi", "cite": "compute_engine.rs:911-918 scatter_multi_sum_and_count_cpu",
         "phis": ["v", "1.0"], "keys": [0, 0, 1, 1, 2], "values": encl([1, 2, 3, 4, 5]), "n_groups": 3,
         "expect": [encl([3, 7, 5]), encl([2, 2, 1])]})
    add({"kind": "scatter_multi_phi", "cite": "compute_engine.rs:921-929 scatter_multi_three_phis_cpu",
         "phis": ["v", "v * v", "1.0"], "keys": [0, 0], "values": encl([3, 4]), "n_groups": 1,
         "expect": [encl([7]), encl([25]), encl([2])]})
    add({"kind": "scatter_phi_masked", "cite": "compute_engine.rs:1028-1037 scatter_masked_sum_cpu", "phi": "v",
         "keys": [0, 0, 1, 1, 2], "values": encl([1, 2, 3, 4, 5]), "mask": [str(0b10101)], "n_groups": 3,
         "expect": encl([1, 3, 5])})
    add({"kind": "scatter_phi_masked", "cite": "compute_engine.rs:1040-1047 scatter_masked_all_pass_cpu",
         "phi": "v", "keys": [0, 0, 1], "values": encl([1, 2, 3]), "mask": [str(0b111)], "n_groups": 2,
         "expect": encl([3, 3])})
    add({"kind": "scatter_phi_masked", "cite": "compute_engine.rs:1050-1057 scatter_masked_none_pass_cpu",
         "phi": "v", "keys": [0, 0, 1], "values": encl([1, 2, 3]), "mask": ["0"], "n_groups": 2,
         "expect": encl([0, 0])})
    add({"kind": "unsupported_phi", "cite": "compute_engine.rs:1077-1083 unsupported_scatter_phi_errors",
         "phi": "sin(v) * cos(r)"})

    # ---- ScatterEngine CPU tests (scatter_engine.rs:488-578)
    add({"kind": "scatter_phi", "cite": "scatter_engine.rs:500-506 scatter_phi_sum_sq", "phi": "v * v",
         "keys": [0, 0], "values": encl([2, 3]), "n_groups": 1, "expect": encl([13])})
    add({"kind": "scatter_phi", "cite": "scatter_engine.rs:509-519 scatter_phi_centered_sum", "phi": "v - r",
         "keys": [0, 0, 1], "values": encl([1, 3, 10]), "refs": encl([2, 10]), "n_groups": 2,
         "expect": encl([0, 0])})
    add({"kind": "scatter_phi", "cite": "scatter_engine.rs:522-529 scatter_phi_count", "phi": "1.0",
         "keys": [0, 0, 1, 1, 1], "values": encl([99] * 5), "n_groups": 2, "expect": encl([2, 3])})
    add({"kind": "scatter_phi", "cite": "scatter_engine.rs:532-540 scatter_phi_centered_sum_sq",
         "phi": "(v - r) * (v - r)", "keys": [0, 0], "values": encl([1, 5]), "refs": encl([3]), "n_groups": 1,
         "expect": encl([8])})
    add({"kind": "scatter_multi_phi", "cite": "scatter_engine.rs:545-566 multi_phi_sum_sq_count",
         "phis": ["v", "v * v", "1.0"], "keys": [0, 0, 1, 1, 2], "values": encl([1, 2, 3, 4, 5]), "n_groups": 3,
         "expect": [encl([3, 7, 5]), encl([5, 25, 25]), encl([2, 2, 1])]})

    # ---- DescriptiveEngine grouped tests (descriptive.rs:1634-1697)
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1635-1654 grouped_basic",
         "values": encl([1, 2, 3, 4, 5, 6]), "keys": [0, 0, 0, 1, 1, 1], "n_groups": 2,
         "expect": {"count": [3, 3], "mean": [2, 5], "var_pop": [2 / 3, 2 / 3], "min": [1, None],
                    "max": [3, None]}, "tol": 1e-10})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1657-1672 grouped_with_nan",
         "values": encl([1, math.nan, 3, 4, 5, math.nan]), "keys": [0, 0, 0, 1, 1, 1], "n_groups": 2,
         "expect": {"count": [2, 2], "mean": [2, 4.5]}, "tol": 1e-10})
    add({"kind": "mean_grouped", "cite": "descriptive.rs:1675-1682 grouped_mean_shortcut",
         "values": encl([10, 20, 30, 40]), "keys": [0, 1, 0, 1], "n_groups": 2, "expect": [20, 30],
         "tol": 1e-10})
    add({"kind": "moments_grouped_m34", "cite": "descriptive.rs:1685-1696 grouped_higher_moments",
         "values": encl([1, 2, 3, 4, 5, 10, 20, 30]), "keys": [0, 0, 0, 0, 0, 1, 1, 1], "n_groups": 2,
         "expect_g0": {"skew_biased": 0.0, "kurt_excess_biased": -1.3}, "tol": 1e-10})
    # ungrouped moments tests reused as a single group (descriptive.rs:1381-1480)
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1382-1393 moments_basic (one group)",
         "values": encl([1, 2, 3, 4, 5]), "keys": [0] * 5, "n_groups": 1,
         "expect": {"count": [5], "mean": [3], "min": [1], "max": [5], "var_pop": [2], "var_samp": [2.5]},
         "tol": 1e-10})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1442-1449 single_element (one group)",
         "values": encl([42]), "keys": [0], "n_groups": 1,
         "expect": {"count": [1], "mean": [42], "var_pop": [0.0], "var_samp": ["nan"]}, "tol": 1e-10})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1452-1458 all_same_values (one group)",
         "values": encl([7, 7, 7, 7]), "keys": [0] * 4, "n_groups": 1,
         "expect": {"mean": [7], "var_pop": [0.0]}, "tol": 1e-10})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1461-1467 nan_handling (one group)",
         "values": encl([1, math.nan, 3, math.nan, 5]), "keys": [0] * 5, "n_groups": 1,
         "expect": {"count": [3], "mean": [3], "min": [1], "max": [5]}, "tol": 1e-10})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1470-1474 all_nan (one group)",
         "values": encl([math.nan, math.nan]), "keys": [0, 0], "n_groups": 1,
         "expect": {"count": [0], "mean": ["nan"]}, "tol": 0})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1477-1481 inf_values (one group)",
         "values": encl([1, math.inf, 3]), "keys": [0] * 3, "n_groups": 1,
         "expect": {"count": [3], "max": ["inf"]}, "tol": 0})
    add({"kind": "moments_grouped", "cite": "descriptive.rs:1484-1494 two_elements (one group)",
         "values": encl([1, 3]), "keys": [0, 0], "n_groups": 1,
         "expect": {"mean": [2], "var_pop": [1], "var_samp": [2]}, "tol": 1e-10})

    # ---- AccumulateEngine ByKey tests (accumulate.rs:963-990, 1617-1690)
    add({"kind": "scatter_phi", "cite": "accumulate.rs:964-976 bykey_add_matches_scatter_sum", "phi": "v",
         "keys": [0, 0, 1, 1, 2], "values": encl([1, 2, 3, 4, 5]), "n_groups": 3, "expect": encl([3, 7, 5])})
    add({"kind": "extremum", "cite": "accumulate.rs:1610-1645 bykey_max_per_group / bykey_min_per_group",
         "keys": [0, 0, 0, 1, 1, 1, 2], "values": encl([3.0, 1.0, 4.0, 1.5, 9.0, 2.6, 5.0]), "n_groups": 3,
         "expect_min": encl([1.0, 1.5, 5.0]), "expect_max": encl([4.0, 9.0, 5.0])})
    add({"kind": "extremum", "cite": "accumulate.rs:1648-1667 bykey_max_min_single_element_groups",
         "keys": [0, 1, 2, 3], "values": encl([7.0, 3.0, 9.0, 1.0]), "n_groups": 4,
         "expect_min": encl([7.0, 3.0, 9.0, 1.0]), "expect_max": encl([7.0, 3.0, 9.0, 1.0])})
    add({"kind": "extremum", "cite": "accumulate.rs:1670-1698 ohlcv_high_low_via_max_min_scatter",
         "keys": [0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2],
         "values": encl([100, 105, 98, 102, 102, 108, 101, 106, 106, 107, 103, 104]), "n_groups": 3,
         "expect_min": encl([98, 101, 103]), "expect_max": encl([105, 108, 107])})

    # ---- cancellation canaries: variance at large offsets (gold_standard_parity.rs:5942-6000)
    for off in (1e4, 1e6, 1e8, 1e10, 1e12):
        vals = [off + i * 0.001 for i in range(100)]
        add({"kind": "moments_grouped", "cite": f"gold_standard_parity.rs:5939-5988 canary offset {off:g}",
             "values": encl(vals), "keys": [0] * 100, "n_groups": 1,
             "expect": {"var_pop": [(100 * 100 - 1) * 0.001 * 0.001 / 12.0]}, "tol": 0.01, "rel": True})

    # ---- FilterJit::filter_mask tests (filter_jit.rs:565-614): words as hex, `check` = asserted bits
    def fm(cite, pred, thr, vals, expect, check):
        add({"kind": "filter_mask", "cite": cite, "pred": pred, "threshold": enc(thr), "values": encl(vals),
             "expect": [hex(w) for w in expect], "check": [hex(c) for c in check]})
    fm("filter_jit.rs:565-575 filter_gt_threshold", "gt", 4.0, [1.0, 5.0, 3.0, 7.0, 2.0, 8.0], [0b101010], [0x3F])
    fm("filter_jit.rs:577-582 filter_all_pass", "gt", 0.0, [1.0, 2.0, 3.0, 4.0], [0xF], [0xF])
    fm("filter_jit.rs:585-590 filter_none_pass", "gt", 100.0, [1.0, 2.0, 3.0], [0], [0x7])
    fm("filter_jit.rs:593-602 filter_exactly_64_rows", "gt", 0.5, [0.0 if i % 2 == 0 else 1.0 for i in range(64)],
       [0xAAAAAAAAAAAAAAAA], [0xFFFFFFFFFFFFFFFF])
    fm("filter_jit.rs:605-614 filter_65_rows_two_words", "gt", 0.5, [1.0] * 65,
       [0xFFFFFFFFFFFFFFFF, 0x1], [0xFFFFFFFFFFFFFFFF, 0xFFFFFFFFFFFFFFFF])

    # ---- mask algebra (filter_jit.rs:616-628, 643-744; CPU and GPU variants assert the same values)
    def mw(xs):
        return [hex(x) for x in xs]
    for op, exp, cites in (("and", 0b0100, "643-646 cpu_mask_and / 688-693 gpu_mask_and"),
                           ("or", 0b0111, "649-652 cpu_mask_or / 695-700 gpu_mask_or"),
                           ("xor", 0b0011, "655-658 cpu_mask_xor / 702-707 gpu_mask_xor")):
        add({"kind": "mask_binary", "cite": f"filter_jit.rs:{cites}", "op": op,
             "a": mw([0b0101]), "b": mw([0b0110]), "expect": mw([exp])})
    add({"kind": "mask_not", "cite": "filter_jit.rs:661-664 cpu_mask_not_full_word",
         "a": mw([0xFFFFFFFFFFFFFFFF]), "n_rows": 64, "expect": mw([0])})
    add({"kind": "mask_not", "cite": "filter_jit.rs:667-673 cpu_mask_not_partial_last_word / 709-714 gpu",
         "a": mw([0b0101]), "n_rows": 4, "expect": mw([0b1010])})
    add({"kind": "mask_not", "cite": "filter_jit.rs:676-681 cpu_mask_not_trailing_bits_zeroed",
         "a": mw([0]), "n_rows": 4, "expect": mw([0b1111])})
    for n_rows, exp in ((128, 4), (66, 3), (6, 2)):
        add({"kind": "mask_popcount", "cite": f"filter_jit.rs:616-627 filter_mask_popcount n_rows={n_rows}",
             "mask": mw([0b0110, 0b1001]), "n_rows": n_rows, "expect": exp})
    add({"kind": "mask_popcount", "cite": "filter_jit.rs:717-724 gpu_mask_popcount_full_words",
         "mask": mw([0b0101, 0b1001]), "n_rows": 128, "expect": 4})
    add({"kind": "mask_popcount", "cite": "filter_jit.rs:727-734 gpu_mask_popcount_partial_last_word",
         "mask": mw([0xFFFFFFFFFFFFFFFF, 0b11]), "n_rows": 66, "expect": 66})
    add({"kind": "mask_and_popcount", "cite": "filter_jit.rs:737-744 gpu_mask_and_then_popcount",
         "a": mw([0b0101, 0b0101]), "b": mw([0b0110, 0b0110]), "n_rows": 128, "expect": 2})

    # ---- tile statistics (tb_io.rs:295-333 roundtrip_simple, :336-366 multi_tile_roundtrip):
    # global min / max / count / mean over the tiles' TileColumnStats (format.rs:141-175)
    add({"kind": "tile_stats_global", "cite": "tb_io.rs:295-333 roundtrip_simple",
         "values": encl([1.0, 2.0, 3.0, 4.0, 5.0]), "tile_rows": 65536, "n_tiles": 1,
         "expect": {"min": enc(1.0), "max": enc(5.0), "count": 5, "mean": enc(3.0)}, "tol": 1e-10})
    add({"kind": "tile_stats_global", "cite": "tb_io.rs:336-366 multi_tile_roundtrip", "arange": 10000,
         "tile_rows": 1024, "n_tiles": 10,
         "expect": {"min": enc(0.0), "max": enc(9999.0), "count": 10000, "mean": enc(4999.5)}, "tol": 0.01})

    OUT.write_text(json.dumps(g, indent=1))
    print(f"wrote {OUT} ({len(g['cases'])} cases)")


if __name__ == "__main__":
    main()
