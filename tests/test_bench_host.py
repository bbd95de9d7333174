"""Host-side logic of bench.py that needs no GPU: the compact per-routine summary carried
on the final JSON line, and the pure helpers around it."""

import bench


def test_summary_fields_in_order():
    """[value, unit, roofline fraction, ms per call] first, then the optional extras in a
    fixed order: end-to-end value, exchange share, and the measured ceilings."""
    suite = {
        "spmv": {"value": 1956.54321, "unit": "GB/s", "roofline": {"frac": 0.29912}, "ms": 0.30061,
                 "e2e": {"value": 52.0712}, "gather_ceiling": {"spmv_frac_of_ceiling": 0.83219}},
        "spmv_t": {"value": 1449.4, "unit": "GB/s", "roofline": {"frac": 0.2218}, "ms": 0.4058,
                   "scatter_ceiling": {"spmv_t_frac_of_ceiling": 0.93311}},
        "spmm": {"value": 1083.4, "unit": "GB/s", "roofline": {"frac": 0.166}, "ms": 0.6244,
                 "row_gather_ceiling": {"spmm_frac_of_ceiling": 0.7194}},
        "spmv_dist": {"value": 2488.5, "unit": "GB/s", "roofline": {"frac": 0.19}, "ms": 0.2363,
                      "exchange_share": 0.17251},
    }
    out = bench.summarize(suite)
    assert out["spmv"] == [1956.5, "GB/s", 0.299, 0.3006, {"e2e": 52.07},
                           {"frac_of_gather_ceiling": 0.832}]
    assert out["spmv_t"] == [1449.4, "GB/s", 0.222, 0.4058, {"frac_of_scatter_ceiling": 0.933}]
    assert out["spmm"] == [1083.4, "GB/s", 0.166, 0.6244, {"frac_of_row_gather_ceiling": 0.719}]
    assert out["spmv_dist"] == [2488.5, "GB/s", 0.19, 0.2363, {"exchange_share": 0.173}]


def test_summary_errors_and_missing_fields():
    """A routine that failed is reported by its error (cut to 120 characters); missing
    roofline or time read as None; an empty suite gives no summary."""
    assert bench.summarize(None) is None
    assert bench.summarize({}) is None
    out = bench.summarize({"fft": {"error": "RuntimeError: " + "x" * 200},
                           "dgemm": {"value": 28.861, "unit": "TFLOP/s"}})
    assert out["fft"][0] == "error" and len(out["fft"][1]) == 120
    assert out["dgemm"] == [28.861, "TFLOP/s", None, None]
    # a routine whose host-buffer leg was skipped (--no-e2e, or N > 1) carries no e2e entry
    assert bench.summarize({"sgemm": {"value": 59.7, "unit": "TFLOP/s", "ms": 0.036,
                                      "e2e": None}})["sgemm"] == [59.7, "TFLOP/s", None, 0.036]
