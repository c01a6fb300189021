"""The decode harness's bookkeeping (nanoquant_b200/harness.py) without a GPU: the reference's
row fields and metric definitions (src/nanoquant/kernel/test_decode.py:685, 781-803, 966-1003)."""
import csv

from nanoquant_b200 import harness


def test_row_and_aggregate_follow_reference_definitions(tmp_path):
    rows = [harness.make_row(i, "m", "", 2, 128, 33, tps, {"gpu_mem_peak_alloc_bytes": 10 + i}, "float16")
            for i, tps in enumerate((400.0, 600.0))]
    # decode loop tokens = batch * (new - 1); time = tokens / tps
    assert rows[0]["decode_tokens_total"] == 64 and rows[0]["decode_tokens_per_seq"] == 32
    assert abs(float(rows[0]["decode_time_s"]) - 64 / 400.0) < 1e-9
    assert rows[0]["decode_tps_per_seq"] == f"{200.0:.6f}"
    agg = harness.aggregate(rows)
    # aggregate tps = summed tokens / summed time (not the mean of the rates)
    assert abs(float(agg["decode_tps_total"]) - 128 / (64 / 400.0 + 64 / 600.0)) < 1e-3
    assert agg["gpu_mem_peak_alloc_bytes"] == "11" and agg["iter"] == "AVG"
    path = tmp_path / "d.csv"
    harness.write_csv(rows + [agg], str(path))
    with open(path) as f:
        r = list(csv.DictReader(f))
    assert list(r[0].keys()) == harness.ROW_FIELDS and len(r) == 3


def test_row_with_single_token_has_no_rate():
    row = harness.make_row(0, "m", "", 1, 8, 1, 0.0, {}, "float16")
    assert row["decode_tokens_total"] == 0 and row["decode_tps_total"] == ""
