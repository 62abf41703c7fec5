"""bench.py and the phase-trace summary, checked without a GPU.

* The reference arm prints exactly the config object of the repository arm
  for the same N (so the driver compares like with like) and says n_gpus 1;
* every workload class can describe itself without a device;
* forgert_b200.phase_trace.summarise attributes records to launches by the
  launch ordinal each CTA stamped, even when launches overlap in time.
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from forgert_b200 import phase_trace as P  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 8])
def test_reference_arm_config_equals_ours(world):
    ours = bench.cfg3_config(world, 28)
    assert ours["parallelism"].startswith(f"{world} GPU")
    # the reference arm builds its config with the same function and arguments
    src = (ROOT / "bench.py").read_text()
    assert '"impl": "reference", "config": cfg3_config(world, args.layers)' in src
    assert json.loads(json.dumps(ours)) == ours


def test_reference_arm_line_small_sample(monkeypatch):
    """One tiny step of the reference arm: the same config, n_gpus 1."""
    lines = []
    monkeypatch.setattr(bench, "emit", lines.append)
    tiny = [(np.zeros((28, 128), np.float32), np.zeros((n, 4, 128), np.float32),
             np.zeros((n, 4, 128), np.float32), n) for n in (64, 130, 7, 1)]
    monkeypatch.setattr(bench, "_cfg3_host_calls", lambda max_seqs=None: tiny)
    args = bench.parse_args(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    bench.run_reference(args, 0, 4)
    line = lines[-1]
    assert line["impl"] == "reference" and line["n_gpus"] == 1
    assert line["config"] == bench.cfg3_config(4, 28)
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["cpu"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["value"] > 0


def test_cpu_model_named():
    assert isinstance(bench.cpu_model(), str) and bench.cpu_model()


def test_phase_trace_summary_separates_overlapping_launches():
    rec = np.dtype([("t", "<u8"), ("launch", "<u4"), ("ev_sm", "<u4")])
    per_cta = {}
    # 4 launches, 2 CTAs; launch k+1 starts before launch k's CTAs finish
    for c in range(2):
        rows = []
        for k in range(4):
            t0 = 1000 * k + 10 * c
            rows += [(t0, k, 1), (t0 + 1500, k, 4), (t0 + 1900, k, 9)]
        per_cta[c] = np.array(sorted(rows), dtype=rec)
    out = P.summarise(per_cta)
    assert out["launches"] == 2                    # the window's edge launches are dropped
    assert out["period_us_median"] == 1.0
    assert out["dep_wait"]["median_cta_us"] == pytest.approx(1.505)
    assert out["stored"]["latest_cta_us"] == pytest.approx(1.91)


def test_phase_trace_reads_nonzero_records_in_time_order():
    """The trace buffer is zeroed before a run: records_by_cta keeps the
    non-empty records of each CTA, sorted by time, and drops idle CTAs."""
    raw = np.zeros((3, 8), dtype=P.REC)
    raw[0][[5, 1]] = [(300, 7, 4), (100, 7, 1)]     # written out of order
    raw[2][[0]] = [(50, 9, 1)]
    out = P.records_by_cta(raw)
    assert sorted(out) == [0, 2]
    assert list(out[0]["t"]) == [100, 300] and list(out[0]["launch"]) == [7, 7]
    assert list(out[2]["ev_sm"]) == [1]


def test_e2e_pipelines_only_per_layer_workloads():
    """The end-to-end leg overlaps host copies with the calls only for
    workloads that expose one call per layer; the paged workload (one call
    per step) keeps the serial copies."""
    assert callable(getattr(bench.Cfg3, "run_layer", None))
    assert getattr(bench.Cfg3Paged, "run_layer", None) is None
