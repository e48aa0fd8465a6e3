"""CPU checks of bench.py's plumbing: the committed ncu summaries that the
bench line's `traffic` fields are read from parse, the defaults keep the
driver's no-flag run short, and the peaks come from the measured file when
it is there."""
import importlib
import json
import sys

import pytest

ROOT = __import__("pathlib").Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, str(ROOT))
    return importlib.import_module("bench")


def test_profile_summaries_give_traffic(bench):
    gemm = bench._profile_traffic(ROOT / "profiles" / "wgemm_gate_up_qwen3_4b_verify.md")
    attn = bench._profiled_traffic()
    # the gate/up launch streams its 99.6 MB weight once
    assert gemm is not None and 99_614_720 <= gemm < 1.1 * 100_425_728
    assert attn is not None and attn > 0


def test_missing_or_malformed_summary_gives_none(bench, tmp_path):
    assert bench._profile_traffic(tmp_path / "absent.md") is None
    f = tmp_path / "bad.md"
    f.write_text("traffic_bytes_per_launch: n/a\n")
    assert bench._profile_traffic(f) is None


def test_default_run_is_short(bench, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.gpus == 1 and a.workload == "decode" and a.impl == "ours"
    assert a.warmup >= 3 and 1 <= a.steps <= 5
    monkeypatch.setattr(sys, "argv", ["bench.py", "--kernel", "gemm"])
    k = bench.parse()
    assert k.warmup >= 3


def test_peaks_prefer_the_measured_file(bench):
    p = bench._peaks()
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        assert p["source"] == "measured" and p["hbm_gbs"] == float(d["hbm_gbs"])
    else:
        assert p["source"] == "fallback" and p["hbm_gbs"] == 6650.0
