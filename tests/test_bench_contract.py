"""The reference arm of ``bench.py`` (``--impl reference``) on the CPU: one JSON line with the bench
contract's keys, the same ``metric`` / ``unit`` / ``higher_is_better`` / ``config`` as the repo arm, whole
steps actually timed (``ms_per_step x steps`` matches the time it spent), ``e2e`` with no host copies, and
nothing printed by ranks other than 0. A tiny Llama shape stands in for the workload so the test is fast."""

import contextlib
import io
import json
import types

import pytest

import bench
from microgen_b200 import model_spec as MS

TINY = dict(family="llama", hidden=64, layers=3, heads=4, kv_heads=2, head_dim=16, inter=128, vocab=300, eps=1e-5,
            rope_theta=500000.0)


@pytest.fixture
def tiny_workload(monkeypatch):
    monkeypatch.setattr(MS, "TINY_BENCH", TINY, raising=False)
    monkeypatch.setitem(bench.WORKLOADS, "tiny", dict(shape="TINY_BENCH", batch=2, prompt=16, shared=0, decode=8))
    monkeypatch.setenv("MG_REFERENCE_BUDGET_S", "5")
    return "tiny"


def _run(args, rank="0", monkeypatch=None):
    monkeypatch.setenv("RANK", rank)
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        bench.run_reference(args)
    return out.getvalue()


def test_reference_arm_line(tiny_workload, monkeypatch):
    args = types.SimpleNamespace(workload=tiny_workload, gpus=1, steps=3, warmup=1)
    lines = [l for l in _run(args, "0", monkeypatch).splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "tokens/s"
    assert d["higher_is_better"] is True and d["vs_baseline"] is None
    assert d["config"] == bench.workload_config("tiny", bench.WORKLOADS["tiny"], 1)  # the repo arm's config
    assert 1 <= d["steps"] <= 3 and d["value"] > 0
    assert d["value"] == pytest.approx(2 / (d["ms_per_step"] / 1e3), rel=1e-3)     # batch / step time
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1
    assert f"{d['steps']} whole steps" in cb["sample"]


def test_reference_arm_other_ranks_print_nothing(tiny_workload, monkeypatch):
    args = types.SimpleNamespace(workload=tiny_workload, gpus=2, steps=3, warmup=1)
    assert _run(args, "1", monkeypatch) == ""
