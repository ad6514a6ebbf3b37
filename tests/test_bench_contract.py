"""Host logic of bench.py (no GPU): argument defaults per workload, the config block
and the clock-sample summary that rejects throttled runs."""
import sys

import pytest


@pytest.fixture()
def bench(monkeypatch):
    import bench as b
    return b


def _parse(bench, monkeypatch, argv):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    return bench.parse()


def test_defaults_per_workload(bench, monkeypatch):
    a = _parse(bench, monkeypatch, [])
    assert (a.gpus, a.steps, a.warmup, a.workload, a.impl) == (1, 300, 5, "verify_step", "native")
    assert (a.nodes, a.prefix) == (128, 3000)
    a = _parse(bench, monkeypatch, ["--workload", "frame_replay"])
    assert (a.steps, a.warmup, a.streams) == (2, 1, 16)
    a = _parse(bench, monkeypatch, ["--kernel-case", "config2", "--steps", "50"])
    assert (a.kernel_case, a.steps, a.warmup) == ("config2", 50, 5)
    a = _parse(bench, monkeypatch, ["--steps", "7", "--warmup", "3", "--gpus", "2"])
    assert (a.steps, a.warmup, a.gpus) == (7, 3, 2)


def test_config_block(bench):
    c = bench.config_block(1)
    assert c["workload"].startswith("config3:") and c["trie_nodes"] == 128 and c["prefix"] == 3000
    assert c["parallelism"] == "replicas1" and "l2" in c
    c = bench.config_block(4, 256, 4096)
    assert not c["workload"].startswith("config3") and c["parallelism"] == "replicas4"
    assert (c["trie_nodes"], c["prefix"]) == (256, 4096)


def test_clock_summary(bench, tmp_path):
    clk = bench.Clocks(0)
    clk.path = tmp_path / "clocks.csv"
    clk.proc = object()  # samples already written, as by a finished nvidia-smi
    clk.path.write_text(
        "0, 1800, 1965, 900.1, 0x4, Not Active, Not Active, Not Active, Active\n"
        "0, 1700, 1965, 980.3, 0x4, Not Active, Not Active, Not Active, Active\n"
        "0, 1900, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
        "garbage line\n")
    s = clk.summary()
    assert s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]
    clk.path.write_text("0, 900, 1965, 500.0, 0x8, Active, Not Active, Not Active, Not Active\n")
    assert clk.summary()["reasons"] == ["hw_slowdown"]
    clk.path.write_text("")
    assert clk.summary()["reasons"] == ["no samples"]
    clk.proc = None
    assert clk.summary()["reasons"] == ["nvidia-smi unavailable"]
