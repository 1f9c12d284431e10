"""The bench's own arithmetic and look-ups, on the CPU: the algorithmic byte
count of the roofline, the DRAM-traffic look-up in the committed profile
(every line it holds parses, each workload key is found, and a workload
without a capture gets None), and the command line's defaults."""
import importlib.util
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_bytes_of_c4(bench):
    # per head: K and V tiles of each block (64 d B), the Q tile and the fp32
    # O tile of each window (96 d B); plus 4 B per block and 8 B per window
    B, nrw = 15_777_732, 65_536
    assert bench.alg_bytes(8, 64, B, nrw) == 8 * (64 * 64 * B + 96 * 64 * nrw) + 4 * B + 8 * nrw
    assert bench.alg_bytes(8, 64, B, nrw) == 520_289_582_864  # the figure the C4 bench line reports
    assert bench.alg_flops(8, 64, B) == 1024 * 64 * 8 * B


def test_traffic_lookup_matches_the_profile(bench):
    text = (ROOT / "profiles" / "k_fused3s_dram_traffic.md").read_text()
    lines = [ln for ln in text.splitlines() if ln.startswith("dram_bytes_per_launch[")]
    assert lines, "the profile holds no machine-readable traffic lines"
    for ln in lines:
        key, value = ln.split("]:")
        config, heads, dim, split, order, hints = key[len("dram_bytes_per_launch["):].split(",")
        got = bench.ncu_traffic(config, int(heads[1:]), int(dim[1:]), split, order, hints[len("hints-"):])
        assert got == pytest.approx(float(value)), ln
    # C4 with the automatic plan: 408.27 GB read + 2.15 GB written
    assert bench.ncu_traffic("c4", 8, 64, "auto", "balanced", "on") == pytest.approx(4.1042062e11)
    # no capture of the full-size C5 launch: no traffic figure
    assert bench.ncu_traffic("c5", 4, 128, "auto", "balanced", "on") is None


def test_default_workload_is_the_largest_graph(bench):
    import argparse

    captured = {}

    def fake_parse(self, argv=None, namespace=None):
        captured["defaults"] = {a.dest: a.default for a in self._actions}
        raise SystemExit(0)

    orig = argparse.ArgumentParser.parse_args
    argparse.ArgumentParser.parse_args = fake_parse
    try:
        with pytest.raises(SystemExit):
            bench.main([])
    finally:
        argparse.ArgumentParser.parse_args = orig
    d = captured["defaults"]
    assert d["config"] == "c5" and d["gpus"] == 1 and d["warmup"] >= 3
