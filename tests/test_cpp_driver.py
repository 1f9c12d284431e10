"""The drop-in C++ boundary: a driver written like the reference's own v2
harness, against include/fused3s.hpp, compiled here and run on the GPU."""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import ROOT
from fused3s_b200 import graphs as G

CUDA_INC = "/usr/local/cuda/include"


def _nvcc():
    return shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def test_header_compiles_host_only():
    src = ROOT / "tests" / "cpp" / "f3s_v2_driver.cpp"
    for extra in ([], ["-DF3S_REFERENCE_TIE_ORDER"]):
        r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", f"-I{ROOT / 'include'}", f"-I{CUDA_INC}", *extra,
                            str(src)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def write_dataset(d: Path, g):
    d.mkdir(parents=True, exist_ok=True)
    (d / "meta.txt").write_text(f"{g.num_nodes} {g.num_edges}\n")
    np.savetxt(d / "row_ptr.txt", g.row_ptr, fmt="%d")
    np.savetxt(d / "col_idx.txt", g.col_ind, fmt="%d")


@pytest.mark.gpu
@pytest.mark.parametrize("config", ["c1", "c2"])
def test_cpp_driver_runs_like_the_reference_harness(lib, tmp_path, config):
    oracle.port()  # builds liboracle.so if needed
    exe = tmp_path / "f3s_v2_driver"
    cmd = [_nvcc(), "-std=c++17", "-O2", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "cpp" / "f3s_v2_driver.cpp"),
           f"-L{ROOT / 'fused3s_b200'}", "-lfused3s", f"-L{ROOT / 'oracle'}", "-loracle",
           f"-Xlinker=-rpath={ROOT / 'fused3s_b200'}", f"-Xlinker=-rpath={ROOT / 'oracle'}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    g = G.make_graph(config)
    write_dataset(tmp_path / config, g)
    r = subprocess.run([str(exe), str(tmp_path / config)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "SUCCESS" in r.stdout, r.stdout + r.stderr
