"""f3s_probe_mma_sync: the throughput of the fused kernel's tensor-core
instruction on this GPU (the tensor-side roofline denominator)."""
import ctypes

import pytest
import torch

from fused3s_b200 import _lib

pytestmark = pytest.mark.gpu


def test_mma_sync_probe_reports_a_plausible_peak(lib):
    out = ctypes.c_double(0.0)
    assert lib.f3s_probe_mma_sync(16, 2048, out, torch.cuda.current_stream().cuda_stream) == _lib.F3S_SUCCESS
    # dense fp16 on a B200 is 2.25 PFLOP/s through tcgen05; the warp-level
    # instruction reaches a fraction of it, far above a latency-bound chain
    assert 100.0 < out.value < 2500.0, out.value
    assert lib.f3s_probe_mma_sync(0, 10, out, None) == _lib.F3S_ERR_INVALID_VALUE
