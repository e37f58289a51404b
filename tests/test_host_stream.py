"""HostScan argument checks (host side, no GPU needed: they raise before any CUDA call)."""
import pytest
import torch

from simpletrain_b200.host_stream import HostScan


def _t(*shape, dtype=torch.bfloat16):
    return torch.zeros(*shape, dtype=dtype)


def test_rejects_non_host_and_mismatched_inputs():
    scan = HostScan("cuda:0")
    q = _t(2, 2, 64, 64)
    with pytest.raises(ValueError, match="shape"):
        scan(q, _t(2, 2, 32, 64), q)
    with pytest.raises(ValueError, match="dtype"):
        scan(q, q, _t(2, 2, 64, 64, dtype=torch.float16))
    with pytest.raises(TypeError):
        scan(_t(2, 2, 64, 64, dtype=torch.float32), q, q)
    with pytest.raises(ValueError, match="initial_state"):
        scan(q, q, q, None, 0.9, initial_state=torch.zeros(2, 2, 64, 32))
    with pytest.raises(ValueError, match="outermost"):
        qt = _t(64, 2, 2, 64).permute(1, 2, 0, 3)   # batch not outermost in memory
        scan(qt, qt, qt)
    with pytest.raises(ValueError, match=r"\[B, H, T, D\]"):
        scan(_t(2, 64, 64), q, q)


def test_rejects_conflicting_semantics_and_non_cuda_device():
    with pytest.raises(ValueError):
        HostScan("cuda:0", per_step=True, reference_exact=True)
    with pytest.raises(RuntimeError):
        HostScan("cpu")
