"""The drop-in ``kernels.kda_kernel`` module on the host: import routing and the
dispatch's dtype and device rules (no kernel launches; runs without a GPU).

The reference's dispatch (``kernels/kda_kernel.py:303-328``) on an sm_100 GPU
sends ``use_triton=True`` calls to its Triton wrapper, which asserts fp16/bf16
before anything else (``:204``), and ``use_triton=False`` calls to its torch
loop, which takes fp32.  The drop-in keeps those rules; it has no CPU path.
"""
import sys

import pytest
import torch

import simpletrain_b200
from simpletrain_b200 import kda_kernel


def test_install_routes_the_reference_module_names():
    saved = {n: sys.modules.get(n) for n in ("kernels", "kernels.kda_kernel", "kernels.fused_ops")}
    try:
        simpletrain_b200.install()
        import kernels.fused_ops
        import kernels.kda_kernel
        assert kernels.kda_kernel is kda_kernel
        assert kernels.kda_kernel.kda_chunked_scan is kda_kernel.kda_chunked_scan
        assert kernels.fused_ops is simpletrain_b200.fused_ops
        from kernels.kda_kernel import kda_chunked_scan
        assert kda_chunked_scan is kda_kernel.kda_chunked_scan
    finally:
        for n, m in saved.items():
            if m is None:
                sys.modules.pop(n, None)
            else:
                sys.modules[n] = m


def test_fp32_with_triton_asserts_like_the_reference_wrapper():
    q = torch.randn(1, 1, 64, 64)
    with pytest.raises(AssertionError):
        kda_kernel.kda_chunked_scan(q, q, q, use_triton=True)
    with pytest.raises(AssertionError):
        kda_kernel.kda_chunked_scan_triton(q, q, q)


def test_host_tensors_raise_instead_of_falling_back():
    for dtype in (torch.float32, torch.bfloat16):
        q = torch.randn(1, 1, 64, 64).to(dtype)
        with pytest.raises(RuntimeError, match="CUDA"):
            kda_kernel.kda_chunked_scan(q, q, q, use_triton=False)
    q = torch.randn(1, 1, 64, 64).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        kda_kernel.kda_chunked_scan(q, q, q, use_triton=True)


def test_non_float_inputs_raise_type_error():
    q = torch.zeros(1, 1, 64, 64, dtype=torch.float64)
    with pytest.raises(TypeError):
        kda_kernel.kda_chunked_scan(q, q, q, use_triton=False)


def test_layer_reads_use_triton_from_its_config():
    from types import SimpleNamespace

    from simpletrain_b200.kda_layer import KDALayer, _use_triton
    assert _use_triton(KDALayer(64, 1, 64)) is True
    assert _use_triton(KDALayer(64, 1, 64, use_triton=False)) is False
    assert _use_triton(SimpleNamespace(cfg=SimpleNamespace(use_triton=False))) is False
