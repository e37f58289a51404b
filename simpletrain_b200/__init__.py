"""B200-native (sm_100a) Kimi Delta Attention chunked scan for SimpleTrain.

Public API
----------
``kda_chunk(q, k, v, g, decay, initial_state, chunk_size, reference_exact,
output_final_state) -> (y, final_state)``
    the extended scan (initial / final state, tensor decay), differentiable.
``kda_chunked_scan(q, k, v, gate, decay, chunk_size, use_triton) -> y``
    SimpleTrain's own dispatch signature (``kernels/kda_kernel.py:303``).
``install()``
    make ``kernels.kda_kernel`` resolve to the drop-in module.
``device_status()``
    read device-side error bits (bounded waits that expired).
"""
from .ops import device_status, kda_chunk  # noqa: F401
from .kda_kernel import install, kda_chunked_scan  # noqa: F401

__all__ = ["kda_chunk", "kda_chunked_scan", "install", "device_status"]
