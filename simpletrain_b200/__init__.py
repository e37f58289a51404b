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
__all__ = ["kda_chunk", "kda_chunked_scan", "install", "device_status"]


def __getattr__(name):
    # loaded on first use, so that building (``python -m simpletrain_b200.build``)
    # does not need the built libraries
    if name in ("kda_chunk", "device_status"):
        from . import ops
        return getattr(ops, name)
    if name in ("install", "kda_chunked_scan"):
        from . import kda_kernel
        return getattr(kda_kernel, name)
    raise AttributeError(f"module 'simpletrain_b200' has no attribute {name!r}")
