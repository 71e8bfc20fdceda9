"""adakv_b200: B200-native (sm_100a) AdaKV decode hot path.

Host-side mirror of the reference's operator interface (``adakv.attention``,
``adakv.runtime``, ``adakv.kernels.block_sparse_decode``, ``adakv.patch``)
over hand-written CUDA kernels reached through the C-ABI library
``libadakv_b200.so`` (declared in ``include/adakv_b200.h``).  There is no CPU
fallback: every operator raises if the library or a CUDA device is missing.
"""
__version__ = "0.1.0"
