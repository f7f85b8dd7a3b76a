"""m3ssd: B200-native (sm_100a) complex chunkwise SSD operator, a drop-in for
models/ssd_complex.py:ssd_complex_chunkwise of atandra2000/Mamba-3-Lite.

    from m3ssd import ssd_complex_chunkwise
    y = ssd_complex_chunkwise(x, A, B_t, C_t, dt, chunk_size=64)   # CUDA tensors only
    y = ssd_from_proj(proj, A, n_heads, head_dim, state_dim)         # the block's in_proj output
    y, hT = ssd_complex_chunkwise_state(x, A, B_t, C_t, dt, h0)      # one segment, state carried

The compute runs in libm3ssd.so (C ABI in include/m3ssd.h); this package is the host-side
mirror of the reference's Python interface plus the autograd/torch.compile registration.
"""
from .ssd_complex import implementation, ssd_complex_chunkwise  # noqa: F401
from .ssd_proj import ssd_from_proj, unpack_proj, proj_width  # noqa: F401
from .ssd_state import ssd_complex_chunkwise_state  # noqa: F401
from ._lib import M3SsdError, load  # noqa: F401

__all__ = ["ssd_complex_chunkwise", "ssd_complex_chunkwise_state", "ssd_from_proj", "unpack_proj",
           "proj_width", "implementation", "M3SsdError", "load"]
