"""Bounded waits end instead of hanging, and say so.

Every wait in the tensor-core kernels (on an mbarrier for TMA data or MMA results, on another
CTA's hand-off flag) polls a bounded number of times; when the bound runs out the kernel sets a
bit in the workspace status word and carries on, so a lost hand-off shows up as a status the
host reads, never as a hung GPU. m3ssd_selftest_bounded_waits runs the same wait helpers against
an mbarrier nobody arrives at and a flag nobody sets. The test checks both bits, and that the
context still runs the operator correctly afterwards.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import cases
from oracle import ssd_oracle as O
from tolerances import TOL

pytestmark = pytest.mark.gpu

MMA_WAIT, FLAG_WAIT = 0x2, 0x4


def test_expired_waits_report_and_context_survives(cuda_device):
    from m3ssd import _lib
    import m3ssd
    lib = _lib.load()
    ws = torch.full((256,), 0xFF, dtype=torch.uint8, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert lib.m3ssd_selftest_bounded_waits(ctypes.c_void_p(ws.data_ptr()), 256, stream) == 0
    torch.cuda.synchronize(cuda_device)
    status = int(ws[:4].view(torch.int32).item())
    assert status == MMA_WAIT | FLAG_WAIT, hex(status)
    # argument checks (no device work)
    assert lib.m3ssd_selftest_bounded_waits(None, 256, stream) == 6
    assert lib.m3ssd_selftest_bounded_waits(ctypes.c_void_p(ws.data_ptr()), 64, stream) == 6
    # the context is intact: the tensor-core operator still matches the oracle
    inp, _, chunk = cases.make_case("block_small_raw")
    t = [torch.from_numpy(np.ascontiguousarray(inp[k])).to(cuda_device)
         for k in ("x", "A", "B_t", "C_t", "dt")]
    y = m3ssd.ssd_complex_chunkwise(*t, chunk_size=chunk).cpu().numpy()
    ref = O.ssd_naive(**inp).real
    assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < TOL["tensor"]["y_normwise"]
