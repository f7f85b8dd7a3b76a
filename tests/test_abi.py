"""C ABI checks that need no GPU: the library loads, exports every symbol include/m3ssd.h
declares, and its host-side validation returns the documented status codes."""
import ctypes
import os
import re

import pytest

from m3ssd import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "m3ssd.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(m3ssd_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def prob(**kw):
    d = dict(batch=2, seqlen=256, nheads=4, headdim=64, dstate=64, chunk=64, flags=0, reserved=0)
    d.update(kw)
    return _lib.Problem(**d)


def test_header_declares_the_expected_api():
    syms = declared_symbols()
    assert set(syms) == set(_lib.SIGNATURES), syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.m3ssd_abi_version() == 1


def test_strerror_covers_all_codes(lib):
    for code in list(_lib.STATUS_NAMES) + [999]:
        msg = lib.m3ssd_strerror(code).decode()
        assert msg
    assert lib.m3ssd_strerror(3).decode().startswith("m3ssd: chunk_size")


@pytest.mark.parametrize("kw,code", [
    (dict(), 0),
    (dict(chunk=0), 3), (dict(chunk=257), 3),
    (dict(headdim=257), 4), (dict(dstate=300), 4),
    (dict(batch=0), 2), (dict(seqlen=-1), 2), (dict(nheads=0), 2),
    (dict(flags=0x200), 9), (dict(flags=0x30), 9), (dict(reserved=1), 9),
    # bf16 y: tensor-core shapes only
    (dict(flags=0x100, headdim=64, dstate=64), 0), (dict(flags=0x100, headdim=32), 2),
    (dict(flags=0x100 | 0x10, headdim=64, dstate=64), 2),
    (dict(flags=0x100 | 0x1, headdim=64, dstate=64), 2),
    (dict(batch=70000, nheads=1), 2),
    (dict(seqlen=64 * 70000, chunk=64), 2),
    (dict(chunk=4, seqlen=20), 0), (dict(chunk=1, seqlen=3, headdim=1, dstate=1), 0),
])
def test_check_problem(lib, kw, code):
    assert lib.m3ssd_check_problem(ctypes.byref(prob(**kw))) == code


def test_sizes(lib):
    p = prob()
    nc = 256 // 64
    # tensor-core shape: chunk-entry states (fp32 [64][128] per chunk) + a 1824-byte decay record
    assert lib.m3ssd_states_bytes(ctypes.byref(p)) == (8 * 64 * 64 + 1824) * 2 * 4 * nc
    q = prob(headdim=32)  # fp32 path only: complex64 [D][N] per chunk
    assert lib.m3ssd_states_bytes(ctypes.byref(q)) == 8 * 2 * 4 * nc * 32 * 64
    assert lib.m3ssd_fwd_workspace_bytes(ctypes.byref(p)) > 0
    assert lib.m3ssd_bwd_workspace_bytes(ctypes.byref(p)) > 0
    bad = prob(chunk=0)
    assert lib.m3ssd_states_bytes(ctypes.byref(bad)) == 0
    assert lib.m3ssd_fwd_path(ctypes.byref(bad)) == b"invalid"


def test_long_few_sequences_run_as_chains(lib):
    """The block shape runs in one pass; a few long sequences (B4 L16384 with the two heads one of
    eight GPUs holds) run as chains (forward: records, first pass, segment chain, second pass;
    backward: carry pass, segment chain, end-state terms, backward, dA), and more scratch."""
    block = prob(batch=16, seqlen=2048, nheads=16)
    assert lib.m3ssd_launch_count(ctypes.byref(block), 0) == 2
    assert lib.m3ssd_launch_count(ctypes.byref(block), 1) == 2
    long_ = prob(batch=4, seqlen=16384, nheads=2)
    assert lib.m3ssd_launch_count(ctypes.byref(long_), 0) == 4
    assert lib.m3ssd_launch_count(ctypes.byref(long_), 1) == 5
    one_pass = 256 + 4 * 4 * 2 * 256  # status word, counter, one flag per chunk
    assert lib.m3ssd_fwd_workspace_bytes(ctypes.byref(long_)) > one_pass
    # the chained shapes of tests/test_proj_gpu.py
    for kw in (dict(batch=1, seqlen=4096, nheads=2), dict(batch=2, seqlen=4096, nheads=4)):
        p = prob(**kw)
        assert lib.m3ssd_launch_count(ctypes.byref(p), 0) == 4, kw
        assert lib.m3ssd_launch_count(ctypes.byref(p), 1) == 5, kw
    # the fp32 path has no chained form, and complex x runs as two one-pass real passes
    assert lib.m3ssd_launch_count(ctypes.byref(prob(batch=4, seqlen=16384, nheads=2, flags=0x11)),
                                  0) == lib.m3ssd_launch_count(ctypes.byref(prob(headdim=32)), 0)
    assert lib.m3ssd_launch_count(ctypes.byref(prob(batch=4, seqlen=16384, nheads=2, flags=0x1)),
                                  0) == 3


def test_null_arguments_rejected_before_any_device_work(lib):
    assert lib.m3ssd_fwd(None, None) == 1
    assert lib.m3ssd_bwd(None, None) == 1
    a = _lib.FwdArgs()
    a.prob = prob()
    assert lib.m3ssd_fwd(ctypes.byref(a), None) == 1
    a.prob = prob(chunk=0)
    assert lib.m3ssd_fwd(ctypes.byref(a), None) == 3
    b = _lib.BwdArgs()
    b.prob = prob()
    assert lib.m3ssd_bwd(ctypes.byref(b), None) == 1


def _fake_fwd_args(p, ptr=0x10000):
    """Args whose device pointers are non-null and aligned but never dereferenced: every case
    below is rejected by host-side validation before the library looks at the device."""
    a = _lib.FwdArgs()
    a.prob = p
    a.x = a.A = a.B = a.C = a.dt = a.y = a.states = a.workspace = ptr
    a.workspace_bytes = 1 << 30
    _contiguous_strides(a, p)
    return a


def _fake_bwd_args(p, ptr=0x10000):
    b = _lib.BwdArgs()
    b.prob = p
    b.x = b.A = b.B = b.C = b.dt = b.dy = b.states = ptr
    b.dx = b.dA = b.dB = b.dC = b.ddt = b.workspace = ptr
    b.workspace_bytes = 1 << 30
    _contiguous_strides(b, p)
    b.dy_strides = _lib.I64x4(*b.x_strides)
    return b


def _contiguous_strides(a, p):
    T, H, D, N = p.seqlen, p.nheads, p.headdim, p.dstate
    a.x_strides = _lib.I64x4(T * H * D, H * D, D, 1)
    a.b_strides = _lib.I64x4(T * H * N, H * N, N, 1)
    a.c_strides = _lib.I64x4(T * H * N, H * N, N, 1)
    a.dt_strides = _lib.I64x3(T * H, H, 1)


def test_state_carry_entry_points_validate_on_the_host(lib):
    assert lib.m3ssd_fwd_state(None, None, None, None) == 1
    assert lib.m3ssd_bwd_state(None, None, None, None, None) == 1
    # tensor-core shapes with T a multiple of 64 only
    for kw in (dict(headdim=32), dict(seqlen=100), dict(flags=0x1), dict(flags=0x10)):
        assert lib.m3ssd_fwd_state(ctypes.byref(_fake_fwd_args(prob(**kw))), None, None,
                                   None) == 2, kw
        assert lib.m3ssd_bwd_state(ctypes.byref(_fake_bwd_args(prob(**kw))), None, None, None,
                                   None) == 2, kw
    a = _lib.FwdArgs()
    a.prob = prob()
    assert lib.m3ssd_fwd_state(ctypes.byref(a), None, None, None) == 1
    # a final state without its gradient (or the reverse) is rejected
    b = _fake_bwd_args(prob())
    assert lib.m3ssd_bwd_state(ctypes.byref(b), 0x20000, None, None, None) == 1
    assert lib.m3ssd_bwd_state(ctypes.byref(b), None, 0x20000, None, None) == 1
    # state pointers are complex64: 8-byte aligned
    assert lib.m3ssd_fwd_state(ctypes.byref(_fake_fwd_args(prob())), 0x20004, None, None) == 5
    assert lib.m3ssd_bwd_state(ctypes.byref(b), None, None, 0x20004, None) == 5


def test_state_carry_cpu_tensors_raise_no_fallback():
    import torch
    from m3ssd import ssd_complex_chunkwise_state
    x = torch.randn(1, 64, 2, 64)
    A = torch.randn(2, dtype=torch.complex64)
    B = torch.randn(1, 64, 2, 64, dtype=torch.complex64)
    dt = torch.randn(1, 64, 2)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ssd_complex_chunkwise_state(x, A, B, B, dt)


def test_error_maps_to_runtime_error():
    with pytest.raises(RuntimeError, match="chunk_size"):
        _lib.check(3)
    _lib.check(0)


def test_cpu_tensors_raise_no_fallback():
    import torch
    from m3ssd import ssd_complex_chunkwise
    x = torch.randn(1, 8, 2, 4)
    A = torch.randn(2, dtype=torch.complex64)
    B = torch.randn(1, 8, 2, 4, dtype=torch.complex64)
    dt = torch.randn(1, 8, 2)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ssd_complex_chunkwise(x, A, B, B, dt, chunk_size=4)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="not found"):
        _lib.load(str(tmp_path / "libm3ssd.so"))


def test_complex_x_runs_as_two_tensor_core_passes(lib):
    """Complex x at head_dim = state_dim = 64 takes the tensor-core path as two real-x passes:
    states hold both passes' state tiles and one set of decay records, the forward launches the
    records kernel once and the forward kernel twice, the backward two backward passes and the dx
    interleave; precision fp32 keeps the CUDA-core path."""
    real = prob(batch=2, seqlen=300, nheads=3)
    cplx = prob(batch=2, seqlen=300, nheads=3, flags=_lib.M3SSD_X_COMPLEX)
    assert lib.m3ssd_fwd_path(ctypes.byref(cplx)) == b"tcgen05-bf16x2"
    chunks = 2 * 3 * 5
    h_tiles = chunks * 64 * 128 * 4
    recs = chunks * 1824
    assert lib.m3ssd_states_bytes(ctypes.byref(real)) >= h_tiles + recs
    assert lib.m3ssd_states_bytes(ctypes.byref(cplx)) >= 2 * h_tiles + recs
    assert lib.m3ssd_launch_count(ctypes.byref(cplx), 0) == 3
    assert lib.m3ssd_launch_count(ctypes.byref(cplx), 1) == 5
    # its backward workspace holds the two real dx parts
    dx_part = 2 * 300 * 3 * 64 * 4
    assert lib.m3ssd_bwd_workspace_bytes(ctypes.byref(cplx)) >= 2 * dx_part
    fp32 = prob(batch=2, seqlen=300, nheads=3, flags=_lib.M3SSD_X_COMPLEX | _lib.M3SSD_PREC_FP32)
    assert lib.m3ssd_fwd_path(ctypes.byref(fp32)) == b"simt-fp32"
    # the in_proj and state-carry entry points take real x only
    a = _lib.ProjFwdArgs()
    a.prob = cplx
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 2
    f = _lib.FwdArgs()
    f.prob = prob(batch=2, seqlen=256, nheads=3, flags=_lib.M3SSD_X_COMPLEX)
    assert lib.m3ssd_fwd_state(ctypes.byref(f), None, None, None) == 2
