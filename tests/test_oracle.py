"""Pin the CPU oracle against fixtures produced by the reference implementation itself.

The fixtures in tests/golden were written by tests/golden/make_golden.py from the reference's
models/ssd_complex.py:58-119 and its torch.autograd gradients. Entries where the reference is not
finite (the exp-then-mask overflow at models/ssd_complex.py:52 and :107) are skipped; the oracle
must be finite there.
"""
import os

import numpy as np
import pytest
import torch

from oracle import cases, metrics
from oracle import ssd_oracle as O
from oracle.ssd_torch_cpu import ssd_chunkwise_torch

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ALL = list(cases.CASES)


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def pick(g, name, key, a):
    a = np.asarray(a)
    if name in cases.SAMPLED_CASES:
        return a.reshape(-1)[g["idx_" + key]]
    return a


@pytest.mark.parametrize("name", ALL)
def test_inputs_regenerate(name):
    """The seeded generator reproduces the inputs the fixtures were made from."""
    inp, dy, chunk = cases.make_case(name)
    g = load(name)
    assert int(g["chunk"]) == chunk
    for k in ("x", "A", "B_t", "C_t", "dt"):
        a = inp[k]
        if np.iscomplexobj(a):
            s = [np.abs(a.real).astype(np.float64).sum(), np.abs(a.imag).astype(np.float64).sum()]
        else:
            s = [np.abs(a).astype(np.float64).sum(), 0.0]
        np.testing.assert_allclose(s, g["sum_" + k], rtol=1e-12)
        if name not in cases.SAMPLED_CASES:
            np.testing.assert_array_equal(a, g["in_" + k])


@pytest.mark.parametrize("name", ALL)
def test_chunkwise_oracle_matches_reference(name):
    inp, dy, chunk = cases.make_case(name)
    g = load(name)
    y = O.ssd_chunkwise(**inp, chunk_size=chunk)
    assert y.dtype == np.float32 and y.shape == inp["x"].shape[:3] + (inp["x"].shape[3],)
    assert np.isfinite(y).all(), "masked-before-exp oracle must stay finite"
    ref = g["y"]
    fin = np.isfinite(ref)
    assert metrics.normwise(pick(g, name, "y", y), ref, fin) < 5e-6


@pytest.mark.parametrize("name", ALL)
def test_torch_restatement_bit_identical_where_reference_finite(name):
    inp, dy, chunk = cases.make_case(name)
    g = load(name)
    xs = [torch.from_numpy(np.ascontiguousarray(inp[k])) for k in ("x", "A", "B_t", "C_t", "dt")]
    y = ssd_chunkwise_torch(*xs, chunk_size=chunk).numpy()
    ref = g["y"]
    fin = np.isfinite(ref)
    np.testing.assert_array_equal(pick(g, name, "y", y)[fin], ref[fin])
    assert np.isfinite(y).all()


@pytest.mark.parametrize("name", ALL)
def test_naive_fp64_matches_reference_and_chunkwise(name):
    inp, dy, chunk = cases.make_case(name)
    g = load(name)
    yn = O.ssd_naive(**inp).real
    ref = g["y"]
    fin = np.isfinite(ref)
    assert metrics.normwise(pick(g, name, "y", yn), ref, fin) < 5e-6
    y = O.ssd_chunkwise(**inp, chunk_size=chunk)
    assert metrics.normwise(y, yn) < 5e-6


@pytest.mark.parametrize("name", ALL)
def test_adjoint_gradients_match_reference_autograd(name):
    """The hand-derived adjoint (complex128) equals torch.autograd through the reference."""
    inp, dy, chunk = cases.make_case(name)
    g = load(name)
    grads = O.ssd_naive_grads(**inp, dy=dy)
    for key, got in zip(("dx", "dA", "dB", "dC", "ddt"), grads):
        ref = g[key]
        fin = np.isfinite(ref)
        if not fin.any():
            continue
        assert np.asarray(got).dtype.kind == np.asarray(ref).dtype.kind, key
        err = metrics.normwise(pick(g, name, key, got), ref, fin)
        assert err < 1e-5, (key, err)


def test_reference_overflow_is_reproduced_by_the_fixtures():
    """The literal-dt block case is where the reference returns NaN; the oracle does not."""
    g = load("cfg0_literal")
    assert float(g["nonfinite_y"]) > 0.5
    inp, dy, chunk = cases.make_case("cfg0_literal")
    assert np.isfinite(O.ssd_chunkwise(**inp, chunk_size=chunk)).all()


def test_metrics_floor():
    ref = np.array([1.0, 1e-6, -2.0])
    got = ref + np.array([1e-6, 1e-6, 0.0])
    assert metrics.normwise(got, ref) == pytest.approx(5e-7)
    # second entry is judged against the floor 1e-3 * max|ref| = 2e-3
    assert metrics.floored(got, ref) == pytest.approx(1e-6 / 2e-3)


def _small_state_case(seed=5, B=1, T=12, H=2, D=3, N=2):
    rng = np.random.default_rng(seed)
    inp = cases.ref_style_inputs(seed, B, T, H, D, N, complex_x=False)
    cshape = (B, H, N, D)
    s0 = rng.standard_normal(cshape) + 1j * rng.standard_normal(cshape)
    dsT = rng.standard_normal(cshape) + 1j * rng.standard_normal(cshape)
    dy = rng.standard_normal((B, T, H, D))
    return inp, s0, dsT, dy


def test_naive_state_carry_chains_segments():
    """The recurrence cut at t = 5 and restarted from the carried state is the same recurrence."""
    inp, s0, _, _ = _small_state_case()
    y, sT = O.ssd_naive(**inp, s0=s0, return_state=True)
    first = {k: (v if k == "A" else v[:, :5]) for k, v in inp.items()}
    rest = {k: (v if k == "A" else v[:, 5:]) for k, v in inp.items()}
    y1, s1 = O.ssd_naive(**first, s0=s0, return_state=True)
    y2, s2 = O.ssd_naive(**rest, s0=s1, return_state=True)
    np.testing.assert_allclose(np.concatenate([y1, y2], axis=1), y, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(s2, sT, rtol=1e-12, atol=1e-12)


def test_adjoint_state_gradients_match_finite_differences():
    """ds0 and the other gradients of L = sum(dy Re y) + Re sum(conj(dsT) s_T), checked by
    central differences of the fp64 recurrence (PyTorch's convention: dL/dRe + i dL/dIm)."""
    inp, s0, dsT, dy = _small_state_case()

    def loss(inp_, s0_):
        y, sT = O.ssd_naive(**inp_, s0=s0_, return_state=True)
        return float(np.sum(dy * y.real) + np.sum((np.conj(dsT) * sT).real))

    g = O.ssd_naive_grads(**inp, dy=dy, s0=s0, dsT=dsT)
    assert len(g) == 6
    eps = 1e-6
    idx = (0, 1, 1, 2)
    for part, unit in ((0, 1.0), (1, 1j)):
        sp, sm = s0.copy(), s0.copy()
        sp[idx] += eps * unit
        sm[idx] -= eps * unit
        fd = (loss(inp, sp) - loss(inp, sm)) / (2 * eps)
        got = g[5][idx].real if part == 0 else g[5][idx].imag
        assert abs(fd - got) < 1e-6 * max(1.0, abs(fd)), (part, fd, got)
    # dt at one position (real input), through the carried state as well
    dtp, dtm = dict(inp), dict(inp)
    dtp["dt"] = inp["dt"].astype(np.float64).copy()
    dtm["dt"] = inp["dt"].astype(np.float64).copy()
    dtp["dt"][0, 3, 1] += eps
    dtm["dt"][0, 3, 1] -= eps
    fd = (loss(dtp, s0) - loss(dtm, s0)) / (2 * eps)
    assert abs(fd - g[4][0, 3, 1]) < 1e-6 * max(1.0, abs(fd))


def test_chained_segments_algebra_matches_the_whole_sequence():
    """The decomposition the chained kernels run (tc_long.cu), on the fp64 recurrence: each
    segment from a zero state gives its end state L_s; S_{s+1} = D_s S_s + L_s with D_s the
    segment's total decay; every segment rerun from S_s gives the whole sequence's y. Backward:
    each segment's entry-state gradient P_s with a zero end gradient; dE_{s-1} = P_s +
    conj(D_s) dE_s; every segment rerun with its end gradient dE_s and entry state S_s gives the
    whole sequence's gradients (dA summed over segments)."""
    B, T, H, D, N, G = 1, 24, 2, 3, 2, 4
    inp = cases.ref_style_inputs(9, B, T, H, D, N, complex_x=False)
    rng = np.random.default_rng(9)
    dy = rng.standard_normal((B, T, H, D))
    seg = T // G

    def part(k):
        return {n: (v if n == "A" else v[:, k * seg:(k + 1) * seg]) for n, v in inp.items()}

    sp = O.softplus_f64(inp["dt"])
    A = np.asarray(inp["A"]).astype(np.complex128)
    Dk = [np.exp(np.sum(sp[:, k * seg:(k + 1) * seg] * A, axis=1))[:, :, None, None]
          for k in range(G)]                                              # (B, H, 1, 1)
    L = [O.ssd_naive(**part(k), return_state=True)[1] for k in range(G)]
    S = [np.zeros_like(L[0])]
    for k in range(G):
        S.append(Dk[k] * S[k] + L[k])
    y_full, s_full = O.ssd_naive(**inp, return_state=True)
    y_seg = np.concatenate([O.ssd_naive(**part(k), s0=S[k]) for k in range(G)], axis=1)
    np.testing.assert_allclose(y_seg, y_full, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(S[G], s_full, rtol=1e-12, atol=1e-12)

    full = O.ssd_naive_grads(**inp, dy=dy)
    zero = np.zeros_like(L[0])
    P = [O.ssd_naive_grads(**part(k), dy=dy[:, k * seg:(k + 1) * seg], s0=zero, dsT=zero)[5]
         for k in range(G)]
    dE = [None] * G
    dE[G - 1] = zero
    for k in range(G - 1, 0, -1):
        dE[k - 1] = P[k] + np.conj(Dk[k]) * dE[k]
    parts = [O.ssd_naive_grads(**part(k), dy=dy[:, k * seg:(k + 1) * seg], s0=S[k], dsT=dE[k])
             for k in range(G)]
    for i, name in enumerate(("dx", "dA", "dB", "dC", "ddt")):
        got = (sum(p[i] for p in parts) if name == "dA"
               else np.concatenate([p[i] for p in parts], axis=1))
        np.testing.assert_allclose(got, full[i], rtol=1e-10, atol=1e-12, err_msg=name)
