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
