"""Error figures used in parity reports (test infrastructure).

Three figures, because a plain per-element relative error is not meaningful near zero and even
the fp32 reference misses 1e-4 per element against an exact recurrence:

* ``normwise``   max|got - ref| / max|ref|
* ``floored``    max over elements of |got - ref| / max(|ref|, floor * max|ref|)  (floor 1e-3)
* ``allclose``   the reference tests' own criterion, |got - ref| <= atol + rtol |ref|
"""
from __future__ import annotations

import numpy as np

FLOOR = 1e-3


def _arr(a):
    a = np.asarray(a)
    if np.iscomplexobj(a):
        return a.astype(np.complex128)
    return a.astype(np.float64)


def normwise(got, ref, mask=None):
    g, r = _arr(got), _arr(ref)
    if mask is not None:
        g, r = g[mask], r[mask]
    if r.size == 0:
        return 0.0
    scale = np.max(np.abs(r))
    if scale == 0:
        return float(np.max(np.abs(g - r)))
    return float(np.max(np.abs(g - r)) / scale)


def floored(got, ref, floor=FLOOR, mask=None):
    g, r = _arr(got), _arr(ref)
    if mask is not None:
        g, r = g[mask], r[mask]
    if r.size == 0:
        return 0.0
    scale = np.max(np.abs(r))
    if scale == 0:
        return float(np.max(np.abs(g - r)))
    den = np.maximum(np.abs(r), floor * scale)
    return float(np.max(np.abs(g - r) / den))


def report(got, ref, mask=None):
    return {"normwise": normwise(got, ref, mask), "floored": floored(got, ref, mask=mask)}
