"""Per-phase timing of the tensor-core kernels (measurement build only).

``python mamba-3-lite_b200/m3ssd/build.py --trace`` builds ``libm3ssd_trace.so``: the same kernels
with clock stamps at their phase boundaries (csrc/tc_trace.cuh; the default library has none).
``capture`` runs a callable with that library loaded and the stamp buffers armed, and
``summarize`` turns the stamps of one kernel into the median time of every phase boundary after
the start of a chunk ticket, over the tickets of the first 16 CTAs.
"""
from __future__ import annotations

import ctypes
import os

from . import _lib

TRACE_LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libm3ssd_trace.so")
CTAS, ITERS, SLOTS = 16, 64, 48  # kTraceCtas, kTraceIters, kTraceSlots of csrc/tc_trace.cuh

# stamp slots of k_bwd_tc (W: lane 0 of worker warp 0; C: the control lane; R: the hand-off warp)
BWD_PHASES = {
    0: "W ticket start", 1: "W C tile landed", 44: "W x, dy split stored", 45: "W staging free",
    2: "W x, dy, e dy written (opa)", 3: "W C conversion start", 46: "W C raw read",
    4: "W C' written (opc)", 5: "W B tile landed", 47: "W B raw read", 6: "W B' written (ops1)",
    7: "W H tile landed", 8: "W conj(H) written (oph)", 9: "W dS landed", 10: "W dS' written",
    11: "W MMA batch 1 done (G, dM, Q)", 40: "W epi1 rows 0-7 loaded", 41: "W epi1 rows 0-7 done",
    42: "W epi1 rows 8-15 loaded", 43: "W epi1 rows 8-15 done", 12: "W epilogue 1 done (ops2)",
    13: "W carry done", 14: "W carry published (ops3)", 15: "W dCa done (epilogue 2 start)",
    32: "W dC rows 0-7 loaded", 33: "W dC rows 0-7 done", 34: "W dC rows 8-15 loaded",
    35: "W dC rows 8-15 done", 16: "W dC staged", 17: "W dXa, dXb done", 18: "W dx staged",
    19: "W dBa, dBb done", 36: "W dB rows 0-7 loaded", 37: "W dB rows 0-7 done",
    38: "W dB rows 8-15 loaded", 39: "W dB rows 8-15 done", 20: "W dB staged",
    21: "C x, dy operands seen (dM issued)", 22: "C C' seen (Q issued)",
    23: "C B' seen (G issued)", 24: "C conj(H) seen (dCb issued)",
    25: "C epilogue 1 seen (dCa, dXa, dXb issued)", 26: "C carry seen (dBa issued)",
    27: "C dCa columns free (dBb issued)", 28: "C dC staged (stored)", 29: "C dB staged (stored)",
    30: "C next dS load issued", 31: "R d Sigma started",
}
# stamp slots of k_fwd_tc (lane 0 of warp 0, which also issues the MMAs; ctrl: warp 7)
FWD_PHASES = {
    0: "ticket start", 1: "B, C tiles landed", 2: "B raw read", 3: "B', x, x~ written, C read",
    4: "S~ issue point", 5: "C' written", 17: "G issue start", 6: "G issued", 7: "G done",
    19: "epilogue 1 loaded", 8: "epilogue 1 done", 9: "H_z loaded", 10: "conj(H) written",
    18: "Y issue start", 20: "Y1 issued", 11: "Y2 issued", 12: "state update done",
    16: "ctrl: H_{z+1} released", 13: "Y1, Y2 done", 14: "y staged",
}


def load():
    if not os.path.exists(TRACE_LIB):
        raise RuntimeError(f"{TRACE_LIB} not built: python mamba-3-lite_b200/m3ssd/build.py --trace")
    lib = _lib.load(TRACE_LIB)
    for name in ("m3ssd_trace_set_fwd", "m3ssd_trace_set_bwd"):
        getattr(lib, name).argtypes = [ctypes.c_void_p]
        getattr(lib, name).restype = ctypes.c_int
    return lib


def capture(fn, device, warmup=3):
    """Runs fn() `warmup` times, then once with the stamp buffers armed, all with the trace build
    loaded as the operator's library. Returns (fwd, bwd) stamp arrays [CTAS][ITERS][SLOTS]."""
    import torch
    lib = load()
    saved = _lib._lib
    _lib._lib = lib
    try:
        for _ in range(warmup):
            fn()
        bufs = [torch.zeros(CTAS * ITERS * SLOTS, dtype=torch.int64, device=device)
                for _ in range(2)]
        torch.cuda.synchronize(device)
        if lib.m3ssd_trace_set_fwd(bufs[0].data_ptr()) or lib.m3ssd_trace_set_bwd(bufs[1].data_ptr()):
            raise RuntimeError("could not arm the trace buffers")
        fn()
        torch.cuda.synchronize(device)
        lib.m3ssd_trace_set_fwd(None)
        lib.m3ssd_trace_set_bwd(None)
    finally:
        _lib._lib = saved
    return tuple(b.cpu().numpy().reshape(CTAS, ITERS, SLOTS) for b in bufs)


def summarize(stamps, names, sm_mhz):
    """Median (p10, p90) microseconds of each named stamp after its ticket's start, and the median
    ticket period, over every ticket of the traced CTAs but each CTA's first two and last two."""
    import numpy as np
    rows = []
    for c in range(stamps.shape[0]):
        its = [i for i in range(stamps.shape[1]) if stamps[c, i, 0] != 0]
        rows += [(c, i) for i in its[2:-2] if i + 1 < stamps.shape[1] and stamps[c, i + 1, 0]]
    if not rows:
        return {"tickets": 0}
    per = np.array([stamps[c, i + 1, 0] - stamps[c, i, 0] for c, i in rows]) / sm_mhz
    out = {"tickets": len(rows), "sm_mhz": sm_mhz,
           "ticket_period_us": float(np.median(per)), "phases": []}
    for s, name in names.items():
        v = np.array([stamps[c, i, s] - stamps[c, i, 0] for c, i in rows if stamps[c, i, s]])
        if len(v):
            v = v / sm_mhz
            out["phases"].append({"slot": s, "phase": name, "us": float(np.median(v)),
                                  "p10": float(np.percentile(v, 10)),
                                  "p90": float(np.percentile(v, 90))})
    out["phases"].sort(key=lambda d: d["us"])
    return out
