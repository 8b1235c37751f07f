"""ctypes binding of the CPU oracle (oracle.cpp) — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, and only as the checker / the timed CPU baseline. The product never
imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
TRACE_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int, ctypes.c_void_p)
SEGMENT_FN = ctypes.CFUNCTYPE(ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, _f32p,
                              ctypes.c_void_p)

_lib = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        L = _lib
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_create.restype = ctypes.c_void_p
        L.orc_create.argtypes = [ctypes.c_int]
        L.orc_destroy.argtypes = [ctypes.c_void_p]
        L.orc_set.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int]
        L.orc_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int, _f32p,
                                  TRACE_FN, ctypes.c_void_p]
        L.orc_threads.argtypes = [ctypes.c_int]
        L.orc_gelu.restype = ctypes.c_float
        L.orc_gelu.argtypes = [ctypes.c_float]
        L.orc_std_unbiased.restype = ctypes.c_float
        L.orc_scan_norm.argtypes = [_f32p, ctypes.c_int, ctypes.c_int64, _f32p, _f32p]
        L.orc_separate.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_double, ctypes.c_double, ctypes.c_int, SEGMENT_FN,
                                   ctypes.c_void_p, _f32p]
        L.orc_transition_weight.argtypes = [ctypes.c_int, ctypes.c_double, _f32p]
        L.orc_center_trim.argtypes = [_f32p, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.orc_shift_randint.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64,
                                        ctypes.POINTER(ctypes.c_uint64)]
        L.orc_pos2d.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p]
        L.orc_pos1d.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float, _f32p]
        L.orc_attention_head.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_float, _f32p]
    return _lib


def ptr(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def threads(n: int = 0) -> int:
    return lib().orc_threads(n)


class OracleModel:
    """The reference's host forward on one set of weights."""

    def __init__(self, weights, segment: int = 343980):
        L = lib()
        self._h = L.orc_create(segment)
        self.segment = segment
        for name, value in weights.items():
            value = np.ascontiguousarray(value, dtype=np.float32)
            shape = (ctypes.c_int64 * value.ndim)(*value.shape)
            L.orc_set(self._h, name.encode(), ptr(value), shape, value.ndim)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_destroy(self._h)
            self._h = None

    def forward(self, mix, trace=None):
        """mix (B, 2, length<=segment) -> (B, 4, 2, length). ``trace`` is a
        dict filled with named intermediates (reference layouts)."""
        mix = np.ascontiguousarray(mix, dtype=np.float32)
        B, C, length = mix.shape
        out = np.empty((B, 4, C, length), dtype=np.float32)
        cb = TRACE_FN(0)
        if trace is not None:
            def _record(name, data, shape, ndim, _user):
                dims = tuple(shape[i] for i in range(ndim))
                trace[name.decode()] = np.ctypeslib.as_array(data, shape=dims).copy()
            cb = TRACE_FN(_record)
        rc = lib().orc_forward(self._h, ptr(mix), B, length, ptr(out), cb, None)
        if rc:
            raise RuntimeError(lib().orc_last_error().decode())
        return out

    def separate(self, mix, shifts=1, overlap=0.25, transition_power=1.0, batch=1,
                 forward=None):
        """Whole-track separation of a raw (2, length) mix -> (4, 2, length).
        ``forward(padded (G, 2, seg)) -> (G, 4, 2, seg)`` replaces the oracle's
        own forward (identity mocks, or the CUDA path under test)."""
        mix = np.ascontiguousarray(mix, dtype=np.float32)
        length = mix.shape[1]
        stems = np.empty((4, 2, length), dtype=np.float32)
        fwd = forward or self.forward
        error = []

        def _segment(padded, group, seg, out, _user):
            try:
                x = np.ctypeslib.as_array(padded, shape=(group, 2, seg)).copy()
                y = np.ascontiguousarray(fwd(x), dtype=np.float32)
                np.ctypeslib.as_array(out, shape=(group, 4, 2, seg))[...] = y
                return 0
            except Exception as exc:  # pragma: no cover - surfaced below
                error.append(exc)
                return 1

        cb = SEGMENT_FN(_segment)
        rc = lib().orc_separate(ptr(mix), length, self.segment, shifts, overlap,
                                transition_power, batch, cb, None, ptr(stems))
        if error:
            raise error[0]
        if rc:
            raise RuntimeError(lib().orc_last_error().decode())
        return stems


def separate_with(forward, mix, segment, shifts=0, overlap=0.25, transition_power=1.0, batch=1):
    """The driver alone, over an arbitrary segment forward (no weights)."""
    m = OracleModel({}, segment)
    return m.separate(mix, shifts=shifts, overlap=overlap, transition_power=transition_power,
                      batch=batch, forward=forward)


def bag_forward(forwards, weights, requested=None):
    """BagCombineForward::start (api.rs:319-361) over per-network segment
    forwards: returns a forward ``padded (G, 2, seg) -> (G, 4, 2, seg)``.

    A network runs only if it carries a nonzero weight on a requested source
    (api.rs:330-337); per source the combination starts from zeros, adds each
    running network's lane times its weight (f32 product, then f32 sum) in bag
    order, and divides by the f32 sum of those weights (api.rs:338-360);
    sources that are not requested stay zero. ``requested`` is a sequence of
    source indices (None = all four)."""
    w = np.asarray(weights, dtype=np.float32)
    sources = w.shape[1]
    req = [requested is None or s in requested for s in range(sources)]

    def forward(padded):
        batch, channels, time = padded.shape
        combined = np.zeros((batch, sources, channels, time), dtype=np.float32)
        totals = [np.float32(0.0)] * sources
        for k, fwd in enumerate(forwards):
            if not any(w[k, s] != 0 and req[s] for s in range(sources)):
                continue
            out = np.asarray(fwd(padded), dtype=np.float32)
            for s in range(sources):
                if w[k, s] == 0 or not req[s]:
                    continue
                combined[:, s] += out[:, s] * w[k, s]
                totals[s] = np.float32(totals[s] + w[k, s])
        for s in range(sources):
            if not req[s]:
                continue
            if totals[s] == 0:
                raise ValueError(f"no network covers stem index {s}")
            combined[:, s] /= totals[s]
        return combined

    return forward
