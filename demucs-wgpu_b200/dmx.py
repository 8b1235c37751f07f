"""ctypes binding of libdmx_cuda.so (include/dmx.h).

The binding is a thin mirror of the C ABI; it never falls back to anything:
if the library is missing or fails to load, every call raises.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdmx_cuda.so")
SEGMENT = 343980

FP32, TF32, BF16, TF32X3 = 0, 1, 2, 3

# The symbols include/dmx.h declares, in order.
EXPORTS = (
    "dmx_default_config", "dmx_create", "dmx_destroy", "dmx_last_error", "dmx_forward_start",
    "dmx_forward_collect", "dmx_forward_device", "dmx_separate_track",
    "dmx_separate_track_device", "dmx_normalize_track_device", "dmx_normalize_track_noalloc",
    "dmx_bag_combine_device", "dmx_bag_forward_device", "dmx_separate_track_bag",
    "dmx_separate_track_bag_device", "dmx_separate_batch", "dmx_separate_batch_device",
    "dmx_separate_track_emit", "dmx_selftest_wait_timeout", "dmx_separate_track_multi",
    "dmx_num_chunks", "dmx_track_finish", "dmx_track_shard", "dmx_set_trace",
    "dmx_set_stage_timing", "dmx_stage_times", "dmx_kernel_launches", "dmx_stream",
    "dmx_synchronize", "dmx_read_tensor", "dmx_shift_offsets", "dmx_ipc_export", "dmx_ipc_open",
    "dmx_ipc_close", "dmx_rows_copy", "dmx_rows_add", "dmx_separate_track_windowed",
)

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
TRACE_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, _f32p, _i64p, ctypes.c_int, ctypes.c_void_p)
PROGRESS_FN = ctypes.CFUNCTYPE(None, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p)
FRAMES_FN = ctypes.CFUNCTYPE(None, ctypes.c_int64, ctypes.c_int64, _f32p, ctypes.c_void_p)
READ_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _f32p, _f32p,
                           ctypes.c_void_p)


class Config(ctypes.Structure):
    _fields_ = [("sources", ctypes.c_int), ("audio_channels", ctypes.c_int),
                ("samplerate", ctypes.c_int), ("segment_samples", ctypes.c_int),
                ("precision", ctypes.c_int), ("max_batch", ctypes.c_int)]


class SeparateOpts(ctypes.Structure):
    _fields_ = [("shifts", ctypes.c_int), ("overlap", ctypes.c_double),
                ("transition_power", ctypes.c_double), ("batch", ctypes.c_int),
                ("segment", ctypes.c_double)]


class DmxError(RuntimeError):
    def __init__(self, code, message):
        super().__init__(f"dmx error {code}: {message}")
        self.code = code


_lib = None

CLI_PATH = os.path.join(HERE, "dmx")


def cli_path():
    """Path of the ``dmx`` command-line tool (built by build.py beside the library)."""
    if not os.path.exists(CLI_PATH):
        raise ImportError(f"{CLI_PATH} is not built; run demucs-wgpu_b200/build.py")
    return CLI_PATH


def lib():
    """Load libdmx_cuda.so (raises if it is absent: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run demucs-wgpu_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        L.dmx_default_config.argtypes = [ctypes.POINTER(Config)]
        L.dmx_create.argtypes = [ctypes.POINTER(Config), ctypes.c_void_p, ctypes.c_size_t,
                                 ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        L.dmx_destroy.argtypes = [ctypes.c_void_p]
        L.dmx_last_error.restype = ctypes.c_char_p
        L.dmx_forward_start.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int64,
                                        ctypes.POINTER(ctypes.c_void_p)]
        L.dmx_forward_collect.argtypes = [ctypes.c_void_p, _f32p]
        L.dmx_forward_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                         ctypes.c_void_p, ctypes.c_void_p]
        L.dmx_separate_track.argtypes = [ctypes.c_void_p, _f32p, _f32p, ctypes.c_int64,
                                         ctypes.POINTER(SeparateOpts), _f32p, PROGRESS_FN,
                                         ctypes.c_void_p]
        L.dmx_separate_track_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                                ctypes.POINTER(SeparateOpts), ctypes.c_void_p,
                                                PROGRESS_FN, ctypes.c_void_p]
        L.dmx_normalize_track_device.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                                 ctypes.c_void_p, ctypes.c_void_p]
        L.dmx_normalize_track_noalloc.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                                  ctypes.c_void_p, ctypes.c_void_p]
        _hpp = ctypes.POINTER(ctypes.c_void_p)
        _ip = ctypes.POINTER(ctypes.c_int)
        L.dmx_bag_combine_device.argtypes = [_hpp, ctypes.c_int, _f32p, _ip, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        L.dmx_bag_forward_device.argtypes = [_hpp, ctypes.c_int, _f32p, _ip, ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.c_void_p]
        L.dmx_separate_track_bag.argtypes = [_hpp, ctypes.c_int, _f32p, _ip, _f32p, _f32p,
                                             ctypes.c_int64, ctypes.POINTER(SeparateOpts), _f32p,
                                             PROGRESS_FN, ctypes.c_void_p]
        L.dmx_separate_track_bag_device.argtypes = [_hpp, ctypes.c_int, _f32p, _ip,
                                                    ctypes.c_void_p, ctypes.c_int64,
                                                    ctypes.POINTER(SeparateOpts), ctypes.c_void_p,
                                                    PROGRESS_FN, ctypes.c_void_p]
        L.dmx_separate_track_emit.argtypes = [ctypes.c_void_p, _f32p, _f32p, ctypes.c_int64,
                                              ctypes.POINTER(SeparateOpts), FRAMES_FN,
                                              PROGRESS_FN, ctypes.c_void_p]
        L.dmx_separate_track_windowed.argtypes = [ctypes.c_void_p, READ_FN, ctypes.c_int64,
                                                  ctypes.POINTER(SeparateOpts), FRAMES_FN,
                                                  PROGRESS_FN, ctypes.c_void_p]
        _f32pp = ctypes.POINTER(_f32p)
        L.dmx_separate_batch.argtypes = [ctypes.c_void_p, _f32pp, _f32pp, _i64p, ctypes.c_int,
                                         ctypes.POINTER(SeparateOpts), _f32pp, PROGRESS_FN,
                                         ctypes.c_void_p]
        L.dmx_separate_batch_device.argtypes = [ctypes.c_void_p, _hpp, _i64p, ctypes.c_int,
                                                ctypes.POINTER(SeparateOpts), _hpp, PROGRESS_FN,
                                                ctypes.c_void_p]
        L.dmx_track_finish.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_double,
                                       ctypes.c_double, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]
        L.dmx_read_tensor.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, _f32p,
                                      ctypes.c_int64, _i64p, ctypes.POINTER(ctypes.c_int)]
        L.dmx_shift_offsets.argtypes = [ctypes.c_int, ctypes.c_int64, _i64p]
        L.dmx_ipc_export.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, _i64p]
        L.dmx_ipc_open.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                   ctypes.POINTER(ctypes.c_void_p)]
        L.dmx_ipc_close.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_int64]
        for name in ("dmx_rows_copy", "dmx_rows_add"):
            getattr(L, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                         ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_int64]
        L.dmx_set_stage_timing.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.dmx_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.dmx_separate_track_multi.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                               _f32p, _f32p, ctypes.c_int64,
                                               ctypes.POINTER(SeparateOpts), _f32p]
        L.dmx_stream.restype = ctypes.c_void_p
        L.dmx_stream.argtypes = [ctypes.c_void_p]
        L.dmx_synchronize.argtypes = [ctypes.c_void_p]
        L.dmx_num_chunks.restype = ctypes.c_int64
        L.dmx_num_chunks.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_double]
        L.dmx_track_shard.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_double, ctypes.c_double, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_int64, ctypes.c_int64]
        L.dmx_set_trace.argtypes = [ctypes.c_void_p, TRACE_FN, ctypes.c_void_p]
        L.dmx_stage_times.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_char_p), _f32p,
                                      ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double),
                                      ctypes.POINTER(ctypes.c_double), ctypes.c_int]
        L.dmx_kernel_launches.restype = ctypes.c_int64
        L.dmx_kernel_launches.argtypes = [ctypes.c_void_p]
        _lib = L
    return _lib


def _opts(shifts=1, overlap=0.25, transition_power=1.0, batch=0, segment=0.0):
    """dmx_separate_opts (SeparateOptions, pipeline.rs:17-38); ``segment`` in
    seconds, 0 = the model's."""
    return SeparateOpts(shifts, overlap, transition_power, batch, segment or 0.0)


def _check(rc):
    if rc != 0:
        raise DmxError(rc, lib().dmx_last_error().decode())


def _ptr(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def default_config():
    c = Config()
    lib().dmx_default_config(ctypes.byref(c))
    return c


class Handle:
    """One loaded network on one GPU (dmx_create / dmx_destroy)."""

    def __init__(self, blob: bytes, device: int = 0, precision: int = FP32, max_batch: int = 8):
        L = lib()
        cfg = default_config()
        cfg.precision = precision
        cfg.max_batch = max_batch
        self._blob = blob
        buf = ctypes.create_string_buffer(blob, len(blob))
        self._buf = buf
        h = ctypes.c_void_p()
        _check(L.dmx_create(ctypes.byref(cfg), ctypes.cast(buf, ctypes.c_void_p), len(blob),
                            device, ctypes.byref(h)))
        self._h = h
        self._destroy = L.dmx_destroy  # kept: module globals may be gone at interpreter exit
        self.device = device
        self.max_batch = max_batch
        self._trace_cb = None

    def close(self):
        if getattr(self, "_h", None):
            self._destroy(self._h)
            self._h = None

    __del__ = close

    # SegmentForward.start / collect
    def forward_start(self, mix):
        mix = np.ascontiguousarray(mix, dtype=np.float32)
        assert mix.ndim == 3 and mix.shape[1:] == (2, SEGMENT), mix.shape
        pending = ctypes.c_void_p()
        _check(lib().dmx_forward_start(self._h, _ptr(mix), mix.shape[0], ctypes.byref(pending)))
        return pending, mix.shape[0]

    def forward_collect(self, pending):
        p, n = pending
        out = np.empty((n, 4, 2, SEGMENT), dtype=np.float32)
        _check(lib().dmx_forward_collect(p, _ptr(out)))
        return out

    def forward(self, mix):
        return self.forward_collect(self.forward_start(mix))

    def forward_device(self, mix_ptr: int, n: int, out_ptr: int, stream: int = 0):
        _check(lib().dmx_forward_device(self._h, ctypes.c_void_p(mix_ptr), n,
                                        ctypes.c_void_p(out_ptr), ctypes.c_void_p(stream)))

    def separate_track(self, left, right, shifts=1, overlap=0.25, transition_power=1.0,
                       batch=0, progress=None, out=None, segment=0.0):
        """Whole-track separation of host arrays; ``out`` (4, 2, n) float32 may
        be supplied (e.g. pinned memory) to avoid a fresh allocation."""
        left = np.ascontiguousarray(left, dtype=np.float32)
        right = np.ascontiguousarray(right, dtype=np.float32)
        n = left.shape[0]
        stems = np.empty((4, 2, n), dtype=np.float32) if out is None else out
        assert stems.shape == (4, 2, n) and stems.dtype == np.float32 and stems.flags.c_contiguous
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        cb = PROGRESS_FN(0) if progress is None else PROGRESS_FN(lambda d, t, _u: progress(d, t))
        _check(lib().dmx_separate_track(self._h, _ptr(left), _ptr(right), n, ctypes.byref(opts),
                                        _ptr(stems), cb, None))
        return stems

    def separate_track_emit(self, left, right, on_frames, shifts=1, overlap=0.25,
                            transition_power=1.0, batch=0, progress=None, segment=0.0):
        """Demucs::separate_streaming: ``on_frames(t0, block)`` receives each
        finished (8, count) block of denormalised stems in ascending order
        (the block is copied out of the library's staging first)."""
        left = np.ascontiguousarray(left, dtype=np.float32)
        right = np.ascontiguousarray(right, dtype=np.float32)
        error = []

        def _frames(t0, count, block, _u):
            try:
                on_frames(t0, np.ctypeslib.as_array(block, shape=(8, count)).copy())
            except Exception as exc:  # pragma: no cover - surfaced below
                error.append(exc)

        fcb = FRAMES_FN(_frames)
        pcb = PROGRESS_FN(0) if progress is None else PROGRESS_FN(lambda d, t, _u: progress(d, t))
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        _check(lib().dmx_separate_track_emit(self._h, _ptr(left), _ptr(right), left.shape[0],
                                             ctypes.byref(opts), fcb, pcb, None))
        if error:
            raise error[0]

    def separate_track_windowed(self, read, n, on_frames, shifts=1, overlap=0.25,
                                transition_power=1.0, batch=0, progress=None, segment=0.0):
        """Demucs::separate_streaming over a windowed source: ``read(t0, count)``
        returns the track's samples [t0, t0 + count) as (left, right) arrays;
        ``on_frames(t0, block)`` receives each finished (8, count) block in
        ascending order. The track is never held whole by the library."""
        error = []

        def _read(t0, count, left, right, _u):
            try:
                lr = read(t0, count)
                np.ctypeslib.as_array(left, shape=(count,))[:] = lr[0]
                np.ctypeslib.as_array(right, shape=(count,))[:] = lr[1]
                return 0
            except Exception as exc:
                error.append(exc)
                return 1

        def _frames(t0, count, block, _u):
            try:
                on_frames(t0, np.ctypeslib.as_array(block, shape=(8, count)).copy())
            except Exception as exc:  # pragma: no cover - surfaced below
                error.append(exc)

        rcb = READ_FN(_read)
        fcb = FRAMES_FN(_frames)
        pcb = PROGRESS_FN(0) if progress is None else PROGRESS_FN(lambda d, t, _u: progress(d, t))
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        status = lib().dmx_separate_track_windowed(self._h, rcb, n, ctypes.byref(opts), fcb, pcb,
                                                   None)
        if error:
            raise error[0]
        _check(status)

    def separate_batch(self, tracks, shifts=1, overlap=0.25, transition_power=1.0, batch=0,
                       progress=None, outs=None, segment=0.0):
        """Many (2, n_i) host tracks in one call with their chunks pooled into
        full forwards (dmx_separate_batch); returns a list of (4, 2, n_i)."""
        lefts = [np.ascontiguousarray(t[0], dtype=np.float32) for t in tracks]
        rights = [np.ascontiguousarray(t[1], dtype=np.float32) for t in tracks]
        lengths = (ctypes.c_int64 * len(tracks))(*[x.shape[0] for x in lefts])
        if outs is None:
            outs = [np.empty((4, 2, x.shape[0]), dtype=np.float32) for x in lefts]
        for o, x in zip(outs, lefts):
            assert o.shape == (4, 2, x.shape[0]) and o.dtype == np.float32 and o.flags.c_contiguous
        arr = lambda xs: (_f32p * len(xs))(*[_ptr(x) for x in xs])  # noqa: E731
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        cb = PROGRESS_FN(0) if progress is None else PROGRESS_FN(lambda d, t, _u: progress(d, t))
        _check(lib().dmx_separate_batch(self._h, arr(lefts), arr(rights), lengths, len(tracks),
                                        ctypes.byref(opts), arr(outs), cb, None))
        return outs

    def separate_batch_device(self, lr_ptrs, lengths, stems_ptrs, shifts=1, overlap=0.25,
                              batch=0, transition_power=1.0, segment=0.0):
        """Enqueue dmx_separate_batch_device on device buffers (returns at once)."""
        n = len(lr_ptrs)
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        _check(lib().dmx_separate_batch_device(
            self._h, (ctypes.c_void_p * n)(*lr_ptrs), (ctypes.c_int64 * n)(*lengths), n,
            ctypes.byref(opts), (ctypes.c_void_p * n)(*stems_ptrs), PROGRESS_FN(0), None))

    def track_shard(self, mix_norm_ptr, length, shift_offset, max_shift, overlap, chunk_lo,
                    chunk_hi, batch, acc_ptr, view_lo, view_hi, transition_power=1.0,
                    segment_samples=SEGMENT):
        _check(lib().dmx_track_shard(self._h, ctypes.c_void_p(mix_norm_ptr), length, shift_offset,
                                     max_shift, segment_samples, overlap, transition_power,
                                     chunk_lo, chunk_hi, batch, ctypes.c_void_p(acc_ptr), view_lo,
                                     view_hi))

    def set_trace(self, store: dict | None):
        if store is None:
            self._trace_cb = TRACE_FN(0)
        else:
            def _record(name, data, shape, ndim, _user):
                dims = tuple(shape[i] for i in range(ndim))
                store[name.decode()] = np.ctypeslib.as_array(data, shape=dims).copy()
            self._trace_cb = TRACE_FN(_record)
        _check(lib().dmx_set_trace(self._h, self._trace_cb, None))

    def separate_track_device(self, lr_ptr: int, n: int, stems_ptr: int, shifts=1,
                              overlap=0.25, batch=0, transition_power=1.0, segment=0.0):
        """Enqueue a whole-track separation on device buffers (returns at once)."""
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        _check(lib().dmx_separate_track_device(self._h, ctypes.c_void_p(lr_ptr), n,
                                               ctypes.byref(opts), ctypes.c_void_p(stems_ptr),
                                               PROGRESS_FN(0), None))

    def normalize_track_device(self, lr_ptr: int, n: int, mix_norm_ptr: int, mean_std_ptr: int):
        """Enqueue the global normalisation of a (2, n) device track."""
        _check(lib().dmx_normalize_track_device(self._h, ctypes.c_void_p(lr_ptr), n,
                                                ctypes.c_void_p(mix_norm_ptr),
                                                ctypes.c_void_p(mean_std_ptr)))

    def track_finish(self, acc_ptr, length, shift_offset, max_shift, overlap, shifts,
                     mean_std_ptr, stems_ptr, t_lo=0, t_hi=-1, transition_power=1.0,
                     segment_samples=SEGMENT):
        _check(lib().dmx_track_finish(self._h, ctypes.c_void_p(acc_ptr), length, shift_offset,
                                      max_shift, segment_samples, overlap, transition_power,
                                      shifts, ctypes.c_void_p(mean_std_ptr),
                                      ctypes.c_void_p(stems_ptr), t_lo, t_hi))

    def selftest_wait_timeout(self, wait_ms: int = 200):
        """dmx_selftest_wait_timeout: raises DmxError with code 4 (DMX_ERR_TIMEOUT)
        after a device wait that nothing satisfies gives up."""
        _check(lib().dmx_selftest_wait_timeout(self._h, wait_ms))

    def rows_copy(self, dst_ptr, dst_ld, src_ptr, src_ld, rows, width):
        """dmx_rows_copy on the handle's stream (src may be a mapped peer buffer)."""
        _check(lib().dmx_rows_copy(self._h, ctypes.c_void_p(dst_ptr), dst_ld,
                                   ctypes.c_void_p(src_ptr), src_ld, rows, width))

    def rows_add(self, dst_ptr, dst_ld, src_ptr, src_ld, rows, width):
        """dmx_rows_add: dst += src, each sum rounded on its own."""
        _check(lib().dmx_rows_add(self._h, ctypes.c_void_p(dst_ptr), dst_ld,
                                  ctypes.c_void_p(src_ptr), src_ld, rows, width))

    def set_stage_timing(self, on: bool):
        _check(lib().dmx_set_stage_timing(self._h, int(bool(on))))

    def stage_times(self, work: bool = False):
        """{kernel tag: (total ms, launches)} of the last forward with timing on;
        with ``work`` the tuples also carry the tag's algorithmic FLOPs and bytes."""
        names = (ctypes.c_char_p * 64)()
        ms = (ctypes.c_float * 64)()
        counts = (ctypes.c_int * 64)()
        flops = (ctypes.c_double * 64)()
        nbytes = (ctypes.c_double * 64)()
        n = lib().dmx_stage_times(self._h, names, ms, counts, flops, nbytes, 64)
        if work:
            return {names[i].decode(): (ms[i], counts[i], flops[i], nbytes[i]) for i in range(n)}
        return {names[i].decode(): (ms[i], counts[i]) for i in range(n)}

    @property
    def stream(self) -> int:
        return lib().dmx_stream(self._h) or 0

    def synchronize(self):
        _check(lib().dmx_synchronize(self._h))

    def kernel_launches(self) -> int:
        return lib().dmx_kernel_launches(self._h)


SOURCES = ("drums", "bass", "other", "vocals")


def _bag_args(weights, requested):
    w = np.ascontiguousarray(weights, dtype=np.float32)
    if w.ndim != 2 or w.shape[1] != len(SOURCES):
        raise ValueError(f"bag weights must be (n_nets, {len(SOURCES)}), got {w.shape}")
    req = None
    if requested is not None:
        flags = [1 if (s in requested or i in requested) else 0 for i, s in enumerate(SOURCES)]
        req = (ctypes.c_int * len(SOURCES))(*flags)
    return w, req


class Bag:
    """A bag of networks (htdemucs_ft): BagCombineForward (api.rs:319-371).

    ``handles`` are loaded networks on one device, ``weights`` the
    (n_nets, 4) per-source weight matrix (identity for htdemucs_ft) and
    ``requested`` the stems wanted (names or indices; None = all), which
    decides which networks run. The handles stay owned by the caller."""

    def __init__(self, handles, weights, requested=None):
        self.handles = list(handles)
        self.weights, self._req = _bag_args(weights, requested)
        if self.weights.shape[0] != len(self.handles):
            raise ValueError("one weight row per network")
        self._nets = (ctypes.c_void_p * len(self.handles))(*[h._h.value for h in self.handles])

    def forward_device(self, mix_ptr: int, n: int, out_ptr: int):
        """Enqueue the bag forward of n device segments (lead network's stream)."""
        _check(lib().dmx_bag_forward_device(self._nets, len(self.handles), _ptr(self.weights),
                                            self._req, ctypes.c_void_p(mix_ptr), n,
                                            ctypes.c_void_p(out_ptr)))

    def separate_track(self, left, right, shifts=1, overlap=0.25, transition_power=1.0,
                       batch=0, progress=None, out=None, segment=0.0):
        left = np.ascontiguousarray(left, dtype=np.float32)
        right = np.ascontiguousarray(right, dtype=np.float32)
        n = left.shape[0]
        stems = np.empty((4, 2, n), dtype=np.float32) if out is None else out
        assert stems.shape == (4, 2, n) and stems.dtype == np.float32 and stems.flags.c_contiguous
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        cb = PROGRESS_FN(0) if progress is None else PROGRESS_FN(lambda d, t, _u: progress(d, t))
        _check(lib().dmx_separate_track_bag(self._nets, len(self.handles), _ptr(self.weights),
                                            self._req, _ptr(left), _ptr(right), n,
                                            ctypes.byref(opts), _ptr(stems), cb, None))
        return stems

    def separate_track_device(self, lr_ptr: int, n: int, stems_ptr: int, shifts=1, overlap=0.25,
                              batch=0, transition_power=1.0, segment=0.0):
        opts = _opts(shifts, overlap, transition_power, batch, segment)
        _check(lib().dmx_separate_track_bag_device(self._nets, len(self.handles),
                                                   _ptr(self.weights), self._req,
                                                   ctypes.c_void_p(lr_ptr), n, ctypes.byref(opts),
                                                   ctypes.c_void_p(stems_ptr), PROGRESS_FN(0),
                                                   None))


def separate_track_multi(handles, left, right, shifts=1, overlap=0.25, batch=0, out=None,
                         transition_power=1.0, segment=0.0):
    """dmx_separate_track_multi: one track over several handles (one per GPU,
    the same network on each) from this thread; returns (4, 2, n)."""
    left = np.ascontiguousarray(left, dtype=np.float32)
    right = np.ascontiguousarray(right, dtype=np.float32)
    n = left.shape[0]
    stems = np.empty((4, 2, n), dtype=np.float32) if out is None else out
    assert stems.shape == (4, 2, n) and stems.dtype == np.float32 and stems.flags.c_contiguous
    hs = (ctypes.c_void_p * len(handles))(*[h._h.value for h in handles])
    opts = _opts(shifts, overlap, transition_power, batch, segment)
    _check(lib().dmx_separate_track_multi(hs, len(handles), _ptr(left), _ptr(right), n,
                                          ctypes.byref(opts), _ptr(stems)))
    return stems


def bag_combine_device(out_ptrs, weights, requested, n_segments: int, samples: int,
                       combined_ptr: int, stream: int = 0):
    """dmx_bag_combine_device: ``out_ptrs`` are device pointers (0 for networks
    that carry no requested weight), each (n_segments, 4, 2, samples)."""
    w, req = _bag_args(weights, requested)
    ptrs = (ctypes.c_void_p * len(out_ptrs))(*[p or None for p in out_ptrs])
    _check(lib().dmx_bag_combine_device(ptrs, len(out_ptrs), _ptr(w), req, n_segments, samples,
                                        ctypes.c_void_p(combined_ptr), ctypes.c_void_p(stream)))


def normalize_track_noalloc(lr_ptr: int, n: int, mix_norm_ptr: int, mean_std_ptr: int,
                            stream: int = 0):
    """dmx_normalize_track_noalloc: the track normalisation without a handle
    and without allocating device memory (for callers that may not allocate,
    such as real-time audio callbacks), on the current device's buffers."""
    _check(lib().dmx_normalize_track_noalloc(ctypes.c_void_p(lr_ptr), n,
                                             ctypes.c_void_p(mix_norm_ptr),
                                             ctypes.c_void_p(mean_std_ptr),
                                             ctypes.c_void_p(stream)))


def read_tensor(blob: bytes, name: str):
    """dmx_read_tensor: one tensor of a safetensors blob as float32, decoded by
    the library's loader (no GPU needed)."""
    buf = ctypes.create_string_buffer(blob, len(blob))
    cap = max(1, len(blob))
    out = np.empty(cap, dtype=np.float32)
    shape = (ctypes.c_int64 * 8)()
    ndim = ctypes.c_int()
    _check(lib().dmx_read_tensor(ctypes.cast(buf, ctypes.c_void_p), len(blob), name.encode(),
                                 _ptr(out), cap, shape, ctypes.byref(ndim)))
    dims = tuple(shape[i] for i in range(ndim.value))
    return out[:int(np.prod(dims, dtype=np.int64))].reshape(dims).copy()


def ipc_export(device: int, ptr: int):
    """dmx_ipc_export: (64-byte handle, offset) of a device buffer of `device`."""
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_int64()
    _check(lib().dmx_ipc_export(device, ctypes.c_void_p(ptr), handle, ctypes.byref(offset)))
    return handle.raw, offset.value


def ipc_open(device: int, handle: bytes, offset: int) -> int:
    """dmx_ipc_open: maps another process's exported buffer on `device`."""
    ptr = ctypes.c_void_p()
    _check(lib().dmx_ipc_open(device, handle, offset, ctypes.byref(ptr)))
    return ptr.value


def ipc_close(device: int, ptr: int, offset: int):
    _check(lib().dmx_ipc_close(device, ctypes.c_void_p(ptr), offset))


def shift_offsets(passes: int, max_shift: int = 22050):
    """dmx_shift_offsets: the ShiftRng offsets of each shift pass."""
    out = (ctypes.c_int64 * max(1, passes))()
    _check(lib().dmx_shift_offsets(passes, max_shift, out))
    return [int(out[i]) for i in range(passes)]


def num_chunks(view_length: int, segment: int = SEGMENT, overlap: float = 0.25) -> int:
    return lib().dmx_num_chunks(view_length, segment, overlap)
