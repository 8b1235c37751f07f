"""Whole-track separation on the device (dmx_separate_track) against the
oracle's driver (GPU).

* With the same segment forward on both sides (the CUDA forward), the device
  driver — global normalisation, ShiftRng shift view, centred chunks,
  triangular overlap-add, trim, denormalisation — must reproduce the oracle's
  driver (streaming.rs:52-400, pipeline.rs:380-515) to f32 rounding.
* End to end against the oracle's own forward, within the 1e-4 gate for the
  FP32 and TF32X3 builds and the per-stem SNR >= 60 dB gate for TF32, the
  benchmarked build, including at the benchmark's batching (every chunk of
  the track in one forward).
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu


PRECISIONS = ["FP32", "TF32", "TF32X3", "BF16"]


def _handle(weights, max_batch=4, precision="FP32"):
    import dmx
    return dmx.Handle(synth.write_safetensors(weights), device=0, max_batch=max_batch,
                      precision=getattr(dmx, precision))


def snr_db(ref, x):
    """Energy SNR, 10 log10(sum ref^2 / sum (ref - x)^2)."""
    ref = ref.astype(np.float64)
    return 10 * np.log10(np.sum(ref ** 2) / max(np.sum((ref - x) ** 2), 1e-300))


def _assert_stems_within_gate(got, ref, precision):
    # FP32 / TF32X3: max-abs <= 1e-4 per stem; TF32 / BF16: per-stem energy SNR >= 60 dB
    if precision in ("TF32", "BF16"):
        per_stem = [snr_db(ref[s], got[s]) for s in range(4)]
        assert min(per_stem) >= 60.0, per_stem
    else:
        err = np.abs(got.astype(np.float64) - ref).reshape(4, -1).max(axis=1)
        assert err.max() <= 1e-4, err


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shifts", [0, 1, 2])
def test_device_driver_matches_oracle_driver(shifts, precision):
    w = synth.random_weights(21)
    h = _handle(w, precision=precision)
    track = synth.pink_noise(31, int(44100 * 20))
    got = h.separate_track(track[0], track[1], shifts=shifts, batch=2)
    ref = oracle.separate_with(h.forward, track, synth.SEGMENT_SAMPLES, shifts=shifts, batch=3)
    assert got.shape == ref.shape == (4, 2, track.shape[1])
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-6, err


@pytest.mark.parametrize("precision", PRECISIONS)
def test_track_matches_oracle_end_to_end(precision):
    w = synth.random_weights(22)
    track = synth.pink_noise(32, int(44100 * 11))
    got = _handle(w, precision=precision).separate_track(track[0], track[1], shifts=1)
    ref = oracle.OracleModel(w).separate(track, shifts=1)
    _assert_stems_within_gate(got, ref, precision)


@pytest.fixture(scope="module")
def bench_track_reference():
    # the oracle's own end-to-end separation of a 60 s slice of the benchmark's track
    w = synth.random_weights(0)
    track = synth.pink_noise(2024, int(44100 * 60))
    return w, track, oracle.OracleModel(w).separate(track, shifts=1, batch=4)


@pytest.mark.parametrize("precision", ["TF32", "BF16"])
def test_benchmarked_path_at_full_batch_meets_the_gate(bench_track_reference, precision):
    # the path bench.py times: dmx_separate_track with every chunk of a pink-noise track
    # in one forward (here 60 s: 11 chunks with shifts 1), against the oracle's own
    # end-to-end separation; then the same build one chunk per forward
    import dmx

    w, track, ref = bench_track_reference
    chunks = dmx.num_chunks(track.shape[1] + 22050 - dmx.shift_offsets(1)[0])
    h = _handle(w, max_batch=chunks, precision=precision)
    got = h.separate_track(track[0], track[1], shifts=1, batch=chunks)
    per_stem = [snr_db(ref[s], got[s]) for s in range(4)]
    print(f"{precision} full-batch per-stem SNR (dB):", [round(x, 2) for x in per_stem])
    assert min(per_stem) >= 60.0, per_stem
    one = h.separate_track(track[0], track[1], shifts=1, batch=1)
    assert np.array_equal(one, got)  # batch composition changes no output bit


def test_progress_reports_every_chunk():
    w = synth.random_weights(23)
    h = _handle(w, max_batch=1)
    track = synth.pink_noise(33, int(44100 * 16))
    seen = []
    h.separate_track(track[0], track[1], shifts=0, batch=1, progress=lambda d, t: seen.append((d, t)))
    import dmx
    total = dmx.num_chunks(track.shape[1])
    assert seen == [(i + 1, total) for i in range(total)]


def test_normalize_track_matches_oracle_scan_norm():
    # streaming.rs:52-85: mean / unbiased std (+1e-8) of the channel-mean signal
    import ctypes
    import torch
    import dmx
    h = _handle(synth.random_weights(24), max_batch=1)
    track = synth.pink_noise(34, 1_000_003)
    lr = torch.from_numpy(track).cuda()
    norm = torch.empty_like(lr)
    ms = torch.empty(2, dtype=torch.float32, device="cuda")
    h.normalize_track_device(lr.data_ptr(), track.shape[1], norm.data_ptr(), ms.data_ptr())
    h.synchronize()
    mean, std = ctypes.c_float(), ctypes.c_float()
    oracle.lib().orc_scan_norm(oracle.ptr(track), 2, ctypes.c_int64(track.shape[1]),
                               ctypes.byref(mean), ctypes.byref(std))
    got = ms.cpu().numpy()
    # both reduce in f64, in different orders; the mean is a near-total
    # cancellation (~1e-12), so compare it on the scale of the std
    assert abs(got[0] - mean.value) <= 1e-6 * std.value, (got, mean.value)
    assert abs(got[1] - std.value) <= 1e-6 * std.value, (got, std.value)
    ref = (track - mean.value) / std.value
    np.testing.assert_allclose(norm.cpu().numpy(), ref, rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("shifts,batch", [(0, 2), (1, 2), (1, 1), (2, 2)])
def test_pinned_host_stems_stream_back_during_the_forwards(shifts, batch):
    # with pinned host stems, dmx_separate_track finishes and copies each batch's final
    # samples while later batches run; the result is the device entry point's
    import torch

    h = _handle(synth.random_weights(25), precision="TF32")
    track = synth.pink_noise(37, int(44100 * 20))
    n = track.shape[1]
    out = torch.full((4, 2, n), float("nan")).pin_memory()
    got = h.separate_track(track[0], track[1], shifts=shifts, batch=batch, out=out.numpy())
    lr = torch.from_numpy(track).cuda()
    stems = torch.empty((4, 2, n), device="cuda")
    torch.cuda.synchronize()
    h.separate_track_device(lr.data_ptr(), n, stems.data_ptr(), shifts=shifts, batch=batch)
    h.synchronize()
    ref = stems.cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-6, err


@pytest.mark.parametrize("shifts,batch", [(0, 2), (1, 1), (2, 2)])
def test_emitted_blocks_reassemble_the_separated_track(shifts, batch):
    # Demucs::separate_streaming: ascending blocks of finished stems, each at most one
    # forward's worth (single pass), that put together are dmx_separate_track's result
    h = _handle(synth.random_weights(26), precision="TF32")
    track = synth.pink_noise(38, int(44100 * 21))
    n = track.shape[1]
    blocks = []
    h.separate_track_emit(track[0], track[1], lambda t0, b: blocks.append((t0, b)),
                          shifts=shifts, batch=batch)
    ref = h.separate_track(track[0], track[1], shifts=shifts, batch=batch)
    assert [t0 for t0, _ in blocks] == sorted(t0 for t0, _ in blocks)
    assert blocks[0][0] == 0 and blocks[-1][0] + blocks[-1][1].shape[1] == n
    for (t0, b), (t1, _) in zip(blocks, blocks[1:]):
        assert t0 + b.shape[1] == t1
    if shifts <= 1:
        assert len(blocks) > 1
        assert max(b.shape[1] for _, b in blocks) <= batch * int(0.75 * synth.SEGMENT_SAMPLES)
    got = np.concatenate([b for _, b in blocks], axis=1).reshape(4, 2, n)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("n", [1, 1000, 22050, synth.SEGMENT_SAMPLES + 1])
def test_short_and_ragged_tracks_match_the_oracle_driver(n):
    # one chunk or barely more (the view is padded with zeros on both sides,
    # mix.rs:552-633). A one-sample track normalises to an all-zero segment,
    # whose std is 0: the reference denormalises with affine_in_place(x,
    # -mean / std, std) (host.rs:466-509), which is 0/0 there, so its stems are
    # NaN; the device reproduces that, as the oracle does
    h = _handle(synth.random_weights(27), max_batch=2)
    track = synth.pink_noise(40, max(n, 2))[:, :n].copy() if n > 1 else np.full((2, 1), 0.05, np.float32)
    for shifts in (0, 1):
        got = h.separate_track(track[0], track[1], shifts=shifts)
        ref = oracle.separate_with(h.forward, track, synth.SEGMENT_SAMPLES, shifts=shifts)
        assert got.shape == ref.shape == (4, 2, n)
        assert np.array_equal(np.isnan(got), np.isnan(ref))
        assert np.isnan(got).all() if n == 1 else np.isfinite(got).all()
        ok = ~np.isnan(ref)
        if ok.any():
            err = np.abs(got[ok].astype(np.float64) - ref[ok]).max()
            assert err <= 1e-6 * max(1.0, np.abs(ref[ok]).max()), err


def test_invalid_driver_arguments_are_rejected():
    import dmx

    h = _handle(synth.random_weights(28), max_batch=1)
    x = synth.pink_noise(41, 5000)
    with pytest.raises(dmx.DmxError, match="bad argument"):
        h.separate_track(x[0][:0], x[1][:0])
    with pytest.raises(dmx.DmxError, match="zero stride"):
        h.separate_track(x[0], x[1], overlap=1.0)
    with pytest.raises(dmx.DmxError, match="transition_power"):
        h.separate_track(x[0], x[1], transition_power=0.0)
    with pytest.raises(dmx.DmxError, match="shifts"):
        h.separate_track(x[0], x[1], shifts=-1)
    with pytest.raises(dmx.DmxError, match="model segment is 343980"):
        h.separate_track(x[0], x[1], segment=8.0)


def test_a_device_wait_that_runs_out_reports_timeout_and_the_handle_stays_usable():
    # the bounded-wait error path: a kernel waits on a device flag nothing sets, gives up
    # after 200 ms and raises the handle's error flag; the host reports DMX_ERR_TIMEOUT
    # and the next work on the same handle runs normally
    import time

    import dmx

    h = _handle(synth.random_weights(29), max_batch=1)
    mix = synth.gaussian_audio(9, 1)
    before = h.forward(mix)
    t0 = time.perf_counter()
    with pytest.raises(dmx.DmxError, match="self-test kernel gave up a bounded wait") as e:
        h.selftest_wait_timeout(200)
    assert e.value.code == 4
    assert 0.15 < time.perf_counter() - t0 < 30
    after = h.forward(mix)
    assert np.abs(after.astype(np.float64) - before).max() <= 1e-6
    with pytest.raises(dmx.DmxError, match="wait_ms"):
        h.selftest_wait_timeout(0)
