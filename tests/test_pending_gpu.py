"""SegmentForward through the C ABI with the reference's queue-one-ahead loop (GPU).

The reference's split pass (streaming.rs:341-383; pipeline.rs:596-641) builds
group n, starts its forward, drops the batch, and only then collects group
n - 1, so two forwards are in flight on one runner, each owning its staging
(PendingStems, gpu/htdemucs.rs:2744-2782). This restates that loop in Python
over dmx_forward_start / dmx_forward_collect and checks it against
dmx_separate_track on the same handle.
"""

import ctypes

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu

SEG = synth.SEGMENT_SAMPLES


def _handle(seed, max_batch=2, precision="TF32"):
    import dmx
    return dmx.Handle(synth.write_safetensors(synth.random_weights(seed)), device=0,
                      max_batch=max_batch, precision=getattr(dmx, precision))


def _padded_chunk(mix, start, chunk):
    """mix.rs:552-633 / pipeline.rs:70-103 (shifts 0) through the oracle."""
    out = np.zeros((2, SEG), np.float32)
    oracle.lib().orc_padded_chunk(oracle.ptr(mix), 2, ctypes.c_int64(mix.shape[1]),
                                  ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(start),
                                  ctypes.c_int64(chunk), SEG, oracle.ptr(out))
    return out


def _normalised(track):
    mean, std = ctypes.c_float(), ctypes.c_float()
    oracle.lib().orc_scan_norm(oracle.ptr(track), 2, ctypes.c_int64(track.shape[1]),
                               ctypes.byref(mean), ctypes.byref(std))
    return ((track - mean.value) / std.value).astype(np.float32), mean.value, std.value


def _groups(track, batch):
    mix, _, _ = _normalised(track)
    n = mix.shape[1]
    starts = list(range(0, n, int(0.75 * SEG)))
    return [np.stack([_padded_chunk(mix, s, min(n - s, SEG)) for s in starts[i:i + batch]])
            for i in range(0, len(starts), batch)]


def _split_pass_queue_one_ahead(h, track, batch):
    """stream_split_pass_meta's loop (shifts 0): start(n) before collect(n - 1)."""
    mix, mean, std = _normalised(track)
    n = mix.shape[1]
    stride = int(0.75 * SEG)
    weight = np.empty(SEG, np.float32)
    oracle.lib().orc_transition_weight(SEG, 1.0, oracle.ptr(weight))
    starts = list(range(0, n, stride))
    acc = np.zeros((8, n), np.float32)
    wsum = np.zeros(n, np.float32)
    queued = None
    outs = []
    offset = 0
    while offset < len(starts) or queued is not None:
        resolved = None
        if offset < len(starts):
            spans = [(s, min(n - s, SEG)) for s in starts[offset:offset + batch]]
            batched = np.stack([_padded_chunk(mix, s, c) for s, c in spans])
            pending = h.forward_start(batched)
            del batched  # the reference drops its batch before collect
            offset += len(spans)
            resolved, queued = queued, (spans, pending)
        else:
            resolved, queued = queued, None
        if resolved is None:
            continue
        spans, pending = resolved
        y = h.forward_collect(pending)
        outs.append(y)
        for slot, (s, c) in enumerate(spans):
            trim = (SEG - c) // 2
            acc[:, s:s + c] += weight[:c] * y[slot].reshape(8, SEG)[:, trim:trim + c]
            wsum[s:s + c] += weight[:c]
    stems = (acc / wsum) * std + mean
    return stems.reshape(4, 2, n), outs


def test_queue_one_ahead_loop_matches_the_track_driver():
    h = _handle(91)
    track = synth.pink_noise(92, int(44100 * 30))  # 6 chunks: three groups of two
    got, outs = _split_pass_queue_one_ahead(h, track, batch=2)
    assert len(outs) == 3
    # each queued group's output is the synchronous forward's, bit for bit
    mix_groups = _groups(track, batch=2)
    for y, g in zip(outs, mix_groups):
        assert np.array_equal(y, h.forward(g))
    ref = h.separate_track(track[0], track[1], shifts=0, batch=2)
    scale = np.abs(ref).max()
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-5 * scale, (err, scale)
    h.close()


def test_two_forwards_in_flight_return_their_own_results_in_any_order():
    import dmx

    h = _handle(93, precision="FP32")
    a = synth.gaussian_audio(94, 2)
    b = synth.gaussian_audio(95, 1)
    ya = h.forward(a)
    yb = h.forward(b)
    pa = h.forward_start(a)
    pb = h.forward_start(b)
    with pytest.raises(dmx.DmxError, match="already in flight"):
        h.forward_start(a)
    got_b = h.forward_collect(pb)  # collected out of order
    got_a = h.forward_collect(pa)
    assert np.array_equal(got_a, ya) and np.array_equal(got_b, yb)
    # both slots are free again
    pc = h.forward_start(b)
    assert np.array_equal(h.forward_collect(pc), yb)
    h.close()
