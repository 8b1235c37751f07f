"""The windowed streaming driver (dmx_separate_track_windowed, GPU): the
track is read through a callback in windows (WindowedMix, mix.rs:61-360) and
overlap-added in a sliding device window (OlaRing, streaming.rs:96-261). Its
stems must equal dmx_separate_track's bit for bit, for every shift mode,
batching, segment override and ragged length, while each read stays within
one forward's chunks and the device memory it holds does not grow with the
track."""

import numpy as np
import pytest

import dmx
import synth

pytestmark = pytest.mark.gpu

STRIDE = int(0.75 * synth.SEGMENT_SAMPLES)


def _handle(seed, max_batch=16, precision="TF32"):
    return dmx.Handle(synth.write_safetensors(synth.random_weights(seed)), device=0,
                      max_batch=max_batch, precision=getattr(dmx, precision))


def windowed(h, track, **kw):
    n = track.shape[1]
    reads, blocks = [], []

    def read(t0, count):
        assert 0 <= t0 and t0 + count <= n
        reads.append((t0, count))
        return track[0, t0:t0 + count], track[1, t0:t0 + count]

    h.separate_track_windowed(read, n, lambda t0, b: blocks.append((t0, b)), **kw)
    assert blocks[0][0] == 0
    for (t0, b), (t1, _) in zip(blocks, blocks[1:]):
        assert t0 + b.shape[1] == t1
    assert blocks[-1][0] + blocks[-1][1].shape[1] == n
    return np.concatenate([b for _, b in blocks], axis=1).reshape(4, 2, n), reads


@pytest.mark.parametrize("shifts,batch,segment,overlap,power", [
    (0, 1, 0.0, 0.25, 1.0),
    (1, 2, 0.0, 0.25, 1.0),
    (1, 16, 0.0, 0.25, 1.0),
    (2, 3, 0.0, 0.25, 1.0),
    (1, 4, 5.0, 0.4, 2.0),
])
def test_windowed_stems_equal_the_whole_track_driver(shifts, batch, segment, overlap, power):
    h = _handle(71)
    track = synth.pink_noise(72, int(44100 * 31.7) + 13)
    kw = dict(shifts=shifts, batch=batch, segment=segment, overlap=overlap,
              transition_power=power)
    got, reads = windowed(h, track, **kw)
    ref = h.separate_track(track[0], track[1], **kw)
    assert np.array_equal(got, ref)
    # a split-pass read covers one forward's chunks and their centring margin
    chunk = int(44100 * segment) if segment else synth.SEGMENT_SAMPLES
    stride = int((1 - overlap) * chunk)
    bound = max((batch - 1) * stride + chunk + chunk // 2 + 1, 296 * 512)
    assert max(c for _, c in reads) <= bound


@pytest.mark.parametrize("n", [1000, 22050, synth.SEGMENT_SAMPLES + 1, 296 * 512 * 3 + 7])
def test_short_and_ragged_tracks(n):
    h = _handle(73, max_batch=2)
    track = synth.pink_noise(74, n)
    for shifts in (0, 1, 2):
        got, _ = windowed(h, track, shifts=shifts, batch=2)
        ref = h.separate_track(track[0], track[1], shifts=shifts, batch=2)
        assert np.array_equal(got, ref), shifts


def test_device_memory_does_not_grow_with_the_track():
    import torch

    h = _handle(75, max_batch=2)
    h.forward(synth.gaussian_audio(1, segments=2))  # the forward's own workspace
    torch.cuda.synchronize()
    base = torch.cuda.mem_get_info()[0]
    short = synth.pink_noise(76, 44100 * 30)
    windowed(h, short, shifts=1, batch=2)
    after_short = torch.cuda.mem_get_info()[0]
    long = np.tile(short, (1, 20))  # 10 minutes
    got, reads = windowed(h, long, shifts=1, batch=2)
    after_long = torch.cuda.mem_get_info()[0]
    # the driver's window, accumulators, output blocks and chunk staging at
    # batch 2 (about 115 MB), the same for 30 s and for 10 min
    assert abs(after_long - after_short) <= 8 * 2**20, (base - after_short, base - after_long)
    assert base - after_long < 256 * 2**20, base - after_long
    ref = h.separate_track(long[0], long[1], shifts=1, batch=2)
    assert np.array_equal(got, ref)


def test_a_failing_read_stops_the_separation_and_the_handle_stays_usable():
    h = _handle(77, max_batch=2)
    track = synth.pink_noise(78, 44100 * 20)
    n = track.shape[1]

    def read(t0, count):
        if t0 > 0:  # every window after the first
            raise OSError("disk went away")
        return track[0, t0:t0 + count], track[1, t0:t0 + count]

    with pytest.raises(OSError, match="disk went away"):
        h.separate_track_windowed(read, n, lambda t0, b: None, shifts=0, batch=1)
    got, _ = windowed(h, track, shifts=0, batch=1)
    assert np.array_equal(got, h.separate_track(track[0], track[1], shifts=0, batch=1))
