"""Many tracks with pooled chunks (dmx_separate_batch) on the device (GPU).

Pooling only changes which chunks share a forward; every track must come out
as dmx_separate_track makes it (which the track tests pin to the oracle's
driver), to the f32 rounding by which the forward may differ between batch
compositions. Windows here straddle tracks and shift passes on purpose.
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu


def _handle(seed, max_batch=3):
    import dmx
    return dmx.Handle(synth.write_safetensors(synth.random_weights(seed)), device=0,
                      max_batch=max_batch)


def _units(n, shifts):
    """Chunks of all shift passes of an n-sample track (streaming.rs:88-94)."""
    import shard

    stride = int(0.75 * synth.SEGMENT_SAMPLES)
    if shifts == 0:
        return -(-n // stride)
    return sum(-(-(n + 22050 - o) // stride) for o in shard.shift_offsets(shifts, 22050))


@pytest.mark.parametrize("shifts,batch,seconds", [
    (2, 3, (5.0, 14.0, 9.0)),          # windows span passes and tracks
    (0, 3, (1.0, 0.5, 2.0, 1.5, 0.25)),  # one chunk per track: three tracks share a forward
    (1, 2, (8.5,)),
])
def test_pooled_tracks_match_single_track_driver(shifts, batch, seconds):
    h = _handle(61)
    tracks = [synth.pink_noise(70 + i, int(44100 * s)) for i, s in enumerate(seconds)]
    seen = []
    got = h.separate_batch(tracks, shifts=shifts, batch=batch,
                           progress=lambda d, t: seen.append((d, t)))
    for t, g in zip(tracks, got):
        ref = h.separate_track(t[0], t[1], shifts=shifts, batch=2)
        err = np.abs(g.astype(np.float64) - ref).max()
        assert err <= 1e-6, err
    units = sum(_units(t.shape[1], shifts) for t in tracks)
    assert seen[-1] == (units, units)
    assert [d for d, _ in seen] == sorted(d for d, _ in seen)
    h.close()


def test_batch_device_entry_point_against_oracle_driver():
    import torch

    h = _handle(62, max_batch=4)
    tracks = [synth.pink_noise(80 + i, int(44100 * s)) for i, s in enumerate((6.0, 3.0))]
    lr = [torch.from_numpy(t).cuda() for t in tracks]
    stems = [torch.full((4, 2, t.shape[1]), float("nan"), device="cuda") for t in tracks]
    torch.cuda.synchronize()
    h.separate_batch_device([x.data_ptr() for x in lr], [t.shape[1] for t in tracks],
                            [s.data_ptr() for s in stems], shifts=1, batch=4)
    h.synchronize()
    for t, s in zip(tracks, stems):
        ref = oracle.separate_with(h.forward, t, synth.SEGMENT_SAMPLES, shifts=1, batch=2)
        err = np.abs(s.cpu().numpy().astype(np.float64) - ref).max()
        assert err <= 1e-6, err
    h.close()


def test_batch_rejects_an_empty_track():
    import dmx

    h = _handle(63, max_batch=1)
    with pytest.raises(dmx.DmxError, match="track 1 is empty"):
        h.separate_batch([synth.pink_noise(1, 1000), np.zeros((2, 0), np.float32)])
    h.close()
