"""SeparateOptions beyond the defaults on the device drivers (GPU).

* transition_power != 1: the triangular overlap-add window raised to that
  power (pipeline.rs:117-131), both for the weights and their sums.
* segment < 7.8 s: chunks of int(44100 * segment) samples, each zero padded
  to the model's 343980 samples for the forward and trimmed back to the chunk
  (streaming.rs:315-321; Htdemucs::forward, host.rs:210-229).

Each device result is checked against the oracle's driver with the device
forward plugged in, so only the driver arithmetic differs.
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu

SEG = synth.SEGMENT_SAMPLES


def _handle(seed, max_batch=3):
    import dmx
    return dmx.Handle(synth.write_safetensors(synth.random_weights(seed)), device=0,
                      max_batch=max_batch, precision=dmx.TF32)


def _padded_forward(h):
    """The model forward on chunks shorter than its segment: zero padded at the
    end to 343980 samples, output trimmed to the chunk (host.rs:217-229, 493-501)."""

    def fwd(x):
        g, c, chunk = x.shape
        wide = np.zeros((g, c, SEG), np.float32)
        wide[:, :, :chunk] = x
        return h.forward(wide)[:, :, :, :chunk]

    return fwd


@pytest.mark.parametrize("shifts,power,segment", [
    (1, 2.0, 0.0),     # power only
    (0, 1.0, 4.0),     # segment only
    (2, 0.5, 3.25),    # both, several shift passes
])
def test_track_driver_options_match_the_oracle_driver(shifts, power, segment):
    h = _handle(101)
    track = synth.pink_noise(102, int(44100 * 17))
    got = h.separate_track(track[0], track[1], shifts=shifts, transition_power=power,
                           segment=segment, batch=3)
    chunk = int(44100 * segment) if segment else SEG
    ref = oracle.separate_with(_padded_forward(h), track, chunk, shifts=shifts,
                               transition_power=power, batch=2)
    assert got.shape == ref.shape
    err = np.abs(got.astype(np.float64) - ref).max()
    assert err <= 1e-6 * max(1.0, np.abs(ref).max()), err
    h.close()


def test_pooled_batch_and_emit_honour_the_options():
    h = _handle(103)
    tracks = [synth.pink_noise(104 + i, int(44100 * s)) for i, s in enumerate((9.0, 5.5))]
    opts = dict(shifts=1, transition_power=1.5, segment=5.0, batch=3)
    pooled = h.separate_batch(tracks, **opts)
    for t, g in zip(tracks, pooled):
        ref = h.separate_track(t[0], t[1], **opts)
        assert np.abs(g.astype(np.float64) - ref).max() <= 1e-6
    blocks = []
    h.separate_track_emit(tracks[0][0], tracks[0][1], lambda t0, b: blocks.append(b), **opts)
    got = np.concatenate(blocks, axis=1).reshape(pooled[0].shape)
    assert np.abs(got.astype(np.float64) - pooled[0]).max() <= 1e-6
    h.close()


def test_multi_handle_driver_rejects_half_overlap_and_honours_the_options():
    import dmx

    hs = [_handle(105, max_batch=2), _handle(105, max_batch=2)]
    track = synth.pink_noise(106, int(44100 * 15))
    with pytest.raises(dmx.DmxError, match="overlap < 0.5"):
        dmx.separate_track_multi(hs, track[0], track[1], shifts=1, overlap=0.6)
    got = dmx.separate_track_multi(hs, track[0], track[1], shifts=1, transition_power=2.0,
                                   segment=6.0)
    ref = hs[0].separate_track(track[0], track[1], shifts=1, transition_power=2.0, segment=6.0)
    assert np.abs(got.astype(np.float64) - ref).max() <= 1e-6
    for h in hs:
        h.close()
