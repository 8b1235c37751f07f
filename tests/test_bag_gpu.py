"""Bags of networks (htdemucs_ft) on the device (GPU), through the C ABI.

* dmx_bag_combine_device against the oracle's combination (api.rs:338-360),
  bit for bit: both form the same f32 products, sums and quotient.
* dmx_separate_track_bag (four networks, lockstep combination before the
  overlap-add) against the oracle's driver over the oracle's bag forward with
  the same (device) network forwards, to f32 rounding.
* End to end against the oracle's own networks, within the 1e-4 gate.
"""

import numpy as np
import pytest

import oracle
import synth

pytestmark = pytest.mark.gpu

IDENTITY = np.eye(4, dtype=np.float32)
MIXED = np.array([[0.5, 0.0, 1.0, 0.0],
                  [0.0, 2.0, 0.25, 0.0],
                  [0.5, 0.0, 0.0, 1.0],
                  [0.0, 0.0, 0.0, 0.0]], dtype=np.float32)


def _handles(seeds, max_batch=2):
    import dmx
    return [dmx.Handle(synth.write_safetensors(synth.random_weights(s)), device=0,
                       max_batch=max_batch) for s in seeds]


@pytest.mark.parametrize("weights,requested", [(IDENTITY, None), (MIXED, None),
                                               (MIXED, ["vocals", "bass"])])
def test_bag_combine_device_is_bitwise_the_reference_combination(weights, requested):
    import torch
    import dmx

    g, samples = 3, 10_001  # odd length: the scalar kernel; samples * 8 % 4 == 0 lanes below
    for n in (samples, 343980):
        outs = [torch.randn((g, 4, 2, n), device="cuda") for _ in range(4)]
        combined = torch.full((g, 4, 2, n), float("nan"), device="cuda")
        dmx.bag_combine_device([o.data_ptr() for o in outs], weights, requested, g, n,
                               combined.data_ptr())
        torch.cuda.synchronize()
        req = None if requested is None else [dmx.SOURCES.index(r) for r in requested]
        host = [o.cpu().numpy() for o in outs]
        ref = oracle.bag_forward([(lambda x, h=h: h) for h in host], weights, req)(
            np.zeros((g, 2, n), np.float32))
        assert np.array_equal(combined.cpu().numpy(), ref)


def test_bag_rejects_an_uncovered_stem():
    import dmx

    hs = _handles([1, 2, 3], max_batch=1)
    bag = dmx.Bag(hs, MIXED[:3] * np.array([1, 1, 1, 0], dtype=np.float32))
    track = synth.pink_noise(5, 44100)
    with pytest.raises(dmx.DmxError, match="no network covers stem index 3"):
        bag.separate_track(track[0], track[1])


@pytest.mark.parametrize("weights,requested,shifts", [(IDENTITY, None, 1), (MIXED, [1, 2, 3], 0)])
def test_device_bag_driver_matches_oracle_lockstep(weights, requested, shifts):
    import dmx

    hs = _handles([11, 12, 13, 14])
    track = synth.pink_noise(35, int(44100 * 14))
    bag = dmx.Bag(hs, weights, requested)
    seen = []
    got = bag.separate_track(track[0], track[1], shifts=shifts, batch=2,
                             progress=lambda d, t: seen.append((d, t)))
    fwd = oracle.bag_forward([h.forward for h in hs], weights, requested)
    ref = oracle.separate_with(fwd, track, synth.SEGMENT_SAMPLES, shifts=shifts, batch=3)
    req = range(4) if requested is None else requested
    for s in req:
        err = np.abs(got[s].astype(np.float64) - ref[s]).max()
        assert err <= 1e-6, (s, err)
    import shard

    running = len([k for k in range(4) if any(weights[k, s] != 0 for s in req)])
    chunks = shard.plan(track.shape[1], 1, shifts=shifts).chunks
    assert seen[-1] == (chunks * running, chunks * running)
    for h in hs:
        h.close()


def test_bag_end_to_end_against_oracle_networks():
    import dmx

    seeds = [41, 42]
    hs = _handles(seeds, max_batch=1)
    w = np.array([[1.0, 0.0, 1.0, 0.5], [0.0, 1.0, 1.0, 0.5]], dtype=np.float32)
    track = synth.pink_noise(36, int(44100 * 9))
    got = dmx.Bag(hs, w).separate_track(track[0], track[1], shifts=0)
    nets = [oracle.OracleModel(synth.random_weights(s)) for s in seeds]
    ref = oracle.separate_with(oracle.bag_forward([m.forward for m in nets], w), track,
                               synth.SEGMENT_SAMPLES, shifts=0)
    err = np.abs(got.astype(np.float64) - ref).reshape(4, -1).max(axis=1)
    assert err.max() <= 1e-4, err


def test_bag_forward_device_is_the_lockstep_segment_forward():
    # BagCombineForward as a SegmentForward (api.rs:319-371) on device buffers
    import torch
    import dmx

    hs = _handles([51, 52], max_batch=2)
    w = np.array([[1.0, 0.0, 0.5, 0.0], [0.0, 1.0, 0.5, 1.0]], dtype=np.float32)
    mix = synth.gaussian_audio(7, 3)
    x = torch.from_numpy(mix).cuda()
    out = torch.full((3, 4, 2, synth.SEGMENT_SAMPLES), float("nan"), device="cuda")
    torch.cuda.synchronize()
    dmx.Bag(hs, w).forward_device(x.data_ptr(), 3, out.data_ptr())
    hs[0].synchronize()
    ref = oracle.bag_forward([h.forward for h in hs], w)(mix)
    err = np.abs(out.cpu().numpy().astype(np.float64) - ref).max()
    assert err <= 1e-6, err


def test_bag_device_entry_point_matches_host_entry_point():
    import torch
    import dmx

    hs = _handles([61, 62], max_batch=2)
    w = np.array([[1.0, 1.0, 0.0, 0.0], [0.0, 0.0, 1.0, 1.0]], dtype=np.float32)
    bag = dmx.Bag(hs, w)
    track = synth.pink_noise(39, int(44100 * 12))
    n = track.shape[1]
    ref = bag.separate_track(track[0], track[1], shifts=1, batch=2)
    lr = torch.from_numpy(track).cuda()
    stems = torch.full((4, 2, n), float("nan"), device="cuda")
    torch.cuda.synchronize()
    bag.separate_track_device(lr.data_ptr(), n, stems.data_ptr(), shifts=1, batch=2)
    hs[0].synchronize()
    err = np.abs(stems.cpu().numpy().astype(np.float64) - ref).max()
    assert err <= 1e-6, err


def test_bag_with_no_requested_stem_is_rejected():
    import dmx

    hs = _handles([71], max_batch=1)
    bag = dmx.Bag(hs, IDENTITY[:1], requested=[])
    track = synth.pink_noise(6, 44100)
    with pytest.raises(dmx.DmxError, match="no stem is requested") as e:
        bag.separate_track(track[0], track[1])
    assert e.value.code == 1
