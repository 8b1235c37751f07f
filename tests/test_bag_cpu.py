"""Bags of networks (htdemucs_ft) on CPU: the oracle's restatement of
BagCombineForward (api.rs:319-371) and the host logic of one network per GPU
group (shard.bag_assign / bag_gather), with gloo ranks and deterministic
stand-in networks (no GPU).
"""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

SEG = int(44100 * 0.25)
IDENTITY = np.eye(4, dtype=np.float32)
# a general matrix: network 3 carries nothing, stem 2 has two contributors
MIXED = np.array([[0.5, 0.0, 1.0, 0.0],
                  [0.0, 2.0, 0.25, 0.0],
                  [0.5, 0.0, 0.0, 1.0],
                  [0.0, 0.0, 0.0, 0.0]], dtype=np.float32)


def _net(k):
    """A deterministic, position-dependent stand-in for network k."""
    def forward(padded):
        g = padded.shape[0]
        out = np.repeat(padded[:, None], 4, axis=1) * np.float32(0.75 + 0.1 * k)
        out += np.float32(0.01) * np.roll(out, 5 + k, axis=-1)
        out *= (np.float32(1.0) + np.float32(0.05) * np.arange(4, dtype=np.float32))[None, :, None, None]
        return out.reshape(g, 4, 2, -1).astype(np.float32)
    return forward


def _track():
    i = np.arange(2 * (SEG * 7 + 123))
    return (np.sin(i * 0.0137) * 0.3 + ((i % 97) - 48) / 480.0).astype(np.float32).reshape(2, -1)


def _combine_np(outs, weights, requested):
    """The combination in numpy f32, as the oracle states it (api.rs:338-360)."""
    import oracle

    idx = [k for k, o in enumerate(outs) if o is not None]
    fwds = [(lambda x, o=o: o[None]) if o is not None else None for o in outs]
    like = outs[idx[0]]
    return oracle.bag_forward(fwds, weights, requested)(np.zeros((1,) + like.shape[1:], np.float32))[0]


def test_identity_bag_selects_each_networks_own_stem():
    import oracle

    x = _track()[None, :, :SEG]
    outs = [_net(k)(x) for k in range(4)]
    got = oracle.bag_forward([_net(k) for k in range(4)], IDENTITY)(x)
    for s in range(4):
        assert np.array_equal(got[:, s], outs[s][:, s])


def test_mixed_weights_combine_in_reference_order():
    import oracle

    x = _track()[None, :, :SEG]
    outs = [_net(k)(x).astype(np.float64) for k in range(4)]
    got = oracle.bag_forward([_net(k) for k in range(4)], MIXED)(x)
    for s in range(4):
        num = sum(MIXED[k, s] * outs[k][:, s] for k in range(4))
        np.testing.assert_allclose(got[:, s], num / MIXED[:, s].sum(), rtol=2e-6, atol=1e-7)


def test_only_networks_weighted_on_requested_stems_run():
    import oracle

    calls = []

    def counted(k):
        f = _net(k)
        return lambda x: (calls.append(k), f(x))[1]

    x = _track()[None, :, :SEG]
    got = oracle.bag_forward([counted(k) for k in range(4)], IDENTITY, requested=[1, 3])(x)
    assert calls == [1, 3]
    assert not got[:, 0].any() and not got[:, 2].any()
    uncovered = MIXED[:3] * np.array([1, 1, 1, 0], dtype=np.float32)
    with pytest.raises(ValueError, match="no network covers stem index 3"):
        oracle.bag_forward([_net(k) for k in range(3)], uncovered)(x)


def test_lockstep_bag_equals_per_network_separation_for_identity_weights():
    # api.rs:315-317: combining per segment before the overlap-add equals the
    # full-buffer combination of each network's separation (identity weights:
    # exactly, since every stem has a single contributor of weight 1)
    import oracle

    track = _track()
    bag = oracle.separate_with(oracle.bag_forward([_net(k) for k in range(4)], IDENTITY), track,
                               SEG, shifts=1)
    for k in range(4):
        single = oracle.separate_with(_net(k), track, SEG, shifts=1)
        assert np.array_equal(bag[k], single[k])


def test_bag_assignment_covers_each_running_network_once():
    import shard

    for world in (1, 2, 4, 8):
        seen = {}
        for r in range(world):
            a = shard.bag_assign(4, world, r, IDENTITY)
            for k in a.nets:
                seen.setdefault(k, set()).update(a.group)
            assert r in a.group
        assert sorted(seen) == [0, 1, 2, 3]
        if world >= 4:
            assert all(len(g) == world // 4 for g in seen.values())
    a = shard.bag_assign(4, 3, 0, MIXED)  # network 3 carries no weight
    assert shard.needed_nets(MIXED) == [0, 1, 2] and a.nets == [0]
    with pytest.raises(ValueError):
        shard.bag_assign(4, 6, 0, IDENTITY)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_stems(dist, shard, oracle, fwd, track, group, index):
    """One network's chunk-sharded separation over `group` (the host logic of
    the multi-GPU driver, as in test_shard_cpu); the group's first rank gets
    the (4, 2, n) stems."""
    import ctypes

    import torch

    n = track.shape[1]
    p = shard.plan(n, len(group), shifts=1, overlap=0.25, segment=SEG)
    mean, std = ctypes.c_float(), ctypes.c_float()
    oracle.lib().orc_scan_norm(oracle.ptr(track), 2, ctypes.c_int64(n), ctypes.byref(mean),
                               ctypes.byref(std))
    mix = ((track - np.float32(mean.value)) / np.float32(std.value)).astype(np.float32)
    weight = np.empty(SEG, np.float32)
    oracle.lib().orc_transition_weight(SEG, 1.0, oracle.ptr(weight))
    me = p.rank(index)
    acc = torch.zeros((8, p.view_length), dtype=torch.float32)
    a = acc.numpy()
    for c in range(me.chunk_lo, me.chunk_hi):
        vstart = c * p.stride
        length = min(p.view_length - vstart, SEG)
        padded = np.empty((2, SEG), np.float32)
        oracle.lib().orc_padded_chunk(oracle.ptr(mix), 2, ctypes.c_int64(n),
                                      ctypes.c_int64(p.offset), ctypes.c_int64(p.max_shift),
                                      ctypes.c_int64(vstart), ctypes.c_int64(length), SEG,
                                      oracle.ptr(padded))
        y = fwd(padded[None])[0].reshape(8, SEG)
        trim = (SEG - length) // 2
        a[:, vstart:vstart + length] += weight[None, :length] * y[:, trim:trim + length]
    shard.exchange_tails(dist, p, index, acc, ranks=group)
    stems = torch.zeros((8, n), dtype=torch.float32)
    s = stems.numpy()
    for t in range(me.t_lo, me.t_hi):
        v = t + p.trim
        sw = np.float32(0.0)
        for c in range(max(0, v // p.stride - 2), min(p.chunks, v // p.stride + 1)):
            u = v - c * p.stride
            if 0 <= u < min(p.view_length - c * p.stride, SEG):
                sw = np.float32(sw + weight[u])
        s[:, t] = (a[:, v] / sw) * np.float32(std.value) + np.float32(mean.value)
    shard.gather_stems(dist, p, index, stems, ranks=group)
    return stems.reshape(4, 2, n)


def _worker(rank, world, port, weights, requested, out_path):
    import datetime
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "demucs-wgpu_b200"), os.path.join(root, "oracle")]
    import oracle
    import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    track = _track()
    assign = shard.bag_assign(len(weights), world, rank, weights, requested)
    mine = {}
    for k in assign.nets:
        if len(assign.group) == 1:
            mine[k] = torch.from_numpy(oracle.separate_with(_net(k), track, SEG, shifts=1))
        else:
            st = _shard_stems(dist, shard, oracle, _net(k), track, assign.group, assign.index)
            if assign.index == 0:
                mine[k] = st

    def combine(outs, w, req):
        return torch.from_numpy(_combine_np([o.numpy() if o is not None else None for o in outs],
                                            w, req))

    like = torch.zeros((4, 2, track.shape[1]), dtype=torch.float32)
    got = shard.bag_gather(dist, rank, assign, mine, weights, requested, combine, like)
    if rank == 0:
        np.save(out_path, got.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,weights,requested,atol", [
    (2, IDENTITY, None, 0.0),    # two whole networks per rank
    (4, IDENTITY, [0, 3], 2e-6),  # two requested stems: one network per pair of ranks
    (3, MIXED, None, 2e-6),      # three running networks, one per rank, general weights
])
def test_bag_over_ranks_matches_lockstep_oracle(world, weights, requested, atol, tmp_path):
    import oracle

    out_path = str(tmp_path / "bag.npy")
    mp.start_processes(_worker, args=(world, _free_port(), weights, requested, out_path),
                       nprocs=world, join=True, start_method="spawn")
    got = np.load(out_path)
    ref = oracle.separate_with(oracle.bag_forward([_net(k) for k in range(4)], weights, requested),
                               _track(), SEG, shifts=1)
    req = range(4) if requested is None else requested
    for s in req:
        np.testing.assert_allclose(got[s], ref[s], rtol=0, atol=atol)
