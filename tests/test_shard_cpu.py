"""Multi-rank chunk sharding of one track, on CPU with gloo (no GPU).

Two (and three) ranks each overlap-add their contiguous chunk range with a
deterministic stand-in forward, exchange the boundary tails, finalise the
samples they own and gather them to rank 0 — the host logic of the multi-GPU
path in bench.py (shard.py) — and rank 0's stems must equal the oracle's
single-process driver (streaming.rs:296-400, pipeline.rs:380-515) on the same
track.
"""

import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

SEG = int(44100 * 0.25)


def _forward(padded):
    # a deterministic, position-dependent stand-in for the network
    g = padded.shape[0]
    out = np.repeat(padded[:, None], 4, axis=1) * np.float32(0.75)
    out += np.float32(0.01) * np.roll(out, 5, axis=-1)
    return out.reshape(g, 4, 2, -1).astype(np.float32)


def _track():
    i = np.arange(2 * (SEG * 7 + 123))
    return (np.sin(i * 0.0137) * 0.3 + ((i % 97) - 48) / 480.0).astype(np.float32).reshape(2, -1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path):
    import datetime
    import sys

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
    n = track.shape[1]
    p = shard.plan(n, world, shifts=1, overlap=0.25, segment=SEG)
    mean, std = ctypes.c_float(), ctypes.c_float()
    oracle.lib().orc_scan_norm(oracle.ptr(track), 2, ctypes.c_int64(n), ctypes.byref(mean),
                               ctypes.byref(std))
    mix = ((track - np.float32(mean.value)) / np.float32(std.value)).astype(np.float32)
    weight = np.empty(SEG, np.float32)
    oracle.lib().orc_transition_weight(SEG, 1.0, oracle.ptr(weight))
    me = p.rank(rank)
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
        y = _forward(padded[None])[0].reshape(8, SEG)
        trim = (SEG - length) // 2
        a[:, vstart:vstart + length] += weight[None, :length] * y[:, trim:trim + length]
    shard.exchange_tails(dist, p, rank, acc)
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
    shard.gather_stems(dist, p, rank, stems)
    if rank == 0:
        np.save(out_path, stems.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_track_matches_single_process_driver(world, tmp_path):
    import oracle

    out_path = str(tmp_path / "stems.npy")
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, out_path), nprocs=world, join=True,
                       start_method="spawn")
    got = np.load(out_path).reshape(4, 2, -1)
    ref = oracle.separate_with(_forward, _track(), SEG, shifts=1)
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6)


def test_plan_rejects_overlaps_of_half_a_segment_or_more():
    # the boundary exchange assumes stride > segment / 2: with more overlap a rank's tail
    # can reach past its neighbour's own span (and a sample gets three contributions)
    import pytest

    import shard

    for overlap in (0.5, 0.6, 0.9):
        with pytest.raises(ValueError, match="overlap < 0.5"):
            shard.plan(10_584_000, 8, shifts=1, overlap=overlap)
    shard.plan(10_584_000, 8, shifts=1, overlap=0.49)


def test_plan_partitions_every_chunk_once():
    import shard

    for world in (1, 2, 3, 8):
        p = shard.plan(10_584_000, world, shifts=1)
        assert p.chunks == 42
        covered = [c for r in p.ranks for c in range(r.chunk_lo, r.chunk_hi)]
        assert covered == list(range(42))
        assert p.ranks[0].t_lo == 0 and p.ranks[-1].t_hi == 10_584_000
        for a, b in zip(p.ranks, p.ranks[1:]):
            assert a.t_hi == b.t_lo and a.own_hi == b.own_lo
            assert a.send_hi - a.send_lo <= p.segment - p.stride


def _fault_worker(rank, world, port, store_port, out_path):
    # rank 0 "dies" between steps: it skips the boundary exchange, so rank 1's
    # receive never completes and its bounded wait must end in ShardTimeout
    import datetime
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "demucs-wgpu_b200")]
    import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", store_port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    p = shard.plan(SEG * 7 + 123, world, shifts=1, overlap=0.25, segment=SEG)
    acc = torch.zeros((8, p.view_length), dtype=torch.float32)
    if rank == 1:
        try:
            shard.exchange_tails(dist, p, rank, acc, timeout=2.0)
            result = "completed"
        except shard.ShardTimeout as exc:
            result = f"timeout {exc.code}"
        with open(out_path, "w") as f:
            f.write(result)
        store.set("rank1_done", "1")
    else:
        store.wait(["rank1_done"], datetime.timedelta(seconds=60))
    # the unmatched receive is still posted on rank 1: leave without a collective
    os._exit(0)


def test_missing_boundary_send_ends_in_a_bounded_timeout(tmp_path):
    out_path = str(tmp_path / "fault.txt")
    mp.start_processes(_fault_worker, args=(2, _free_port(), _free_port(), out_path), nprocs=2,
                       join=True,
                       start_method="spawn")
    assert open(out_path).read() == "timeout 4"


def test_track_assignment_balances_units_and_covers_every_track():
    import shard

    # 64 tracks of 180 s with shifts 2 (the throughput batch): 8 per GPU
    lengths = [180 * 44100] * 64
    per = shard.assign_tracks(lengths, 8, shifts=2)
    assert sorted(i for r in per for i in r) == list(range(64))
    assert [len(r) for r in per] == [8] * 8
    units = shard.track_units(180 * 44100, 2)
    assert units == 2 * 31  # 31 chunks per shift pass
    # ragged lengths: no rank carries more than the lightest rank plus one longest track
    rng = np.random.default_rng(3)
    lengths = [int(x) for x in rng.integers(5 * 44100, 400 * 44100, size=37)]
    per = shard.assign_tracks(lengths, 6, shifts=1)
    loads = [sum(shard.track_units(lengths[i], 1) for i in r) for r in per]
    assert sorted(i for r in per for i in r) == list(range(37))
    assert max(loads) - min(loads) <= max(shard.track_units(n, 1) for n in lengths)


def _tracks_worker(rank, world, port, out_path):
    # the throughput batch over ranks: each rank separates its share of the tracks (here
    # with the oracle driver over a stand-in forward), rank 0 gathers every track's stems
    import datetime
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "demucs-wgpu_b200"), os.path.join(root, "oracle")]
    import oracle
    import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    lengths = [SEG * k + 17 * k for k in (1, 5, 2, 7, 3)]
    tracks = [_track()[:, :n].copy() for n in lengths]
    per_rank = shard.assign_tracks(lengths, world, shifts=2)
    mine = {i: torch.from_numpy(oracle.separate_with(_forward, tracks[i], SEG, shifts=2))
            for i in per_rank[rank]}
    got = shard.gather_tracks(dist, rank, per_rank, mine, lengths, timeout=30)
    if rank == 0:
        np.savez(out_path, *[got[i].numpy() for i in range(len(lengths))])
    dist.barrier()
    dist.destroy_process_group()


def test_tracks_over_ranks_gather_to_rank0(tmp_path):
    import oracle

    out_path = str(tmp_path / "tracks.npz")
    mp.start_processes(_tracks_worker, args=(3, _free_port(), out_path), nprocs=3, join=True,
                       start_method="spawn")
    got = np.load(out_path)
    lengths = [SEG * k + 17 * k for k in (1, 5, 2, 7, 3)]
    for i, n in enumerate(lengths):
        ref = oracle.separate_with(_forward, _track()[:, :n].copy(), SEG, shifts=2)
        assert np.array_equal(got[f"arr_{i}"], ref)


def _peer_fail_worker(rank, world, port, out_dir):
    # no GPU here, so exporting a device buffer fails on every rank: each rank must
    # still join the handle exchange and then raise, none may be left waiting
    import datetime
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "demucs-wgpu_b200")]
    import shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        shard.PeerBuffers(dist, 0, 0x1000)
        result = "mapped"
    except RuntimeError as exc:
        result = "raised: " + str(exc).split(":")[0]
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(result)
    dist.barrier()
    dist.destroy_process_group()


def test_peer_buffer_setup_fails_on_every_rank_together(tmp_path):
    mp.start_processes(_peer_fail_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        assert open(tmp_path / f"rank{r}.txt").read() == "raised: peer buffer export failed"
