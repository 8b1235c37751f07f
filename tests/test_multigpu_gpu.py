"""Chunk-sharded separation over 2, 4 or 8 GPUs (NCCL) reproduces the 1-GPU result.

Each rank forwards its contiguous chunk range (dmx_track_shard), the boundary
tail crosses to the neighbour, each rank finalises the samples it owns
(dmx_track_finish) and rank 0 gathers the stems, which are compared with
dmx_separate_track on one GPU. Each rank count runs when that many GPUs are
visible.

The single-process multi-GPU entry point (dmx_separate_track_multi) is tested
with 2-4 handles placed on the visible GPUs in turn, so it also runs on one GPU.

Both must match bit for bit: a segment's forward output does not depend on
which chunks share its forward (every per-segment moment is reduced in an
order fixed by the position inside the segment), and every overlap-add sample
has at most two contributions, whose IEEE sum is the same in either order.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SECONDS = 21


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path, mode="nccl"):
    import datetime
    import sys

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "demucs-wgpu_b200"))
    import dmx
    import shard
    import synth

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device(f"cuda:{rank}"))
    n = 44100 * max(SECONDS, 6 * world)  # at least one chunk per rank
    track = synth.pink_noise(7, n)
    p = shard.plan(n, world, shifts=1)
    me = p.rank(rank)
    h = dmx.Handle(synth.write_safetensors(synth.random_weights(3)), device=rank, max_batch=4,
                   precision=dmx.TF32)
    stream = torch.cuda.ExternalStream(h.stream, device=f"cuda:{rank}")
    dist.barrier()
    with torch.cuda.stream(stream):
        lr = torch.from_numpy(track).cuda()
        mix_norm = torch.empty_like(lr)
        ms = torch.empty(2, device="cuda")
        acc = torch.zeros((8, p.view_length), device="cuda")
        stems = torch.zeros((8, n), device="cuda")
        flag = torch.zeros(1, device="cuda")
    h.synchronize()
    peers_acc = peers_stems = None
    if mode == "peer":
        peers_acc = shard.PeerBuffers(dist, rank, acc.data_ptr())
        peers_stems = shard.PeerBuffers(dist, rank, stems.data_ptr())
    for _ in range(2):  # twice: the second step reuses every buffer (the barriers order it)
        with torch.cuda.stream(stream):
            h.normalize_track_device(lr.data_ptr(), n, mix_norm.data_ptr(), ms.data_ptr())
            acc.zero_()
            h.track_shard(mix_norm.data_ptr(), n, p.offset, p.max_shift, 0.25, me.chunk_lo,
                          me.chunk_hi, 4, acc.data_ptr(), 0, p.view_length)
            if mode == "peer":
                shard.exchange_tails_peer(dist, p, rank, h, acc.data_ptr(), peers_acc, flag)
            else:
                shard.exchange_tails(dist, p, rank, acc)
            h.track_finish(acc.data_ptr(), n, p.offset, p.max_shift, 0.25, 1, ms.data_ptr(),
                           stems.data_ptr(), me.t_lo, me.t_hi)
            if mode == "peer":
                shard.gather_stems_peer(dist, p, rank, h, stems.data_ptr(), peers_stems, flag)
            else:
                shard.gather_stems(dist, p, rank, stems)
    h.synchronize()
    torch.cuda.synchronize()
    if rank == 0:
        single = h.separate_track(track[0], track[1], shifts=1)
        np.save(out_path, np.stack([stems.cpu().numpy().reshape(4, 2, n), single]))
    dist.barrier()
    if peers_acc is not None:
        peers_acc.close()
        peers_stems.close()
    dist.barrier()
    h.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "peer"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharding_over_gpus_matches_one_gpu(world, mode, tmp_path):
    # mode nccl: boundary tails and stems as NCCL point-to-point messages; mode peer:
    # every rank maps its neighbours' buffers (CUDA IPC) and reads them over NVLink
    # between on-stream barriers
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out_path = str(tmp_path / "stems.npy")
    mp.start_processes(_worker, args=(world, _free_port(), out_path, mode), nprocs=world,
                       join=True, start_method="spawn")
    sharded, single = np.load(out_path)
    assert np.isfinite(sharded).all()
    assert np.array_equal(sharded, single)


@pytest.mark.parametrize("ranks,shifts,batch", [(2, 1, 2), (3, 0, 1), (4, 1, 4)])
def test_single_process_multi_handle_driver_matches_one_handle(ranks, shifts, batch):
    # dmx_separate_track_multi with every rank's handle on GPU 0 (or spread over the
    # visible GPUs): the chunk split, the peer-copied boundary tails and the per-rank
    # finish must reproduce dmx_separate_track; ranks without chunks (4 ranks, 3 chunks)
    # contribute nothing
    import dmx
    import synth

    gpus = torch.cuda.device_count()
    blob = synth.write_safetensors(synth.random_weights(5))
    hs = [dmx.Handle(blob, device=k % gpus, max_batch=2, precision=dmx.TF32) for k in range(ranks)]
    seconds = 14 if ranks == 4 else 21
    track = synth.pink_noise(8, 44100 * seconds)
    got = dmx.separate_track_multi(hs, track[0], track[1], shifts=shifts, batch=batch)
    ref = hs[0].separate_track(track[0], track[1], shifts=shifts, batch=batch)
    assert np.isfinite(got).all()
    assert np.array_equal(got, ref)
    for h in hs:
        h.close()
