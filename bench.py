"""Benchmark: audio-seconds separated per second by the B200 HTDemucs v4 backend.

Workload (the full-track htdemucs configuration of the benchmark): one 240 s stereo
44.1 kHz seeded pink-noise track (RMS 0.1), 7.8 s segments, overlap 0.25,
shifts 1 (ShiftRng seed 0x5eed1234), all chunks of the track batched into one
forward; random-init weights (seeded, LayerScale 1e-4). A step is one
whole-track separation. With N GPUs the track's chunks are sharded
contiguously over the ranks (strong scaling: the total work is fixed); the
only exchange is the overlap-add boundary between neighbouring shards plus
the final gather of the stems to rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0). ``--impl reference`` times the reference's CPU
path — here the C++ restatement under oracle/, since the Rust reference cannot
be built in this environment — on all host cores: its whole-track driver on a
two-chunk prefix of the workload's track per step, credited with the prefix's
audio seconds.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "demucs-wgpu_b200"))

import synth  # noqa: E402

TRACK_SECONDS = 240.0
SR = 44100
SEGMENT = synth.SEGMENT_SAMPLES
SEGMENT_GFLOP = 334.9  # algorithmic FLOPs of one segment forward (2*MAC over the layer table)
METRIC = "audio-sec separated/sec (htdemucs)"
UNIT = "audio-s/s"
# Measured DRAM bytes (read + write) per algorithmic byte for a kernel tag and
# build, from one ncu capture of that kernel (profiles/): roofline.traffic =
# ratio x the tag's algorithmic bytes per launch. The attention captures are the
# layer-0 spectral self-attention on a 3-chunk track: tf32, 50.4 MB of DRAM
# traffic for 66.1 MB of q, k, v, o; bf16, 24.8 MB for 33.0 MB. Traffic scales
# with the chunks a launch processes.
TRAFFIC_RATIO = {("xf.attention", "TF32"): 50.393 / 66.060,
                 ("xf.attention", "BF16"): 24.810 / 33.030}


def workload(seconds):
    return (f"full-track htdemucs: {seconds:g} s stereo 44.1 kHz pink noise (RMS 0.1), segment 7.8 s, "
            "overlap 0.25, shifts 1, all chunks batched")


def track_config(seconds):
    """The workload both arms report (the reference arm and ours share it)."""
    import shard

    n = int(seconds * SR)
    p = shard.plan(n, 1, shifts=1, overlap=0.25)
    return {"workload": workload(seconds), "track_samples": n, "chunks_per_step": p.chunks,
            "segment_samples": SEGMENT, "shifts": 1, "overlap": 0.25, "seed": 2024,
            "weights": "random init, seed 0, LayerScale 1e-4",
            "l2": "inputs and workspace larger than L2 (126 MB)"}


def _oracle_threads():
    """All host threads for the CPU legs (torchrun sets OMP_NUM_THREADS=1 for every rank;
    only rank 0 runs these legs, so it takes the whole host)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    return oracle, oracle.threads(os.cpu_count() or 1)


def _prefix_samples(chunks):
    """A prefix of the benchmark track whose shift-1 view holds exactly `chunks` chunks:
    the oracle's driver on it does `chunks` segment forwards, as the workload does
    per chunk (the prefix is credited with its own audio seconds)."""
    import shard

    stride = int(0.75 * SEGMENT)
    trim = shard.plan(SEGMENT, 1, shifts=1).trim
    return chunks * stride - trim


def _peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, "measured"|"fallback")."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return (d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "measured")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def roofline(stages, precision):
    """Roofline of the dominant kernel tag (most device time in the step).

    ``stages``: {tag: (ms, launches, flops, bytes)} from the runtime's
    per-launch accounting (algorithmic FLOPs, minimum HBM bytes), timed per
    launch with CUDA events on the handle's stream. Each launch lasts well
    under a second, so the tensor peak is the measured bf16 burst figure; the
    fraction of the sustained figure and of a tf32 rate (half the bf16 one,
    the datasheet ratio) are given beside it."""
    hbm, bf16_burst, bf16_sustained, kind = _peaks()
    tag, (ms, launches, flops, nbytes) = max(stages.items(), key=lambda kv: kv[1][0])
    s = ms / 1e3
    intensity = flops / nbytes if nbytes else float("inf")
    ridge = bf16_burst * 1e12 / (hbm * 1e9)
    extra = {}
    if flops > 0 and intensity >= ridge:
        bound, achieved, peak, unit = "tensor", flops / s / 1e12, bf16_burst, "TFLOP/s"
        extra = {"frac_of_bf16_sustained": round(achieved / bf16_sustained, 5),
                 "frac_of_tf32_equivalent": round(achieved / (bf16_burst / 2), 5),
                 "note": "tf32-equivalent peak = half the measured bf16 burst (datasheet tf32:bf16 "
                         "dense ratio), not itself measured"}
    else:
        bound, achieved, peak, unit = "hbm", nbytes / s / 1e9, hbm, "GB/s"
    ratio = TRAFFIC_RATIO.get((tag, precision))
    traffic = round(ratio * nbytes / max(launches, 1)) if ratio else None
    out = {"bound": bound, "achieved": round(achieved, 3), "peak": peak, "unit": unit,
           "frac": round(achieved / peak, 5), "traffic": traffic,
           "kernel": tag, "launches": launches,
           "flops_per_launch": flops / max(launches, 1), "bytes_per_launch": nbytes / max(launches, 1),
           "arith_intensity": round(intensity, 2) if nbytes else None,
           "peak_kind": f"{kind} ({'bf16 dense burst' if unit == 'TFLOP/s' else 'HBM copy'})"}
    out.update(extra)
    return out


def build_leg(track_dev, n, chunks, dev, precision, gate, steps=2):
    """Another build on the same workload, device-timed with CUDA events: the
    fp32-accurate tensor-core build (TF32X3, the max-abs 1e-4 gate) and the other
    SNR >= 60 dB build (TF32 beside the BF16 headline, or BF16 beside TF32)."""
    import torch
    import dmx

    h = dmx.Handle(synth.write_safetensors(synth.random_weights(0)), device=dev, max_batch=chunks,
                   precision=getattr(dmx, precision))
    stems = torch.empty((4, 2, n), dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.ExternalStream(h.stream, device=f"cuda:{dev}")
    torch.cuda.synchronize()
    h.separate_track_device(track_dev.data_ptr(), n, stems.data_ptr(), shifts=1, batch=chunks)
    h.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        h.separate_track_device(track_dev.data_ptr(), n, stems.data_ptr(), shifts=1, batch=chunks)
    end.record(stream)
    h.synchronize()
    ms = start.elapsed_time(end) / steps
    del stems
    torch.cuda.empty_cache()
    h.close()
    return {"precision": precision, "value": round(n / SR / (ms / 1e3), 3), "unit": UNIT,
            "ms_per_step": round(ms, 3), "steps": steps, "warmup": 1, "gate": gate}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


def cpu_baseline(seconds_budget=30.0):
    """The oracle (C++ restatement of the reference CPU path) on all host threads: its own
    whole-track driver (normalise, shift view, chunks, forwards, overlap-add) on a prefix of
    the benchmark track holding two chunks, 1 warm-up + up to 2 timed within the budget."""
    oracle, threads = _oracle_threads()
    w = synth.random_weights(0)
    m = oracle.OracleModel(w)
    n = _prefix_samples(2)
    track = synth.pink_noise(2024, int(TRACK_SECONDS * SR))[:, :n].copy()
    m.separate(track, shifts=1, batch=2)
    times = []
    t_all = time.perf_counter()
    while len(times) < 2 and time.perf_counter() - t_all < seconds_budget:
        t0 = time.perf_counter()
        m.separate(track, shifts=1, batch=2)
        times.append(time.perf_counter() - t0)
    t = float(np.median(times))
    return {"value": round(n / SR / t, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"the oracle's whole-track driver on the first {n} samples ({n / SR:.2f} s, "
                       f"2 chunks of the workload's shift-1 view) of the benchmark track, median of "
                       f"{len(times)} after 1 warm-up, {t:.2f} s each")}


def run_reference(args, rank, world):
    if rank != 0:
        return
    oracle, threads = _oracle_threads()
    w = synth.random_weights(0)
    m = oracle.OracleModel(w)
    # each step: the oracle's own track driver on a whole-chunk prefix of the workload
    chunks = max(1, args.ref_chunks)
    n = _prefix_samples(chunks)
    track = synth.pink_noise(2024, int(args.seconds * SR))[:, :n].copy()
    for _ in range(args.warmup):
        m.separate(track, shifts=1, batch=chunks)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.separate(track, shifts=1, batch=chunks)
    dt = (time.perf_counter() - t0) / args.steps
    value = n / SR / dt
    sample = (f"oracle/ C++ restatement of the reference CPU path (the Rust reference is not "
              f"buildable here): its whole-track driver (normalise, ShiftRng view, {chunks} "
              f"chunks, forwards, overlap-add, denormalise) on the first {n} samples "
              f"({n / SR:.2f} s) of the workload's track per step, credited with those seconds")
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": track_config(args.seconds),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class SharedHostStems:
    """(8, n) float32 host stems in a shared-memory file that every rank maps and
    registers as pinned memory: each rank copies its own span of the result over its
    own PCIe link, and the whole result is in host memory once all ranks are done
    (the multi-process counterpart of dmx_separate_track_multi's per-rank copies)."""

    def __init__(self, dist, rank, n):
        import torch

        self.path = f"/dev/shm/dmx_bench_{os.environ.get('MASTER_PORT', '0')}_stems"
        self.rank = rank
        nbytes = 8 * n * 4
        if rank == 0:
            with open(self.path, "wb") as f:
                f.truncate(nbytes)
        dist.barrier()
        self.array = np.memmap(self.path, dtype=np.float32, mode="r+", shape=(8, n))
        self.tensor = torch.from_numpy(self.array)
        rc = torch.cuda.cudart().cudaHostRegister(self.tensor.data_ptr(), nbytes, 0)
        self.registered = int(rc) == 0

    def close(self, dist):
        import torch

        if self.registered:
            torch.cuda.cudart().cudaHostUnregister(self.tensor.data_ptr())
        del self.tensor
        del self.array
        dist.barrier()
        if self.rank == 0:
            os.unlink(self.path)


def _event_ms(torch, events):
    return [round(a.elapsed_time(b), 3) for a, b in zip(events, events[1:])]


def run_ours(args, rank, world, local_rank):
    import datetime

    import torch
    import dmx
    import shard

    dev = local_rank
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device(f"cuda:{dev}"))
    if args.workload == "bag":
        return run_bag(args, rank, world, dev, dist)
    if args.workload == "batch":
        return run_batch(args, rank, world, dev, dist)
    seconds = args.seconds
    n = int(seconds * SR)
    track = synth.pink_noise(2024, n)
    shifts, overlap = 1, 0.25
    p = shard.plan(n, world, shifts=shifts, overlap=overlap)
    me = p.rank(rank)
    mine = me.chunk_hi - me.chunk_lo
    weights = synth.random_weights(0)
    blob = synth.write_safetensors(weights)
    h = dmx.Handle(blob, device=dev, max_batch=max(1, mine if world > 1 else p.chunks),
                   precision=getattr(dmx, args.precision))
    stream = torch.cuda.ExternalStream(h.stream, device=f"cuda:{dev}")
    cuda = f"cuda:{dev}"
    # buffers come from torch's allocator on its default stream and are only
    # used on the handle's stream after a synchronize; they are released before
    # the handle (and its stream) is destroyed
    lr = torch.from_numpy(track).to(cuda).contiguous()
    stems = torch.zeros((4, 2, n), dtype=torch.float32, device=cuda)
    mix_norm = mean_std = acc = None
    if world > 1:
        mix_norm = torch.empty_like(lr)
        mean_std = torch.empty(2, dtype=torch.float32, device=cuda)
        acc = torch.empty((8, p.view_length), dtype=torch.float32, device=cuda)
        flag = torch.zeros(1, dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    peers_acc = peers_stems = None
    exchange = args.exchange if world > 1 else None
    if exchange == "peer":
        # every rank maps its neighbours' accumulator and stems (CUDA IPC): the boundary
        # tail and the gather are SM loads over NVLink between on-stream barriers. If any
        # rank cannot map them, every rank uses the NCCL exchange instead (the decision
        # is collective, so all ranks take the same path)
        err = ""
        try:
            peers_acc = shard.PeerBuffers(dist, dev, acc.data_ptr())
            peers_stems = shard.PeerBuffers(dist, dev, stems.data_ptr())
        except Exception as exc:  # mapping refused by the driver or the platform
            err = f"{type(exc).__name__}: {exc}"
        failed = torch.tensor([1.0 if err else 0.0], device=cuda)
        dist.all_reduce(failed, op=dist.ReduceOp.MAX)
        if failed.item() > 0:
            for pb in (peers_acc, peers_stems):
                if pb is not None:
                    pb.close()
            peers_acc = peers_stems = None
            exchange = "nccl (peer mapping failed" + (f": {err[:120]}" if err else " on another rank") + ")"
    phase_events = None  # set to a list to record (start, forward, exchange, finish, gather)

    def mark():
        if phase_events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            phase_events.append(e)

    def shard_step(gather=True):
        with torch.cuda.stream(stream):
            mark()
            h.normalize_track_device(lr.data_ptr(), n, mix_norm.data_ptr(), mean_std.data_ptr())
            if mine:
                acc[:, me.span_lo:me.span_hi].zero_()  # the only part of the view this rank writes
                h.track_shard(mix_norm.data_ptr(), n, p.offset, p.max_shift, overlap, me.chunk_lo,
                              me.chunk_hi, mine, acc.data_ptr(), 0, p.view_length)
            mark()
            if peers_acc is not None:
                shard.exchange_tails_peer(dist, p, rank, h, acc.data_ptr(), peers_acc, flag)
            else:
                shard.exchange_tails(dist, p, rank, acc)
            mark()
            if me.t_hi > me.t_lo:
                h.track_finish(acc.data_ptr(), n, p.offset, p.max_shift, overlap, shifts,
                               mean_std.data_ptr(), stems.data_ptr(), me.t_lo, me.t_hi)
            mark()
            if gather and peers_stems is not None:
                shard.gather_stems_peer(dist, p, rank, h, stems.data_ptr(), peers_stems, flag)
            elif gather:
                shard.gather_stems(dist, p, rank, stems.view(8, n))
            elif peers_acc is not None:
                shard.device_barrier(dist, flag)  # the neighbour's tail read is done before reuse
            mark()

    def step():
        if world == 1:
            h.separate_track_device(lr.data_ptr(), n, stems.data_ptr(), shifts=shifts,
                                    overlap=overlap, batch=p.chunks)
            return
        shard_step()

    def barrier():
        if dist is not None:
            dist.barrier()

    barrier()
    for _ in range(args.warmup):
        step()
    h.synchronize()
    torch.cuda.synchronize()
    before = h.kernel_launches()
    step()
    h.synchronize()
    launches = h.kernel_launches() if world == 1 else h.kernel_launches() - before
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        h.synchronize()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    if dist is not None:
        t = torch.tensor([ms], device=cuda)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = seconds / (ms / 1e3)

    # N > 1: where one step's time goes on each rank (one more, untimed step)
    phases = None
    if world > 1:
        phase_events = []
        barrier()
        step()
        h.synchronize()
        torch.cuda.synchronize()
        mine_ms = torch.tensor(_event_ms(torch, phase_events), device=cuda)
        phase_events = None
        everyone = [torch.empty_like(mine_ms) for _ in range(world)]
        dist.all_gather(everyone, mine_ms)
        phases = {"unit": "ms", "order": ["normalise+forward+overlap-add", "boundary exchange",
                                          "finish", "gather to rank 0"],
                  "per_rank": [[round(float(x), 3) for x in t.cpu()] for t in everyone]}

    # e2e through the public host API
    pin = torch.from_numpy(track).pin_memory()
    e2e_batch = p.chunks
    if world == 1:
        # pinned host track in, pinned host stems out: the host entry point copies finished
        # stems back while later forwards run. Forwards of e2e_batch chunks: one large forward
        # and a short last one (about a tenth of the chunks), so most of the stems copy back
        # while the last forward runs and the copy left after it is short (measured on B200:
        # 38 + 4 chunks 3416 audio-s/s, 21 + 21 3390, 14 x 3 2861)
        out_pin = torch.empty((4, 2, n), dtype=torch.float32).pin_memory()
        e2e_batch = args.e2e_batch or max(1, p.chunks - max(1, p.chunks // 10))
        left, right, out_np = pin[0].numpy(), pin[1].numpy(), out_pin.numpy()
        h.separate_track(left, right, shifts=shifts, overlap=overlap, batch=e2e_batch, out=out_np)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            h.separate_track(left, right, shifts=shifts, overlap=overlap, batch=e2e_batch, out=out_np)
        e2e_s = (time.perf_counter() - t0) / args.steps
        e2e_api = "dmx_separate_track (pinned host track in, pinned host stems out)"
        h2d, d2h = 2 * n * 4, 8 * n * 4
        del out_pin
    else:
        # every rank copies the track in from its pinned host memory and its own span of the
        # finished stems out into shared pinned host memory (no device gather)
        host = SharedHostStems(dist, rank, n)

        def e2e_step():
            with torch.cuda.stream(stream):
                lr.copy_(pin, non_blocking=True)
            shard_step(gather=False)
            with torch.cuda.stream(stream):
                flat = stems.view(8, n)
                for row in range(8):
                    host.tensor[row, me.t_lo:me.t_hi].copy_(flat[row, me.t_lo:me.t_hi],
                                                            non_blocking=True)
            h.synchronize()
        e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        barrier()
        t = torch.tensor([(time.perf_counter() - t0) / args.steps], device=cuda)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        e2e_api = ("per rank: track copied in from pinned host memory, its chunk shard, boundary "
                   "exchange, its span of the stems copied out into shared pinned host memory "
                   f"(registered: {host.registered})")
        h2d, d2h = 2 * n * 4 * world, 8 * n * 4
        host.close(dist)

    # N > 1: rank 0 separates the same track alone (one handle, the same build) and the
    # gathered stems must equal it bit for bit (batch-invariant forward, exact OLA merge)
    match = None
    if world > 1:
        step()  # the device path again: stems gathered on rank 0
        h.synchronize()
        if rank == 0:
            with torch.cuda.stream(stream):
                alone = torch.empty_like(stems)
            h.synchronize()
            torch.cuda.synchronize()
            h.separate_track_device(lr.data_ptr(), n, alone.data_ptr(), shifts=shifts,
                                    overlap=overlap, batch=max(1, mine))
            h.synchronize()
            match = bool(torch.equal(alone, stems))
            del alone

    # per-kernel device timing of one more (untimed) step for the roofline
    h.set_stage_timing(True)
    step()
    h.synchronize()
    stages = h.stage_times(work=True)
    h.set_stage_timing(False)
    _, _, bf16_sustained, _ = _peaks()
    total_ms = sum(v[0] for v in stages.values()) or 1.0
    whole = SEGMENT_GFLOP * 1e9 * (me.chunk_hi - me.chunk_lo) / (ms / 1e3) / 1e12  # this GPU
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": {"FP32": "f32", "TF32": "tf32", "TF32X3": "tf32x3",
                      "BF16": "bf16 (transformer linears and attention), tf32 (convolutions and DConv)"}[args.precision],
            "data": "synthetic",
            "config": track_config(seconds),
            "precision": args.precision,
            "parallelism": f"chunk-sharded x{world}" + (
                f", boundary tail and stem gather over NVLink ({exchange})" if world > 1 else ""),
            "chunks_per_gpu": [r.chunk_hi - r.chunk_lo for r in p.ranks],
            "e2e": {"value": round(seconds / e2e_s, 3), "unit": UNIT,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "chunks_per_forward": e2e_batch, "api": e2e_api},
            "gpu_launches": int(launches) * args.steps,
            "clocks": clocks.summary(),
            "roofline": roofline(stages, args.precision),
            "whole_forward": {"achieved": round(whole, 3), "unit": "TFLOP/s",
                              "frac_of_bf16_sustained": round(whole / bf16_sustained, 5),
                              "note": "334.9 GFLOP per segment over the whole step, rank 0's chunks"},
            "kernels": {k: {"ms": round(v[0], 3), "launches": v[1], "share": round(v[0] / total_ms, 4),
                            "tflops": round(v[2] / (v[0] / 1e3) / 1e12, 2) if v[0] else None,
                            "gbs": round(v[3] / (v[0] / 1e3) / 1e9, 1) if v[0] else None}
                        for k, v in sorted(stages.items(), key=lambda kv: -kv[1][0])}}
    if phases is not None:
        line["phases"] = phases
    if match is not None:
        line["stems_match_1gpu"] = match
    if world == 1 and args.precision in ("TF32", "BF16") and not args.no_fp32_class:
        line["fp32_class"] = build_leg(lr, n, p.chunks, dev, "TF32X3",
                                       "per-stem max-abs <= 1e-4 vs the oracle (tests/test_track_gpu.py)")
        other = "TF32" if args.precision == "BF16" else "BF16"
        line[other.lower() + "_build"] = build_leg(
            lr, n, p.chunks, dev, other,
            "per-stem SNR >= 60 dB vs the oracle (tests/test_track_gpu.py, tests/test_tf32_gpu.py)",
            steps=3)
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    h.synchronize()
    torch.cuda.synchronize()
    if peers_acc is not None:
        dist.barrier()  # no rank unmaps while another may still read
        peers_acc.close()
        peers_stems.close()
        dist.barrier()
    del lr, stems, mix_norm, mean_std, acc, pin
    torch.cuda.empty_cache()
    h.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _timed(torch, stream, dev, dist, step, steps, warmup):
    """W warm-up steps, then K steps between events on `stream`, max over ranks (ms)."""
    cuda = f"cuda:{dev}"
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clocks:
        start.record(stream)
        for _ in range(steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if dist is not None:
        t = torch.tensor([ms], device=cuda)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clocks.summary()


def run_bag(args, rank, world, dev, dist):
    """htdemucs_ft bag (the bag configuration of the benchmark): four independently
    seeded networks, identity weights (network k gives stem k), one 240 s pink-noise
    track, shifts 0. One GPU: the lockstep bag driver (every network forwards each
    chunk batch, combined before the overlap-add). Fewer GPUs than networks: whole
    networks per GPU. 4 GPUs: one network per GPU. 8 GPUs: one network per GPU pair,
    its chunks sharded inside the pair. The weighted stem lanes meet on rank 0, which
    combines them (dmx_bag_combine_device)."""
    import torch
    import dmx
    import shard

    seconds = args.seconds
    n = int(seconds * SR)
    track = synth.pink_noise(2024, n)
    weights = np.eye(4, dtype=np.float32)
    cuda = f"cuda:{dev}"
    lr = torch.from_numpy(track).to(cuda)
    stems = torch.zeros((4, 2, n), dtype=torch.float32, device=cuda)
    chunks = shard.plan(n, 1, shifts=0).chunks
    if world == 1:
        hs = [dmx.Handle(synth.write_safetensors(synth.random_weights(k)), device=dev,
                         max_batch=chunks, precision=getattr(dmx, args.precision)) for k in range(4)]
        bag = dmx.Bag(hs, weights)
        stream = torch.cuda.ExternalStream(hs[0].stream, device=cuda)
        torch.cuda.synchronize()

        def step():
            bag.separate_track_device(lr.data_ptr(), n, stems.data_ptr(), shifts=0, batch=chunks)
        parallelism = "lockstep bag on one GPU"
    else:
        assign = shard.bag_assign(4, world, rank, weights)
        group = assign.group
        p = shard.plan(n, len(group), shifts=0)
        me = p.rank(assign.index)
        mine = me.chunk_hi - me.chunk_lo
        hs = [dmx.Handle(synth.write_safetensors(synth.random_weights(k)), device=dev,
                         max_batch=max(1, mine if len(group) > 1 else chunks),
                         precision=getattr(dmx, args.precision)) for k in assign.nets]
        stream = torch.cuda.ExternalStream(hs[0].stream, device=cuda)
        own = {k: torch.zeros((4, 2, n), dtype=torch.float32, device=cuda) for k in assign.nets}
        mix_norm = torch.empty_like(lr)
        mean_std = torch.empty(2, dtype=torch.float32, device=cuda)
        acc = torch.zeros((8, p.view_length), dtype=torch.float32, device=cuda)
        torch.cuda.synchronize()

        def combine(outs, w, req):
            ptrs = [o.data_ptr() if o is not None else 0 for o in outs]
            dmx.bag_combine_device(ptrs, w, None, 1, n, stems.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
            return stems

        def step():
            with torch.cuda.stream(stream):
                for k, h in zip(assign.nets, hs):
                    if len(group) == 1:
                        h.separate_track_device(lr.data_ptr(), n, own[k].data_ptr(), shifts=0,
                                                batch=chunks)
                        continue
                    h.normalize_track_device(lr.data_ptr(), n, mix_norm.data_ptr(),
                                             mean_std.data_ptr())
                    if mine:
                        acc[:, me.span_lo:me.span_hi].zero_()
                        h.track_shard(mix_norm.data_ptr(), n, 0, 0, 0.25, me.chunk_lo, me.chunk_hi,
                                      mine, acc.data_ptr(), 0, p.view_length)
                    shard.exchange_tails(dist, p, assign.index, acc, ranks=group)
                    if me.t_hi > me.t_lo:
                        h.track_finish(acc.data_ptr(), n, 0, 0, 0.25, 0, mean_std.data_ptr(),
                                       own[k].data_ptr(), me.t_lo, me.t_hi)
                    shard.gather_stems(dist, p, assign.index, own[k].view(8, n), ranks=group)
                shard.bag_gather(dist, rank, assign, own, weights, None, combine, stems)
        parallelism = (f"whole networks per GPU x{world}" if world < 4 else
                       f"one network per GPU{' pair' if world == 8 else ''}, x{world}")
    ms, clocks = _timed(torch, stream, dev, dist, step, args.steps, args.warmup)
    value = seconds / (ms / 1e3)
    line = {"metric": METRIC + ", htdemucs_ft bag of 4", "value": round(value, 3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.precision.lower(), "data": "synthetic",
            "config": {"workload": f"htdemucs_ft bag: 4 random-init networks (seeds 0-3), identity "
                                   f"4x4 bag weights, {seconds:g} s stereo pink noise, shifts 0, "
                                   "overlap 0.25", "chunks_per_network": chunks,
                       "l2": "inputs and workspace larger than L2 (126 MB)"},
            "parallelism": parallelism, "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    for h in hs:
        h.synchronize()
    del lr, stems
    torch.cuda.empty_cache()
    for h in hs:
        h.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_batch(args, rank, world, dev, dist):
    """Throughput batch (the many-track configuration of the benchmark): seeded pink-noise
    tracks, shifts 2, segment 7.8 s, overlap 0.25; every rank takes a balanced share of
    the tracks (shard.assign_tracks) and pools all their (track, shift pass, chunk) units
    into full forwards (dmx_separate_batch_device); the stems stay on each rank's GPU.
    The default is the full 64 x 180 s batch; --tracks / --seconds shrink it."""
    import torch
    import dmx
    import shard

    n = int(args.seconds * SR)
    tracks = [synth.pink_noise(5000 + i, n) for i in range(args.tracks)]
    per_rank = shard.assign_tracks([n] * len(tracks), world, shifts=2)
    mine = per_rank[rank]
    units = sum(shard.track_units(n, 2) for _ in mine)
    batch = min(args.max_batch, max(1, units))
    cuda = f"cuda:{dev}"
    h = dmx.Handle(synth.write_safetensors(synth.random_weights(0)), device=dev, max_batch=batch,
                   precision=getattr(dmx, args.precision))
    stream = torch.cuda.ExternalStream(h.stream, device=cuda)
    lrs = [torch.from_numpy(tracks[i]).to(cuda) for i in mine]
    outs = [torch.empty((4, 2, n), dtype=torch.float32, device=cuda) for _ in mine]
    torch.cuda.synchronize()

    def step():
        if mine:
            h.separate_batch_device([x.data_ptr() for x in lrs], [n] * len(mine),
                                    [o.data_ptr() for o in outs], shifts=2, batch=batch)
    ms, clocks = _timed(torch, stream, dev, dist, step, args.steps, args.warmup)
    audio = len(tracks) * args.seconds
    line = {"metric": METRIC + ", many-track batch", "value": round(audio / (ms / 1e3), 3),
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": args.precision.lower(), "data": "synthetic",
            "config": {"workload": f"throughput batch: {len(tracks)} pink-noise tracks of "
                                   f"{args.seconds:g} s, shifts 2, segment 7.8 s, overlap 0.25, "
                                   "units pooled into full forwards", "forwards_per_step_rank0":
                                   -(-shard.track_units(n, 2) * len(per_rank[0]) // batch),
                       "chunks_per_forward": batch, "tracks_per_gpu": [len(t) for t in per_rank],
                       "l2": "inputs and workspace larger than L2 (126 MB)"},
            "parallelism": f"tracks over ranks x{world}", "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    h.synchronize()
    torch.cuda.synchronize()
    del lrs, outs
    torch.cuda.empty_cache()
    h.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_suite(args):
    """Kernel suite (the benchmark's isolated-kernel configuration): every launch of a
    one-segment forward (config 1 shapes: the conv implicit GEMMs such as enc1 96 x 43008 x
    384, the 3x3 decoder rewrites, the transformer linears M = 2688 / 1344, K = 512,
    N = 512 / 1536 / 2048 and FFN2 K = 2048, attention 8 x 64 over 2688^2, 1344^2 and the
    cross shapes) timed with CUDA events, for each build. The GPU is held behind a sleep
    kernel while the host enqueues the forward, so consecutive events bracket kernels that
    run back to back. Inputs: N(0, 0.1^2) audio; random-init weights (LayerScale 1e-4)."""
    import torch
    import dmx

    dev = 0
    torch.cuda.set_device(dev)
    hbm, bf16_burst, _, kind = _peaks()
    blob = synth.write_safetensors(synth.random_weights(0))
    G = args.suite_batch
    mix = torch.from_numpy(synth.gaussian_audio(1, G)).to(f"cuda:{dev}")
    out = torch.empty((G, 4, 2, SEGMENT), dtype=torch.float32, device=f"cuda:{dev}")
    builds = {}
    for prec in args.suite_builds.split(","):
        h = dmx.Handle(blob, device=dev, max_batch=G, precision=getattr(dmx, prec))
        stream = torch.cuda.ExternalStream(h.stream, device=f"cuda:{dev}")
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            h.forward_device(mix.data_ptr(), G, out.data_ptr())
        h.synchronize()
        h.set_stage_timing(True)
        runs = []
        for _ in range(args.steps):
            with torch.cuda.stream(stream):
                torch.cuda._sleep(60_000_000)  # ~30 ms: the whole forward is enqueued behind it
            h.forward_device(mix.data_ptr(), G, out.data_ptr())
            h.synchronize()
            runs.append(h.stage_times(work=True))
        h.set_stage_timing(False)
        tags = {}
        for tag in runs[0]:
            ms = float(np.median([r[tag][0] for r in runs]))
            _, launches, flops, nbytes = runs[0][tag]
            e = {"ms": round(ms, 4), "launches": launches, "us_per_launch": round(1e3 * ms / launches, 2)}
            if flops:
                tf = flops / (ms / 1e3) / 1e12
                e.update(tflops=round(tf, 2), frac_of_bf16_burst=round(tf / bf16_burst, 4),
                         gflop=round(flops / 1e9, 3))
            if nbytes:
                gbs = nbytes / (ms / 1e3) / 1e9
                e.update(gbs=round(gbs, 1), frac_of_hbm=round(gbs / hbm, 4))
            tags[tag] = e
        total = sum(v["ms"] for v in tags.values())
        builds[prec] = {"forward_ms": round(total, 3),
                        "kernels": dict(sorted(tags.items(), key=lambda kv: -kv[1]["ms"]))}
        h.close()
    line = {"suite": "kernels", "segments": G, "steps": args.steps, "warmup": args.warmup,
            "peaks": {"hbm_gbs": hbm, "bf16_tflops_burst": bf16_burst, "kind": kind},
            "note": "per-launch CUDA events with the GPU held behind a sleep kernel while the "
                    "forward is enqueued; TFLOP/s from the algorithmic FLOPs of each launch; "
                    "tf32 dense peak is half the bf16 one (datasheet ratio)",
            "builds": builds}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="BF16", choices=["FP32", "TF32", "TF32X3", "BF16"],
                    help="BF16 (the headline: bf16 transformer linears, single-pass tf32 elsewhere; "
                         "per-stem SNR >= 60 dB at the benchmark's weights), TF32 (tf32 tensor "
                         "cores, 3xTF32 DConv), TF32X3 (fp32-class), FP32 (SIMT)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--no-fp32-class", action="store_true", help="skip the TF32X3 and BF16 legs")
    ap.add_argument("--ref-chunks", type=int, default=2,
                    help="reference arm: chunks of the workload's track per step (a prefix)")
    ap.add_argument("--e2e-batch", type=int, default=0,
                    help="chunks per forward in the host-API (e2e) leg; 0 = half the track's")
    ap.add_argument("--seconds", type=float, default=None,
                    help="track length (the benchmark is 240 s, 180 s per track for --workload "
                         "batch; shorter tracks are for profiling)")
    ap.add_argument("--suite", default=None, choices=["kernels"],
                    help="kernels: time every launch of a forward of --suite-batch segments per build")
    ap.add_argument("--suite-batch", type=int, default=1)
    ap.add_argument("--suite-builds", default="TF32,BF16,TF32X3,FP32")
    ap.add_argument("--workload", default="track", choices=["track", "bag", "batch"],
                    help="track: one 240 s track (the headline); bag: the htdemucs_ft bag of 4; "
                         "batch: the many-track throughput batch")
    ap.add_argument("--tracks", type=int, default=64, help="--workload batch: tracks")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1: boundary tail and stem gather as SM loads from mapped peer "
                         "memory (peer) or as NCCL point-to-point messages (nccl)")
    ap.add_argument("--max-batch", type=int, default=42,
                    help="--workload batch: chunks per forward")
    args = ap.parse_args()
    if args.seconds is None:
        args.seconds = 180.0 if args.workload == "batch" else TRACK_SECONDS
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.suite == "kernels":
        run_suite(args)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
