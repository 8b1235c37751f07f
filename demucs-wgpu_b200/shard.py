"""Chunk sharding of one track over ranks (one process per GPU).

The unit of work is a chunk of the split pass (streaming.rs:296-400): its
forward depends on nothing but its own padded samples, so a track's chunks are
split into contiguous ranges, one per rank. Each rank overlap-adds its chunks
into its own span of the view; spans of neighbouring ranks overlap by at most
``segment - stride`` samples (one chunk's tail), which is the only data that
crosses between GPUs before the final gather of the stems to rank 0.

Every sample receives at most two weighted contributions (stride >
segment / 2), and ``(0 + a) + b == (0 + b) + a`` in IEEE arithmetic, so the
sharded result is identical to the single-GPU one whatever the rank count.
"""

from __future__ import annotations

from dataclasses import dataclass

SEGMENT = 343980
SR = 44100
# Bound on every point-to-point wait of the exchange and the gathers: a peer
# whose data never arrives (a rank that died or skipped the step) turns into
# ShardTimeout instead of a hang.
WAIT_SECONDS = 120.0


class ShardTimeout(TimeoutError):
    """A bounded wait for a peer's data gave up (the C ABI's DMX_ERR_TIMEOUT)."""

    code = 4  # DMX_ERR_TIMEOUT


def _wait_all(works, what, timeout=None):
    """Waits for every request, each at most ``timeout`` seconds (default
    WAIT_SECONDS); a request that does not complete raises ShardTimeout."""
    import datetime

    limit = datetime.timedelta(seconds=WAIT_SECONDS if timeout is None else timeout)
    for work in works:
        try:
            ok = work.wait(timeout=limit)
        except RuntimeError as exc:  # gloo / NCCL report an expired wait by raising
            raise ShardTimeout(f"{what}: no data from the peer within {limit.total_seconds():g} s "
                               f"({exc})") from exc
        if ok is False:
            raise ShardTimeout(f"{what}: no data from the peer within {limit.total_seconds():g} s")


def shift_offsets(shifts: int, max_shift: int):
    """The offsets ShiftRng draws for each pass (pipeline.rs:136-151, 416-418),
    from the library's own generator (dmx_shift_offsets), so every rank and
    the device drivers use one definition."""
    import dmx

    return dmx.shift_offsets(shifts, max_shift)


@dataclass
class RankPlan:
    rank: int
    chunk_lo: int
    chunk_hi: int
    span_lo: int   # view samples this rank's chunks write
    span_hi: int
    own_lo: int    # view samples this rank finalises
    own_hi: int
    send_lo: int   # tail sent to rank + 1 (empty when send_lo >= send_hi)
    send_hi: int
    t_lo: int      # output samples this rank finalises
    t_hi: int


@dataclass
class TrackPlan:
    length: int
    shifts: int
    overlap: float
    segment: int
    stride: int
    max_shift: int
    offset: int
    view_length: int
    trim: int
    chunks: int
    ranks: list

    def rank(self, r: int) -> RankPlan:
        return self.ranks[r]


def plan(length: int, world: int, shifts: int = 1, overlap: float = 0.25,
         segment: int = SEGMENT, samplerate: int = SR) -> TrackPlan:
    """Single-pass plan (shifts 0 or 1) of a ``length``-sample track over ``world`` ranks.

    The stride must exceed half a segment (overlap < 0.5): then every sample
    has at most two contributions and a rank's overlap tail ends inside its
    right neighbour's own span, which is what the boundary exchange assumes."""
    if shifts not in (0, 1):
        raise ValueError("sharding covers one pass: shifts must be 0 or 1")
    stride = int((1.0 - overlap) * segment)
    if stride <= 0:
        raise ValueError("overlap leaves a zero stride")
    if 2 * stride <= segment:
        raise ValueError("chunk sharding needs overlap < 0.5 (a stride longer than half a segment)")
    max_shift = int(0.5 * samplerate) if shifts else 0
    offset = shift_offsets(1, max_shift)[0] if shifts else 0
    view_length = length + max_shift - offset if shifts else length
    trim = max_shift - offset if shifts else 0
    chunks = -(-view_length // stride)
    base, extra = divmod(chunks, world)
    ranks, c = [], 0
    for r in range(world):
        k = base + (1 if r < extra else 0)
        lo, hi = c, c + k
        c = hi
        if k == 0:
            ranks.append(RankPlan(r, lo, hi, 0, 0, 0, 0, 0, 0, 0, 0))
            continue
        span_lo = lo * stride
        span_hi = min(view_length, (hi - 1) * stride + segment)
        own_lo = lo * stride
        own_hi = view_length if hi == chunks else hi * stride
        send_lo, send_hi = own_hi, span_hi if hi < chunks else own_hi
        t_lo = max(0, own_lo - trim)
        t_hi = max(t_lo, min(length, own_hi - trim))
        ranks.append(RankPlan(r, lo, hi, span_lo, span_hi, own_lo, own_hi, send_lo, send_hi,
                              t_lo, t_hi))
    return TrackPlan(length, shifts, overlap, segment, stride, max_shift, offset, view_length,
                     trim, chunks, ranks)


def exchange_tails(dist, p: TrackPlan, rank: int, acc, ranks=None, timeout=None):
    """Rank r adds rank r-1's tail into its own head: ``acc`` is this rank's
    (8, view_length) accumulator (torch tensor on the backend's device).
    ``rank`` is the index in the plan; ``ranks[i]`` is the process-group rank
    of plan index i (default: the identity), so a plan can span a sub-group.
    Each of the 8 rows goes as its own message straight from ``acc`` (a row
    slice is contiguous), so the sender copies nothing. Each wait is bounded
    (``timeout`` seconds, default WAIT_SECONDS)."""
    import torch

    world = len(p.ranks)
    ranks = list(range(world)) if ranks is None else list(ranks)
    me = p.rank(rank)
    ops = []
    recv = None
    if rank + 1 < world and me.send_hi > me.send_lo and p.rank(rank + 1).chunk_hi > p.rank(rank + 1).chunk_lo:
        for row in range(acc.shape[0]):
            ops.append(dist.P2POp(dist.isend, acc[row, me.send_lo:me.send_hi], ranks[rank + 1]))
    if rank > 0:
        prev = p.rank(rank - 1)
        if prev.send_hi > prev.send_lo and me.chunk_hi > me.chunk_lo:
            recv = torch.empty((acc.shape[0], prev.send_hi - prev.send_lo), dtype=acc.dtype,
                               device=acc.device)
            for row in range(acc.shape[0]):
                ops.append(dist.P2POp(dist.irecv, recv[row], ranks[rank - 1]))
    if ops:
        _wait_all(dist.batch_isend_irecv(ops), "overlap-add boundary exchange", timeout)
    if recv is not None:
        prev = p.rank(rank - 1)
        acc[:, prev.send_lo:prev.send_hi] += recv


def gather_stems(dist, p: TrackPlan, rank: int, stems, ranks=None, timeout=None):
    """Plan index 0 receives every plan index's owned output samples into
    ``stems`` (8, length); ``ranks`` as in exchange_tails. Each row of a span
    travels as its own message, from the sender's stems row straight into the
    receiver's (both row slices are contiguous): no staging copies."""
    world = len(p.ranks)
    ranks = list(range(world)) if ranks is None else list(ranks)
    me = p.rank(rank)
    if rank == 0:
        ops = []
        for r in range(1, world):
            q = p.rank(r)
            if q.t_hi > q.t_lo:
                for row in range(stems.shape[0]):
                    ops.append(dist.P2POp(dist.irecv, stems[row, q.t_lo:q.t_hi], ranks[r]))
        if ops:
            _wait_all(dist.batch_isend_irecv(ops), "stem gather", timeout)
    elif me.t_hi > me.t_lo:
        ops = [dist.P2POp(dist.isend, stems[row, me.t_lo:me.t_hi], ranks[0])
               for row in range(stems.shape[0])]
        _wait_all(dist.batch_isend_irecv(ops), "stem gather", timeout)


# ---------------------------------------------------------------------------
# The same exchange and gather as SM loads over NVLink from peer memory
# ---------------------------------------------------------------------------

class PeerBuffers:
    """Every rank's copy of one device buffer, mapped into this process over CUDA
    IPC (dmx_ipc_export / dmx_ipc_open), so a rank reads its neighbours' buffers
    directly. ``ptrs[r]`` is rank r's buffer as this process addresses it (its own
    is the local pointer). Collective: every rank constructs it with its own
    buffer, in the same order."""

    def __init__(self, dist, device: int, ptr: int):
        import dmx

        self.device = device
        self.rank = dist.get_rank()
        # every rank takes part in the exchange even when its own export failed,
        # so a failure raises on every rank instead of leaving the others waiting
        try:
            mine = dmx.ipc_export(device, ptr)
        except Exception as exc:
            mine = ("error", f"{type(exc).__name__}: {exc}")
        everyone = [None] * dist.get_world_size()
        dist.all_gather_object(everyone, mine)
        failed = [e[1] for e in everyone if isinstance(e[0], str)]
        if failed:
            raise RuntimeError("peer buffer export failed: " + failed[0])
        self.offsets = [off for _, off in everyone]
        self.ptrs = []
        try:
            for r, (hnd, off) in enumerate(everyone):
                self.ptrs.append(ptr if r == self.rank else dmx.ipc_open(device, hnd, off))
        except Exception:
            self.close()
            raise

    def close(self):
        import dmx

        for r, ptr in enumerate(self.ptrs):
            if r != self.rank and ptr:
                dmx.ipc_close(self.device, ptr, self.offsets[r])
        self.ptrs = []


def device_barrier(dist, flag):
    """A one-element all-reduce on the current stream: when it completes on a GPU,
    every rank's earlier work on its own stream has completed. Orders peer reads
    after the peer's writes (and the peer's next writes after the reads) without
    a host wait. ``flag`` is a one-element tensor on this rank's GPU."""
    dist.all_reduce(flag)


def exchange_tails_peer(dist, p: TrackPlan, rank: int, h, acc_ptr: int, peers: PeerBuffers,
                        flag, rows: int = 8):
    """exchange_tails over NVLink: after a barrier, rank r adds rank r-1's tail into
    its own accumulator with SM loads straight from the neighbour's (dmx_rows_add).
    ``acc_ptr`` / ``peers`` address the (rows, view_length) accumulators."""
    device_barrier(dist, flag)
    if rank == 0:
        return
    prev, me = p.rank(rank - 1), p.rank(rank)
    width = prev.send_hi - prev.send_lo
    if width > 0 and me.chunk_hi > me.chunk_lo:
        lo = prev.send_lo * 4
        h.rows_add(acc_ptr + lo, p.view_length, peers.ptrs[rank - 1] + lo, p.view_length, rows,
                   width)


def gather_stems_peer(dist, p: TrackPlan, rank: int, h, stems_ptr: int, peers: PeerBuffers,
                      flag, rows: int = 8):
    """gather_stems over NVLink: after a barrier, rank 0 copies every rank's owned
    span of its (rows, length) stems straight from that rank's buffer
    (dmx_rows_copy); a second barrier keeps every rank from overwriting its stems
    before rank 0 has read them."""
    device_barrier(dist, flag)
    if rank == 0:
        for r in range(1, len(p.ranks)):
            q = p.rank(r)
            if q.t_hi > q.t_lo:
                off = q.t_lo * 4
                h.rows_copy(stems_ptr + off, p.length, peers.ptrs[r] + off, p.length, rows,
                            q.t_hi - q.t_lo)
    device_barrier(dist, flag)


# ---------------------------------------------------------------------------
# Bags of networks (htdemucs_ft) over ranks
# ---------------------------------------------------------------------------

def needed_nets(weights, requested=None):
    """Networks that carry a nonzero weight on a requested source
    (api.rs:907-916); ``requested`` holds source indices (None = all)."""
    return [k for k, row in enumerate(weights)
            if any(w != 0 and (requested is None or s in requested) for s, w in enumerate(row))]


@dataclass
class BagAssignment:
    nets: list    # the networks this rank runs, in bag order
    group: list   # process-group ranks that shard each of those networks' chunks
    index: int    # this rank's index in `group`
    owner: dict   # network -> rank that holds its whole-track stems (its group's first)


def bag_assign(n_nets: int, world: int, rank: int, weights=None, requested=None) -> BagAssignment:
    """One network per GPU group: with at least as many ranks as running
    networks (and a multiple of them), network j gets the ranks
    [j*g, (j+1)*g), g = world // running, and its chunks are sharded over
    them; with fewer ranks than networks, rank r runs networks r, r + world, ...
    whole (each rank a group of one)."""
    run = needed_nets(weights, requested) if weights is not None else list(range(n_nets))
    if not run:
        raise ValueError("no network carries a requested stem")
    if world >= len(run):
        if world % len(run):
            raise ValueError(f"{world} ranks do not split evenly over {len(run)} networks")
        g = world // len(run)
        j = rank // g
        owner = {k: i * g for i, k in enumerate(run)}
        return BagAssignment([run[j]], list(range(j * g, (j + 1) * g)), rank - j * g, owner)
    owner = {k: i % world for i, k in enumerate(run)}
    mine = [k for i, k in enumerate(run) if i % world == rank]
    return BagAssignment(mine, [rank], 0, owner)


def bag_gather(dist, rank: int, assign: BagAssignment, stems_by_net: dict, weights, requested,
               combine, like):
    """Rank 0 receives, from each running network's owner, the stem lanes
    that network is weighted on, then calls ``combine(outs, weights,
    requested)`` with ``outs[k]`` a (4, 2, n) tensor per network (None for
    networks that do not run) and returns its result; other ranks return
    None. ``stems_by_net[k]`` is this rank's (4, 2, n) stems of network k
    (ranks that own a network); ``like`` gives shape, dtype and device."""
    import torch

    sources = len(weights[0])
    req = [requested is None or s in requested for s in range(sources)]
    lanes = [(k, s) for k in sorted(assign.owner) for s in range(sources)
             if weights[k][s] != 0 and req[s]]
    if rank == 0:
        outs = [None] * len(weights)
        ops, recvs = [], []
        for k, s in lanes:
            if outs[k] is None:
                outs[k] = torch.zeros_like(like)
            if assign.owner[k] == 0:
                outs[k][s] = stems_by_net[k][s]
            else:
                buf = torch.empty_like(like[0])
                recvs.append((k, s, buf))
                ops.append(dist.P2POp(dist.irecv, buf, assign.owner[k]))
        if ops:
            _wait_all(dist.batch_isend_irecv(ops), "bag lane gather")
        for k, s, buf in recvs:
            outs[k][s] = buf
        return combine(outs, weights, requested)
    ops = [dist.P2POp(dist.isend, stems_by_net[k][s].contiguous(), 0)
           for k, s in lanes if assign.owner[k] == rank]
    if ops:
        _wait_all(dist.batch_isend_irecv(ops), "bag lane gather")
    return None


# ---------------------------------------------------------------------------
# Many tracks (the throughput batch) over ranks
# ---------------------------------------------------------------------------

def track_units(length: int, shifts: int, overlap: float = 0.25, segment: int = SEGMENT,
                samplerate: int = SR) -> int:
    """Forward units (chunks over all shift passes) of one track: one
    split pass per shift, each of ceil(view / stride) chunks
    (streaming.rs:88-94), the view lengthened by max_shift - offset."""
    stride = int((1.0 - overlap) * segment)
    if shifts == 0:
        return -(-length // stride)
    max_shift = int(0.5 * samplerate)
    return sum(-(-(length + max_shift - o) // stride) for o in shift_offsets(shifts, max_shift))


def assign_tracks(lengths, world: int, shifts: int, overlap: float = 0.25):
    """Tracks are independent units: rank r gets a list of track indices so
    that the forward units per rank are balanced (longest track first onto
    the least-loaded rank; ties to the lower rank, so every rank computes the
    same assignment). Each rank then runs dmx_separate_batch on its tracks."""
    units = [track_units(n, shifts, overlap) for n in lengths]
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-units[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += units[i]
    return [sorted(x) for x in out]


def gather_tracks(dist, rank: int, per_rank, stems_by_track: dict, lengths, like=None,
                  timeout=None):
    """Rank 0 receives the (4, 2, n_i) stems of every track the other ranks
    separated (``per_rank`` from assign_tracks) and returns {track: stems};
    other ranks send theirs and return {}. ``stems_by_track`` holds this
    rank's own tracks; ``like`` gives dtype and device (default: any of them).
    Every receive waits at most ``timeout`` seconds (ShardTimeout)."""
    import torch

    if rank == 0:
        out = dict(stems_by_track)
        proto = like if like is not None else next(iter(stems_by_track.values()), None)
        ops, recvs = [], []
        for r, tracks in enumerate(per_rank):
            if r == 0:
                continue
            for i in tracks:
                buf = torch.empty((4, 2, lengths[i]), dtype=torch.float32,
                                  device=proto.device if proto is not None else "cpu")
                recvs.append((i, buf))
                ops.append(dist.P2POp(dist.irecv, buf, r))
        if ops:
            _wait_all(dist.batch_isend_irecv(ops), "track gather", timeout)
        out.update(dict(recvs))
        return out
    ops = [dist.P2POp(dist.isend, stems_by_track[i].contiguous(), 0) for i in per_rank[rank]]
    if ops:
        _wait_all(dist.batch_isend_irecv(ops), "track gather", timeout)
    return {}
