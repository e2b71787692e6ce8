"""Sequence sharding of one KIVI cache over the ranks of a process group.

The reference cache (cache.rs) lives on one device.  Here one logical cache's
token axis is split into contiguous ranges, one per rank (one process per GPU):

* every range but the last holds a multiple of the residual length R, so the
  key groups and the key-flush schedule (cache.rs:382-430) of each shard line
  up with those of the single-device cache;
* interior shards are *sealed* (their fp32 value window is quantized, exactly
  what the single-device cache's later evictions would do, cache.rs:432-484:
  per-token quantization does not depend on neighbours), so their packed
  streams are the single-device cache's streams restricted to their range;
* the last rank owns the residual key block and the value window and is the
  only one that appends while decoding.

Attention (cache.rs:224-279) becomes: each rank computes the partial softmax
state (m, l, o) of its tokens for every query row, the ranks exchange those
states (rows * (head_dim + 2) floats per rank), and every rank merges them in
rank order with the same log-sum-exp merge, so all ranks hold the same,
deterministic output.  The exchange runs either inside one kernel over NVLink
peer memory (exchange="p2p": kivi_cache_decode_exchange_dev stores each
rank's merged states straight into every peer's buffer, no collective call)
or as an NCCL all-gather between two kernels (exchange="nccl"); both give the
same bits.

The host logic here (ranges, exchange) is device-agnostic and runs on gloo/CPU
in the tests; the CUDA work goes through the C ABI of libkivi_gpu.so.

Failures between ranks surface as ``KiviError`` with variant ``Comm`` (the
reference is single-device and returns ``Result<_, KiviError>``,
error.rs:4-45): ``init_shard_group`` bounds the rendezvous, so a rank that
never joins makes the others fail after ``timeout_s`` instead of waiting;
``exchange_partials(..., timeout_s=...)`` and ``SeqShardedCache`` bound each
exchange on the host, and a peer that has left, a failed collective or a
wait that runs out aborts the communicator (so nothing of this rank stays
queued on it) and raises.  A cache whose communicator was aborted refuses
further steps with the same error.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

__all__ = ["ShardPlan", "shard_plan", "exchange_partials", "SeqShardedCache", "init_shard_group",
           "comm_error", "abort_group"]

DEFAULT_TIMEOUT_S = 30.0
_SPIN_S = 0.005   # poll without sleeping for this long (a decode step is ~0.1-1 ms)
_POLL_S = 0.0005  # then sleep this long between polls


@dataclass(frozen=True)
class ShardPlan:
    """Token range [start, end) of one rank; `tail` marks the appending rank."""

    rank: int
    world: int
    start: int
    end: int
    tail: bool

    @property
    def tokens(self) -> int:
        return self.end - self.start


def shard_plan(total_tokens: int, world: int, rank: int, residual_length: int,
               tail_discount: int = 0) -> ShardPlan:
    """R-aligned contiguous ranges: ranks 0..world-2 get `per` tokens each,
    per = floor(total / (world * R)) * R, and the last rank the rest (at least
    `per`, so at least R once total >= world * R).  When total < world * R
    every token stays on the last rank and the others hold empty shards.

    tail_discount > 0 leaves the last rank (which also owns the key residual,
    the value window and every append, so its step is longer) about that many
    tokens fewer than each other rank: per = floor((total + tail_discount) /
    (world * R)) * R, lowered while the last rank would keep fewer than R
    tokens, and never below the undiscounted per."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if residual_length < 1:
        raise ValueError("residual_length must be positive")
    if total_tokens < 0:
        raise ValueError("total_tokens must be non-negative")
    if tail_discount < 0:
        raise ValueError("tail_discount must be non-negative")
    R = residual_length
    per = (total_tokens // (world * R)) * R
    if tail_discount > 0 and world > 1:
        moved = ((total_tokens + tail_discount) // (world * R)) * R
        while moved > per and total_tokens - (world - 1) * moved < R:
            moved -= R
        per = max(per, moved)
    start = rank * per
    end = total_tokens if rank == world - 1 else start + per
    return ShardPlan(rank, world, start, end, rank == world - 1)


def comm_error(message):
    """KiviError with the Comm variant (a communication failure between ranks)."""
    from . import KIVI_ERR_COMM, KiviError

    return KiviError(KIVI_ERR_COMM, 0, 0, None, message)


def init_shard_group(backend, rank=None, world_size=None, timeout_s=DEFAULT_TIMEOUT_S,
                     init_method=None, device=None):
    """torch.distributed.init_process_group with a bounded rendezvous: when a
    rank does not join within `timeout_s` seconds the others raise
    KiviError(Comm) instead of waiting.  The same bound becomes the group's
    collective timeout.  rank/world_size/init_method default to the launcher's
    environment (RANK, WORLD_SIZE, MASTER_ADDR/MASTER_PORT)."""
    import datetime

    import torch.distributed as dist

    kw = dict(timeout=datetime.timedelta(seconds=float(timeout_s)))
    if rank is not None:
        kw["rank"] = rank
    if world_size is not None:
        kw["world_size"] = world_size
    if init_method is not None:
        kw["init_method"] = init_method
    if device is not None:
        kw["device_id"] = device
    t0 = time.monotonic()
    try:
        dist.init_process_group(backend, **kw)
    except Exception as e:  # store or backend rendezvous gave up
        raise comm_error(f"process group ({backend}) not formed within {timeout_s:.1f} s "
                         f"({time.monotonic() - t0:.1f} s): {type(e).__name__}: {e}") from e


def abort_group(group=None):
    """Aborts the communicator of `group` (default: the default group): work
    of this rank queued on it is cancelled, so no collective waits for a peer
    that is gone.  Best effort; the group must not be used afterwards."""
    import torch.distributed as dist

    if not dist.is_initialized():
        return
    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    try:
        pg.abort()
    except Exception:
        pass


def wait_bounded(work, timeout_s, what, group=None, stream=None):
    """Waits for a collective's Work (and, if given, a CUDA stream that runs
    after it) on the host for at most `timeout_s` seconds.  A failed
    collective or a wait that runs out aborts the group and raises
    KiviError(Comm)."""
    start = time.monotonic()
    deadline = start + float(timeout_s)
    err = None
    while True:
        try:
            if work is None or work.is_completed():
                if work is not None:
                    work.wait()  # complete: raises the collective's error, if it failed
                    work = None
                if stream is None or stream.query():
                    return
        except Exception as e:
            err = e
            break
        now = time.monotonic()
        if now > deadline:
            break
        if now - start > _SPIN_S:
            time.sleep(_POLL_S)
    abort_group(group)
    if err is not None:
        raise comm_error(f"{what} failed: {type(err).__name__}: {err}") from err
    raise comm_error(f"{what} did not complete within {timeout_s:.1f} s; communicator aborted")


def exchange_partials(local, gathered=None, group=None, timeout_s=None):
    """All-gather of every rank's packed partial state, in rank order, into
    `gathered` ([world, n] on local's device; allocated when None).  One
    collective: all_gather_into_tensor on NCCL, the list form elsewhere (gloo
    has no single-buffer all-gather).  Runs on torch's current stream.

    With `timeout_s` the collective is waited for on the host, for at most
    that long (wait_bounded: a peer that left or a wait that runs out aborts
    the group and raises KiviError(Comm)); without it the call is
    stream-ordered and the group's own timeout applies."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if gathered is None:
        gathered = torch.empty((world,) + tuple(local.shape), dtype=local.dtype,
                               device=local.device)
    if world == 1:
        gathered[0].copy_(local)
        return gathered
    bounded = timeout_s is not None
    try:
        if dist.get_backend(group) == "nccl":
            work = dist.all_gather_into_tensor(gathered, local, group=group, async_op=bounded)
        else:
            work = dist.all_gather(list(gathered.unbind(0)), local, group=group, async_op=bounded)
    except Exception as e:
        abort_group(group)
        raise comm_error(f"partial-state all-gather failed: {type(e).__name__}: {e}") from e
    if bounded:
        wait_bounded(work, timeout_s, "partial-state all-gather", group)
        work.wait()  # complete already; orders torch's current stream after it
    return gathered


class SeqShardedCache:
    """One logical KiviCache whose tokens are split over the ranks of `group`.

    Each rank constructs it with the same (config, batch, heads, dim,
    total_prefill_tokens); `prefill_local_dev` takes the rank's own slice of the
    prefill (tokens plan.start..plan.end of [batch, heads, seq, dim]).
    `decode_dev` appends the step's token on the tail rank and returns, on every
    rank, the attention output over all shards."""

    def __init__(self, config, batch, num_kv_heads, head_dim, total_prefill_tokens, group=None,
                 device=None, timeout_s=DEFAULT_TIMEOUT_S, exchange="auto", tail_discount=0):
        import torch
        import torch.distributed as dist

        from . import KiviCache

        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.plan = shard_plan(total_prefill_tokens, self.world, self.rank,
                               config.residual_length, tail_discount)
        self.device = torch.cuda.current_device() if device is None else device
        self.batch, self.heads, self.dim = batch, num_kv_heads, head_dim
        self.cache = KiviCache(config, batch, num_kv_heads, head_dim, device=self.device)
        self._bufs = {}
        self.timeout_s = timeout_s  # host bound of each host-path step's exchange
        self._failed = None         # set once the communicator was aborted
        if exchange == "auto":
            exchange = "p2p" if self.world > 1 and dist.get_backend(group) == "nccl" else "nccl"
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p', 'nccl' or 'auto', not {exchange!r}")
        self.exchange = exchange
        self._peer = {}  # rows -> PeerExchange

    def _check_alive(self):
        if self._failed is not None:
            raise comm_error(f"communicator aborted earlier: {self._failed}")

    # -- prefill
    def reserve(self, tokens):
        self.cache.reserve(tokens)

    def prefill_local_dev(self, d_keys, d_values, n, stream=None):
        """Append `n` tokens of this rank's range (device [batch, heads, n, dim])."""
        self.cache.append_dev(d_keys, d_values, n, stream=stream)

    def finish_prefill(self):
        """Seal interior shards once their whole range has been appended."""
        if self.cache.sequence_length() != self.plan.tokens:
            raise ValueError(f"rank {self.rank} holds {self.cache.sequence_length()} tokens, "
                             f"its range has {self.plan.tokens}")
        if not self.plan.tail and self.plan.tokens:
            self.cache.seal()

    def sequence_length(self):
        """Tokens of the logical cache (all shards)."""
        return self.plan.start + self.cache.sequence_length() if self.plan.tail else None

    # -- decode
    def _buffers(self, rows):
        import torch

        from . import packed_partials_floats

        b = self._bufs.get(rows)
        if b is None:
            n = packed_partials_floats(rows, self.dim)
            local = torch.empty(n, dtype=torch.float32, device=f"cuda:{self.device}")
            gathered = torch.empty((self.world, n), dtype=torch.float32,
                                   device=f"cuda:{self.device}")
            b = self._bufs[rows] = (local, gathered)
        return b

    def attention_dev(self, d_query, num_q_heads, scale, d_out, stream, timeout_s=None):
        """Attention of every query row over all shards; the same d_out on every
        rank.  Stream-ordered; with `timeout_s` the exchange is also waited for
        on the host (exchange_partials)."""
        import torch

        from . import merge_packed_partials_dev

        self._check_alive()
        rows = self.batch * num_q_heads
        local, gathered = self._buffers(rows)
        self.cache.attention_partial_packed_dev(d_query, num_q_heads, scale, local, stream=stream)
        try:
            with torch.cuda.stream(stream):
                exchange_partials(local, gathered, self.group, timeout_s=timeout_s)
        except Exception as e:
            self._failed = str(e)
            raise
        merge_packed_partials_dev(self.world, rows, self.dim, gathered, d_out, stream=stream)

    def _peer_exchange(self, rows):
        """This rank's peer-memory exchange for `rows` query rows, set up
        collectively on first use (every rank makes the same calls)."""
        import torch
        import torch.distributed as dist

        from . import PeerExchange

        ex = self._peer.get(rows)
        if ex is None:
            ex = PeerExchange(self.device, self.rank, self.world, rows, self.dim)
            mine = torch.tensor(list(ex.ipc_handle()), dtype=torch.uint8,
                                device=f"cuda:{self.device}")
            every = torch.empty((self.world, mine.numel()), dtype=torch.uint8, device=mine.device)
            exchange_partials(mine, every, self.group, timeout_s=self.timeout_s)
            ex.open(bytes(every.cpu().numpy().reshape(-1)))
            dist.barrier(group=self.group)  # every rank has mapped every buffer
            self._peer[rows] = ex
        return ex

    def decode_dev(self, d_key, d_value, d_query, num_q_heads, scale, d_out, stream,
                   timeout_s=None):
        """RuntimeKv::decode (runtime.rs:46-56) on the sharded cache."""
        self._check_alive()
        if self.exchange == "p2p":
            ex = self._peer_exchange(self.batch * num_q_heads)
            self.cache.decode_exchange_dev(ex, d_key if self.plan.tail else None,
                                           d_value if self.plan.tail else None, d_query,
                                           num_q_heads, scale, d_out, stream=stream)
            return
        if self.plan.tail:
            self.cache.append_dev(d_key, d_value, 1, stream=stream)
        self.attention_dev(d_query, num_q_heads, scale, d_out, stream, timeout_s=timeout_s)

    def synchronize(self, stream, timeout_s=None):
        """Waits on the host, for at most `timeout_s` (default: the cache's),
        until `stream` has run the steps queued on it; a step that does not
        finish in time (a peer that stopped taking part in the exchange) aborts
        the communicator and raises KiviError(Comm)."""
        from . import KiviError, device_wait_status

        self._check_alive()
        try:
            wait_bounded(None, self.timeout_s if timeout_s is None else timeout_s,
                         "sharded decode step", self.group, stream=stream)
            try:  # a peer exchange whose bounded wait gave up leaves a device flag
                device_wait_status(self.device)
            except KiviError as e:
                abort_group(self.group)
                raise comm_error(f"peer exchange gave up waiting for a rank: {e.message}") from e
        except Exception as e:
            self._failed = str(e)
            raise

    def close(self):
        """Releases the peer exchanges (collective: every rank calls it)."""
        import torch.distributed as dist

        if not self._peer:
            return
        for ex in self._peer.values():
            ex.close()
        if self._failed is None and dist.is_initialized():
            dist.barrier(group=self.group)  # no rank still maps a buffer about to be freed
        for ex in self._peer.values():
            ex.free()
        self._peer = {}

    def decode(self, keys, values, query, num_q_heads, scale, out=None, stream=None):
        """Host-buffer decode step (torch CPU tensors, pinned for async copies):
        the query goes to every rank, the step's key/value row to the tail
        rank; returns the [batch, num_q_heads, head_dim] output on the host,
        identical on every rank."""
        import torch

        dev = torch.device("cuda", self.device)
        st = stream if stream is not None else torch.cuda.current_stream(dev)
        with torch.cuda.stream(st):
            dq = query.to(dev, non_blocking=True)
            dk = keys.to(dev, non_blocking=True) if self.plan.tail else None
            dv = values.to(dev, non_blocking=True) if self.plan.tail else None
            dout = torch.empty((self.batch, num_q_heads, self.dim), dtype=torch.float32,
                               device=dev)
        self.decode_dev(dk, dv, dq, num_q_heads, scale, dout, st)
        with torch.cuda.stream(st):
            if out is None:
                out = torch.empty(dout.shape, dtype=torch.float32, pin_memory=True)
            out.copy_(dout, non_blocking=True)
        self.synchronize(st)
        return out
