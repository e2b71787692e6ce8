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
state (m, l, o) of its tokens for every query row, one all-gather exchanges the
packed states (rows * (head_dim + 2) floats per rank), and every rank merges
them in rank order with the same log-sum-exp merge, so all ranks hold the same,
deterministic output.

The host logic here (ranges, exchange) is device-agnostic and runs on gloo/CPU
in the tests; the CUDA work goes through the C ABI of libkivi_gpu.so.
"""
from __future__ import annotations

from dataclasses import dataclass

__all__ = ["ShardPlan", "shard_plan", "exchange_partials", "SeqShardedCache"]


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


def shard_plan(total_tokens: int, world: int, rank: int, residual_length: int) -> ShardPlan:
    """R-aligned contiguous ranges: ranks 0..world-2 get `per` tokens each,
    per = floor(total / (world * R)) * R, and the last rank the rest (at least
    `per`, so at least R once total >= world * R).  When total < world * R
    every token stays on the last rank and the others hold empty shards."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if residual_length < 1:
        raise ValueError("residual_length must be positive")
    if total_tokens < 0:
        raise ValueError("total_tokens must be non-negative")
    per = (total_tokens // (world * residual_length)) * residual_length
    start = rank * per
    end = total_tokens if rank == world - 1 else start + per
    return ShardPlan(rank, world, start, end, rank == world - 1)


def exchange_partials(local, gathered=None, group=None):
    """All-gather of every rank's packed partial state, in rank order, into
    `gathered` ([world, n] on local's device; allocated when None).  One
    collective: all_gather_into_tensor on NCCL, the list form elsewhere (gloo
    has no single-buffer all-gather).  Runs on torch's current stream."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if gathered is None:
        gathered = torch.empty((world,) + tuple(local.shape), dtype=local.dtype,
                               device=local.device)
    if world == 1:
        gathered[0].copy_(local)
    elif dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local, group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), local, group=group)
    return gathered


class SeqShardedCache:
    """One logical KiviCache whose tokens are split over the ranks of `group`.

    Each rank constructs it with the same (config, batch, heads, dim,
    total_prefill_tokens); `prefill_local_dev` takes the rank's own slice of the
    prefill (tokens plan.start..plan.end of [batch, heads, seq, dim]).
    `decode_dev` appends the step's token on the tail rank and returns, on every
    rank, the attention output over all shards."""

    def __init__(self, config, batch, num_kv_heads, head_dim, total_prefill_tokens, group=None,
                 device=None):
        import torch
        import torch.distributed as dist

        from . import KiviCache

        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.plan = shard_plan(total_prefill_tokens, self.world, self.rank,
                               config.residual_length)
        self.device = torch.cuda.current_device() if device is None else device
        self.batch, self.heads, self.dim = batch, num_kv_heads, head_dim
        self.cache = KiviCache(config, batch, num_kv_heads, head_dim, device=self.device)
        self._bufs = {}

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

    def attention_dev(self, d_query, num_q_heads, scale, d_out, stream):
        """Attention of every query row over all shards; the same d_out on every rank."""
        import torch

        from . import merge_packed_partials_dev

        rows = self.batch * num_q_heads
        local, gathered = self._buffers(rows)
        self.cache.attention_partial_packed_dev(d_query, num_q_heads, scale, local, stream=stream)
        with torch.cuda.stream(stream):
            exchange_partials(local, gathered, self.group)
        merge_packed_partials_dev(self.world, rows, self.dim, gathered, d_out, stream=stream)

    def decode_dev(self, d_key, d_value, d_query, num_q_heads, scale, d_out, stream):
        """RuntimeKv::decode (runtime.rs:46-56) on the sharded cache."""
        if self.plan.tail:
            self.cache.append_dev(d_key, d_value, 1, stream=stream)
        self.attention_dev(d_query, num_q_heads, scale, d_out, stream)

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
        st.synchronize()
        return out
