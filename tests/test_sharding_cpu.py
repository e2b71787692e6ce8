"""Sequence sharding host logic on CPU: the shard plan and the rank-ordered
exchange of packed partial states over a world-size-2 gloo group.

The partial states come from the oracle's reconstruction of each shard's
tokens (fp64 softmax pieces); the merge is the log-sum-exp combination the
device merge kernel applies, restated here with numpy.  The merged output must
match the oracle's single-device attention (cache.rs:224-279), which is what
the sharded cache promises.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O
from helpers import synthetic_kv

from kivi_cache.sharding import exchange_partials, shard_plan

R = 128


def packed_layout(rows, dim):
    off_o = (2 * rows + 3) & ~3
    return off_o, (off_o + rows * dim + 3) & ~3


def test_packed_layout_matches_c_abi():
    import kivi_cache as K

    for rows, dim in [(1, 128), (32, 128), (3, 64), (5, 7)]:
        assert K.packed_partials_floats(rows, dim) == packed_layout(rows, dim)[1]


@pytest.mark.parametrize("total,world", [(0, 1), (100, 1), (100, 2), (1000, 2), (1024, 4),
                                         (1_048_576, 8), (1_048_576 + 77, 8), (300, 4)])
def test_shard_plan_covers_the_sequence(total, world):
    plans = [shard_plan(total, world, r, R) for r in range(world)]
    assert plans[0].start == 0 and plans[-1].end == total
    for a, b in zip(plans, plans[1:]):
        assert a.end == b.start
    for p in plans[:-1]:
        assert p.tokens % R == 0 and not p.tail
    assert plans[-1].tail
    assert plans[-1].tokens >= max(p.tokens for p in plans)
    if total >= world * R:
        assert plans[-1].tokens >= R
    else:
        assert all(p.tokens == 0 for p in plans[:-1])


@pytest.mark.parametrize("total,world,disc", [(1_048_575, 8, 16384), (1_048_575, 2, 40000),
                                              (1024, 4, 4096), (300, 4, 1000), (5000, 1, 640)])
def test_shard_plan_tail_discount(total, world, disc):
    """The discount moves R-aligned tokens from the last rank onto the others,
    leaving it about `disc` tokens fewer than each other rank; the ranges still
    tile the sequence and the last rank keeps >= R tokens whenever the
    undiscounted plan gave it that many."""
    plans = [shard_plan(total, world, r, R, disc) for r in range(world)]
    base = [shard_plan(total, world, r, R) for r in range(world)]
    assert plans[0].start == 0 and plans[-1].end == total
    for a, b in zip(plans, plans[1:]):
        assert a.end == b.start
    for p, q in zip(plans[:-1], base[:-1]):
        assert p.tokens % R == 0 and p.tokens >= q.tokens and p.tokens == plans[0].tokens
    assert plans[-1].tokens <= base[-1].tokens
    if base[-1].tokens >= R:
        assert plans[-1].tokens >= R
    if world > 1:
        gap = plans[0].tokens - plans[-1].tokens
        assert gap <= disc
        # short of the discount only where one more R per rank would leave the
        # last rank fewer than R tokens
        capped = total - (world - 1) * (plans[0].tokens + R) < R
        assert gap >= disc - world * R or capped


def test_shard_plan_rejects_bad_arguments():
    with pytest.raises(ValueError):
        shard_plan(10, 2, 2, R)
    with pytest.raises(ValueError):
        shard_plan(10, 0, 0, R)
    with pytest.raises(ValueError):
        shard_plan(-1, 2, 0, R)
    with pytest.raises(ValueError):
        shard_plan(10, 2, 0, 0)
    with pytest.raises(ValueError):
        shard_plan(10, 2, 0, R, -1)


# ---------------------------------------------------------------- gloo, world 2

B, H, HQ, D, TOTAL = 1, 2, 4, 64, 700


def _oracle_full():
    k, v, _ = synthetic_kv(77, B, H, TOTAL, D)
    c = O.KiviCache(O.KiviConfig.try_new(2, 32, R), B, H, D)
    c.append(k, v, TOTAL)
    return c


def _partial(keys, values, q, start, end, scale):
    """(m, l, o) of tokens [start, end) for every query row, fp64."""
    GQ = HQ // H
    rows = B * HQ
    m = np.full(rows, -np.inf)
    l = np.zeros(rows)
    o = np.zeros((rows, D))
    kk = keys.reshape(B, H, TOTAL, D).astype(np.float64)
    vv = values.reshape(B, H, TOTAL, D).astype(np.float64)
    qq = q.reshape(B, HQ, D).astype(np.float64)
    if end > start:
        for b in range(B):
            for h in range(HQ):
                x = kk[b, h // GQ, start:end] @ qq[b, h] * scale
                mx = x.max()
                e = np.exp(x - mx)
                r = b * HQ + h
                m[r], l[r], o[r] = mx, e.sum(), e @ vv[b, h // GQ, start:end]
    return m, l, o


def _merge(gathered, rows):
    off_o, _ = packed_layout(rows, D)
    m = gathered[:, :rows].astype(np.float64)
    l = gathered[:, rows:2 * rows].astype(np.float64)
    o = gathered[:, off_o:off_o + rows * D].reshape(-1, rows, D).astype(np.float64)
    M = np.where(l > 0, m, -np.inf).max(axis=0)
    w = np.where(l > 0, np.exp(m - M), 0.0)
    L = (l * w).sum(axis=0)
    return (o * w[:, :, None]).sum(axis=0) / L[:, None]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        c = _oracle_full()
        keys, values = c.dequantize()
        plan = shard_plan(TOTAL, world, rank, R)
        scale = 1.0 / np.sqrt(D)
        qv = np.random.default_rng(5).standard_normal(B * HQ * D).astype(np.float32)
        rows = B * HQ
        off_o, n = packed_layout(rows, D)
        m, l, o = _partial(keys, values, qv, plan.start, plan.end, scale)
        local = np.zeros(n, np.float32)
        local[:rows], local[rows:2 * rows] = m, l
        local[off_o:off_o + rows * D] = o.reshape(-1)
        gathered = exchange_partials(torch.from_numpy(local)).numpy()
        # rank order: row r of the gathered buffer is rank r's state
        mine = np.asarray(gathered[rank])
        ok_order = bool(np.array_equal(mine, local))
        merged = _merge(gathered, rows).astype(np.float32)
        ref = c.attention(qv, HQ, np.float32(scale))
        err = float(np.linalg.norm(merged.reshape(-1) - ref) / np.linalg.norm(ref))
        q.put((rank, ok_order, err, plan.tokens))
    except Exception as e:  # reported to the parent instead of a queue timeout
        q.put((rank, False, repr(e), -1))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_seq_sharded_exchange_and_merge_gloo_world2():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert [r[3] for r in res] == [256, TOTAL - 256]
    for rank, ok_order, err, _ in res:
        assert ok_order, f"rank {rank}: gathered row is not its own state"
        assert err <= 1e-5, f"rank {rank}: merged attention rel-L2 {err}"


# ---------------------------------------------------------------- failures between ranks
# A peer that never joins, leaves between steps, or stalls inside a step must
# surface as KiviError(Comm) within the bounded wait (the reference returns
# Result<_, KiviError>, error.rs:4-45), never as a hang.  gloo ranks on CPU.

TIMEOUT = 3.0


def _fail_worker(rank, world, port, mode, q):
    import time

    import torch
    import torch.distributed as dist

    from kivi_cache import KiviError
    from kivi_cache.sharding import exchange_partials, init_shard_group

    out = {"rank": rank}
    try:
        t0 = time.monotonic()
        try:
            init_shard_group("gloo", rank=rank, world_size=world, timeout_s=TIMEOUT,
                             init_method=f"tcp://127.0.0.1:{port}")
        except KiviError as e:
            out.update(stage="init", variant=e.variant, elapsed=time.monotonic() - t0)
            q.put(out)
            return
        local = torch.full((8,), float(rank))
        g = exchange_partials(local, timeout_s=TIMEOUT)  # step 1: everyone present
        out["step1"] = g[:, 0].tolist()
        if mode == "leave" and rank == 1:
            dist.destroy_process_group()  # leaves between steps, nothing in flight
            out["stage"] = "left"
            q.put(out)
            return
        if mode == "stall" and rank == 1:
            time.sleep(3 * TIMEOUT)  # alive, but never takes part in step 2
            out["stage"] = "stalled"
            q.put(out)
            return
        if mode == "leave":
            time.sleep(0.5)  # the peer is gone before step 2 starts
        t0 = time.monotonic()
        try:
            exchange_partials(local, timeout_s=TIMEOUT)
            out.update(stage="step2", variant="Ok", elapsed=time.monotonic() - t0)
        except KiviError as e:
            out.update(stage="step2", variant=e.variant, elapsed=time.monotonic() - t0,
                       message=e.message)
        q.put(out)
    except Exception as e:  # reported to the parent instead of a queue timeout
        out.update(stage="error", variant=repr(e))
        q.put(out)


def _run_fail(ranks, world, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, mode, q)) for r in ranks]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=120)
        res[r["rank"]] = r
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_rank_that_never_joins_fails_within_the_timeout():
    res = _run_fail([0], 2, "absent")  # rank 1 of 2 is never started
    r = res[0]
    assert r["stage"] == "init" and r["variant"] == "Comm", r
    assert r["elapsed"] < TIMEOUT + 10, r


def test_rank_that_leaves_between_steps_fails_the_next_exchange():
    res = _run_fail([0, 1], 2, "leave")
    assert res[1]["stage"] == "left" and res[1]["step1"] == [0.0, 1.0]
    r = res[0]
    assert r["step1"] == [0.0, 1.0]
    assert r["stage"] == "step2" and r["variant"] == "Comm", r
    assert r["elapsed"] < TIMEOUT + 5, r


def test_peer_that_stalls_in_a_step_fails_within_the_timeout():
    res = _run_fail([0, 1], 2, "stall")
    r = res[0]
    assert r["stage"] == "step2" and r["variant"] == "Comm", r
    assert TIMEOUT - 0.5 <= r["elapsed"] < TIMEOUT + 5, r
    assert "communicator aborted" in r.get("message", "") or "failed" in r.get("message", "")
