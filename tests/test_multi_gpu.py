"""Sequence-sharded decode on two GPUs (one process per GPU).

Each rank holds an R-aligned token range of one logical cache (the last rank
owns the residuals and appends); a decode step is partial attention on every
rank, an exchange of the packed (m, l, o) states and the rank-ordered merge.
Both exchange forms run on the same data: an NCCL all-gather between two
kernels, and one kernel that stores every rank's merged states straight into
its peers' buffers over NVLink.  The output on every rank must match the
oracle's single-device decode (runtime.rs:46-56) within the attention
tolerance, be bitwise identical across ranks, and the two exchange forms must
agree bit for bit.  A rank that skips a step makes the others' bounded peer
wait run out (about a second) and report it, without a hang.  Skipped on
machines with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

B, H, HQ, D, TOTAL, STEPS = 1, 4, 16, 128, 3 * 128 * 4 + 37, 5
ATOL, RTOL_L2 = 1e-4, 1e-5


def _inputs():
    from helpers import synthetic_kv

    k, v, ch = synthetic_kv(2024, B, H, TOTAL, D)
    rng = np.random.default_rng(11)
    steps = []
    for _ in range(STEPS):
        sk = rng.standard_normal((B, H, 1, D), dtype=np.float32) * ch[None, :, None, :]
        sv = rng.standard_normal((B, H, 1, D), dtype=np.float32)
        sq = rng.standard_normal((B, HQ, D), dtype=np.float32)
        steps.append((sk, sv, sq))
    return k.reshape(B, H, TOTAL, D), v.reshape(B, H, TOTAL, D), steps


def _worker(rank, world, port, q, exchange):
    import datetime

    import torch
    import torch.distributed as dist

    # NVLS (switch multicast) off: the failure case below must not involve it
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import kivi_cache as K
        from kivi_cache.sharding import SeqShardedCache

        keys, values, steps = _inputs()
        cfg = K.KiviConfig.try_new(2, 32, 128)
        sc = SeqShardedCache(cfg, B, H, D, TOTAL, device=rank, exchange=exchange)
        p = sc.plan
        dk = torch.from_numpy(np.ascontiguousarray(keys[:, :, p.start:p.end])).cuda()
        dv = torch.from_numpy(np.ascontiguousarray(values[:, :, p.start:p.end])).cuda()
        st = torch.cuda.Stream()
        torch.cuda.synchronize()
        if p.tokens:
            sc.prefill_local_dev(dk, dv, p.tokens, stream=st)
        st.synchronize()
        sc.finish_prefill()
        scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
        outs = []
        for sk, sv, sq in steps:
            o = sc.decode(torch.from_numpy(sk).pin_memory(), torch.from_numpy(sv).pin_memory(),
                          torch.from_numpy(sq).pin_memory(), HQ, scale, stream=st)
            outs.append(o.numpy().copy())
        skipped = None
        if exchange == "p2p":
            # rank 1 skips one step: rank 0's wait for its states runs out
            import ctypes as C
            import time

            if rank == 0:
                sq = torch.from_numpy(steps[0][2]).cuda()
                dout = torch.empty((B, HQ, D), device="cuda")
                t0 = time.monotonic()
                sc.cache.decode_exchange_dev(sc._peer_exchange(B * HQ), None, None, sq, HQ, scale,
                                             dout, stream=st)
                st.synchronize()
                err = K._Err()
                rc = K.lib().kivi_device_wait_status(rank, C.byref(err))
                skipped = (rc, err.message.decode(), time.monotonic() - t0,
                           float(dout.abs().max().item()))
            dist.barrier()
        sc.close()
        q.put((rank, p.start, p.end, np.stack(outs), skipped))
    except Exception as e:  # reported to the parent instead of a queue timeout
        q.put((rank, -1, -1, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(exchange):
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda r: r[0])
    for pr in procs:
        pr.join(timeout=60)
    for r in res:
        assert not isinstance(r[3], str), f"rank {r[0]} failed: {r[3]}"
    for pr in procs:
        assert pr.exitcode == 0
    return res


def test_seq_sharded_decode_two_gpus_nccl_and_peer_exchange():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    import oracle as O

    res = _run("nccl")
    peer = _run("p2p")
    for a, b in zip(res, peer):
        assert np.array_equal(a[3], b[3]), f"rank {a[0]}: peer exchange differs from the all-gather"
    rc, msg, waited, outmax = peer[0][4]
    assert rc == 100 and "8" in msg, (rc, msg)  # KIVI_ERR_CUDA with the exchange's flag
    assert waited < 30, waited
    assert outmax == 0.0
    assert res[0][1] == 0 and res[0][2] == res[1][1] and res[1][2] == TOTAL
    assert (res[0][2] - res[0][1]) % 128 == 0

    keys, values, steps = _inputs()
    oc = O.KiviCache(O.KiviConfig.try_new(2, 32, 128), B, H, D)
    oc.append(keys.reshape(-1), values.reshape(-1), TOTAL)
    scale = np.float32(1.0) / np.sqrt(np.float32(D))
    for i, (sk, sv, sq) in enumerate(steps):
        oc.append(sk.reshape(-1), sv.reshape(-1), 1)
        ref = oc.attention(sq.reshape(-1), HQ, scale)
        ref64 = oc.attention_f64(sq.reshape(-1), HQ, scale)
        for r in res:
            got = r[3][i].reshape(-1)
            err = np.abs(got - ref).max()
            rel = np.linalg.norm(got - ref64) / np.linalg.norm(ref64)
            assert err <= ATOL, f"step {i} rank {r[0]}: max-abs {err}"
            assert rel <= RTOL_L2, f"step {i} rank {r[0]}: rel-L2 vs fp64 {rel}"
        assert np.array_equal(res[0][3][i], res[1][3][i]), "ranks disagree"
