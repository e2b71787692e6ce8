"""The allocation-free attention entry point, kivi_cache_attention_noalloc_dev.

It serves callers that cannot call cudaMalloc while decoding (engines that
reserve nearly all device memory up front, decode loops that must not hit a
device-synchronising cudaMalloc/cudaFree): its scratch lives in a fixed array
of the library's device image.  It runs the same plan and kernels as
kivi_cache_attention_dev, so its output equals that call's bit for bit, and
both are checked against the CPU oracle.  This file is named to be collected
last.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from helpers import max_abs, rel_l2, synthetic_kv

pytestmark = pytest.mark.gpu

ATOL = 1e-4
RTOL_L2 = 1e-5


@pytest.fixture(scope="module")
def env():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import kivi_cache as K

    return torch, K


def _noalloc(K, cache, dq, hq, scale, dout, stream=None):
    err = K._Err()
    rc = K.lib().kivi_cache_attention_noalloc_dev(cache._h, dq.data_ptr(), hq, C.c_float(scale),
                                                  dout.data_ptr(), stream, C.byref(err))
    return rc, err


def test_noalloc_matches_attention_dev_and_oracle_on_two_calls(env):
    torch, K = env
    batch, kv, hq, dim, seq = 2, 8, 32, 128, 3000
    keys, values, _ = synthetic_kv(77, batch, kv, seq, dim)
    cache = K.KiviCache(K.KiviConfig(), batch, kv, dim)
    cache.append(keys, values, seq)
    ocache = O.KiviCache(O.KiviConfig(), batch, kv, dim)
    ocache.append(keys, values, seq)
    qh = np.random.default_rng(3).standard_normal(batch * hq * dim, dtype=np.float32)
    q = torch.from_numpy(qh).cuda()
    scale = float(np.float32(1.0) / np.sqrt(np.float32(128.0)))
    # first call on this device performs the one-time symbol-address set-up
    warm = torch.empty(batch * hq * dim, device="cuda")
    rc, err = _noalloc(K, cache, q, hq, scale, warm)
    assert rc == 0, err.message
    outs = [torch.full((batch * hq * dim,), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for out in outs:
        rc, err = _noalloc(K, cache, q, hq, scale, out)
        assert rc == 0, err.message
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    K.device_wait_status(0)
    ref = torch.empty(batch * hq * dim, device="cuda")
    cache.attention_dev(q, hq, scale, ref)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    want = ocache.attention(qh, hq, scale)
    want64 = ocache.attention_f64(qh, hq, scale)
    for out in outs:
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert (got.view(np.uint32) == ref.view(np.uint32)).all()  # same plan, same bits
        assert max_abs(got, want) <= ATOL
        assert rel_l2(got, want64) <= RTOL_L2
    # the host-pointer path (the reference-facing API) agrees as well
    host = cache.attention(qh, hq, scale)
    assert max_abs(outs[1].cpu().numpy(), host) <= ATOL


def test_noalloc_takes_a_config1_sized_call(env):
    """BASELINE config 1's shape (batch 16, 8 kv / 32 q heads, 2-bit, 32768
    tokens): the tensor-core plan's scratch fits the static array, and two calls
    in a row equal kivi_cache_attention_dev bit for bit."""
    torch, K = env
    batch, kv, hq, dim, seq = 16, 8, 32, 128, 32768
    cache = K.KiviCache(K.KiviConfig(), batch, kv, dim)
    cache.reserve(seq + 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    chunk = 2048
    for _ in range(seq // chunk):
        k = torch.randn(batch, kv, chunk, dim, device="cuda", generator=g)
        v = torch.randn(batch, kv, chunk, dim, device="cuda", generator=g)
        cache.append_dev(k, v, chunk)
    k = torch.randn(batch, kv, 1, dim, device="cuda", generator=g)
    v = torch.randn(batch, kv, 1, dim, device="cuda", generator=g)
    cache.append_dev(k, v, 1)
    q = torch.randn(batch * hq * dim, device="cuda", generator=g)
    scale = 1.0 / np.sqrt(128.0)
    ref = torch.empty(batch * hq * dim, device="cuda")
    cache.attention_dev(q, hq, scale, ref)
    outs = [torch.full((batch * hq * dim,), float("nan"), device="cuda") for _ in range(2)]
    for out in outs:
        rc, err = _noalloc(K, cache, q, hq, scale, out)
        assert rc == 0, err.message
    torch.cuda.synchronize()
    K.device_wait_status(0)
    for out in outs:
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32))


def test_noalloc_rejects_scratch_beyond_its_static_limit(env):
    torch, K = env
    # head_dim 64 runs the generic 256-token-chunk plan: 64 x 32 query rows x
    # ~38 slots x (64 + 2) floats > 16 MiB
    batch, kv, hq, dim, seq = 64, 8, 32, 64, 8192
    cache = K.KiviCache(K.KiviConfig(), batch, kv, dim)
    cache.reserve(seq)
    chunk = 1024
    for off in range(0, seq, chunk):
        k = torch.randn(batch, kv, chunk, dim, device="cuda")
        v = torch.randn(batch, kv, chunk, dim, device="cuda")
        cache.append_dev(k, v, chunk)
    q = torch.randn(batch * hq * dim, device="cuda")
    out = torch.zeros(batch * hq * dim, device="cuda")
    torch.cuda.synchronize()
    before = K.kernel_launches()
    rc, err = _noalloc(K, cache, q, hq, 0.1, out)
    assert rc == 103  # KIVI_ERR_UNSUPPORTED
    assert b"static limit" in err.message
    assert K.kernel_launches() == before  # rejected before any launch
    torch.cuda.synchronize()
    assert (out == 0).all()
