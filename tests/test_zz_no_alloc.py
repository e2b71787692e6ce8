"""The allocation-free attention entry point, kivi_cache_attention_noalloc_dev.

It serves callers that cannot call cudaMalloc while decoding (engines that
reserve nearly all device memory up front, decode loops that must not hit a
device-synchronising cudaMalloc/cudaFree): its scratch lives in a fixed array
of the library's device image.  This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

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


def test_noalloc_matches_attention_dev_on_two_calls(env):
    torch, K = env
    batch, kv, hq, dim, seq = 2, 8, 32, 128, 3000
    keys, values, _ = synthetic_kv(77, batch, kv, seq, dim)
    cache = K.KiviCache(K.KiviConfig(), batch, kv, dim)
    cache.append(keys, values, seq)
    q = torch.from_numpy(np.random.default_rng(3).standard_normal(batch * hq * dim, dtype=np.float32)).cuda()
    scale = 1.0 / np.sqrt(128.0)
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
    ref = torch.empty(batch * hq * dim, device="cuda")
    cache.attention_dev(q, hq, scale, ref)
    torch.cuda.synchronize()
    ref = ref.cpu().numpy()
    for out in outs:
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        assert max_abs(got, ref) <= ATOL
        assert rel_l2(got, ref) <= RTOL_L2
    # the host-pointer path (the reference-facing API) agrees as well
    host = cache.attention(q.cpu().numpy(), hq, scale)
    assert max_abs(outs[1].cpu().numpy(), host) <= ATOL


def test_noalloc_rejects_scratch_beyond_its_static_limit(env):
    torch, K = env
    # 64 x 8 kv heads x 32 q heads x (128 + 2) floats x ~34 slots > 16 MiB
    batch, kv, hq, dim, seq = 64, 8, 32, 128, 8192
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
    rc, err = _noalloc(K, cache, q, hq, 0.1, out)
    assert rc == 103  # KIVI_ERR_UNSUPPORTED
    assert b"static limit" in err.message
    torch.cuda.synchronize()
    assert (out == 0).all()
