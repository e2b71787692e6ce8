"""QualityGuard (guard.rs): the reference's own tests (tests/guard.rs) against
the C oracle on the CPU and against the device guard on the GPU, plus a
multi-head, multi-flush comparison of every flush check (cosines within the
attention tolerance, identical upgrade decisions).
"""
import math

import numpy as np
import pytest

import oracle as O


def signal(seq, dim, seed):
    """tests/guard.rs:3-11 (32-bit LCG -> uniform [-1, 1), exact in fp32)."""
    out = np.empty(seq * dim, np.float32)
    state = seed
    for i in range(seq * dim):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = ((state >> 8) / float(1 << 24)) * 2.0 - 1.0
    return out


def make_oracle_guard(policy, threshold, max_bits, max_residual):
    """tests/guard.rs:13-26"""
    return O.QualityGuard.try_new(O.KiviConfig.try_new(2, 32, 32), 1, 1, 32, threshold, policy,
                                  max_bits, max_residual)


def make_device_guard(policy, threshold, max_bits, max_residual):
    import kivi_cache as K

    return K.QualityGuard.try_new(K.KiviConfig.try_new(2, 32, 32), 1, 1, 32, threshold, policy,
                                  max_bits, max_residual)


def run_reference_cases(make, P, U):
    """tests/guard.rs:28-124, with guard constructor `make`, policy class P and
    upgrade class U (the oracle's or the device's)."""
    # no_flush_means_no_check (guard.rs:28-37)
    g = make(P.RaiseBits, 0.99, 8, 128)
    checks = g.append(signal(16, 32, 1), signal(16, 32, 2), 16, signal(1, 32, 3), 1, 0.5)
    assert checks == []
    assert g.config().bits == 2
    assert g.sequence_length() == 16

    # passing_cosine_does_not_upgrade (guard.rs:39-52)
    g = make(P.RaiseBits, 0.0, 8, 128)
    checks = g.append(signal(32, 32, 4), signal(32, 32, 5), 32, signal(1, 32, 6), 1, 0.5)
    assert len(checks) == 1
    assert checks[0].upgrades == []
    assert checks[0].cosine_before == checks[0].cosine
    assert checks[0].sequence_tokens == 32
    assert g.config().bits == 2
    assert g.config().residual_length == 32

    # raise_bits_stops_at_the_ceiling (guard.rs:54-69)
    g = make(P.RaiseBits, 1.1, 4, 128)
    checks = g.append(signal(32, 32, 7), signal(32, 32, 8), 32, signal(1, 32, 9), 1, 0.5)
    assert checks[0].upgrades == [U.Bits(2, 4)]
    assert g.config().bits == 4
    assert g.config().residual_length == 32
    assert g.cache().sequence_length() == 32
    assert checks[0].cosine < 1.1

    # lengthen_residual_puts_the_flushed_block_back_in_fp32 (guard.rs:71-89)
    g = make(P.LengthenResidual, 1.1, 8, 64)
    checks = g.append(signal(32, 32, 10), signal(32, 32, 11), 32, signal(1, 32, 12), 1, 0.25)
    assert checks[0].upgrades == [U.Residual(32, 64)]
    assert g.config().residual_length == 64
    assert g.config().bits == 2
    c = g.cache()
    assert c.quantized_key_tokens() == 0
    assert c.quantized_value_tokens() == 0
    assert c.key_residual_len() == 32
    assert c.value_residual_len() == 32
    assert checks[0].cosine > 0.999, checks[0].cosine

    # one_append_checks_every_key_flush (guard.rs:91-102)
    g = make(P.RaiseBits, 0.0, 8, 128)
    checks = g.append(signal(64, 32, 13), signal(64, 32, 14), 64, signal(1, 32, 15), 1, 0.5)
    assert len(checks) == 2
    assert checks[0].sequence_tokens == 32
    assert checks[1].sequence_tokens == 64
    assert all(not c.upgrades for c in checks)

    # four_bit_rebuild_beats_the_two_bit_flush (guard.rs:104-124)
    keys, values, query = signal(32, 32, 21), signal(32, 32, 22), signal(1, 32, 23)
    scale = 1.0 / math.sqrt(32.0)
    loose = make(P.RaiseBits, 0.0, 8, 128)
    before = loose.append(keys, values, 32, query, 1, scale)[0].cosine_before
    g = make(P.RaiseBits, 0.995, 8, 128)
    checks = g.append(keys, values, 32, query, 1, scale)
    assert before < 0.995, f"2-bit cosine {before} did not miss 0.995"
    assert checks[0].upgrades == [U.Bits(2, 4)]
    assert checks[0].cosine > before
    assert checks[0].cosine >= 0.995, checks[0].cosine
    assert g.config().bits == 4


# ---------------------------------------------------------------- CPU: the oracle


def test_oracle_guard_passes_the_reference_tests():
    run_reference_cases(make_oracle_guard, O.QualityPolicy, O.QualityUpgrade)


def test_oracle_fp32_attention_matches_float64():
    """guard.rs:294-341 against a float64 evaluation of the same formula."""
    rng = np.random.default_rng(5)
    B, H, Hq, T, D = 2, 2, 4, 70, 16
    q = rng.standard_normal(B * Hq * D).astype(np.float32)
    k = rng.standard_normal(B * H * T * D).astype(np.float32)
    v = rng.standard_normal(B * H * T * D).astype(np.float32)
    got = O.fp32_attention(q, k, v, B, H, Hq, T, D, 0.25)
    qq = q.reshape(B, Hq, D).astype(np.float64)
    kk = k.reshape(B, H, T, D).astype(np.float64)
    vv = v.reshape(B, H, T, D).astype(np.float64)
    ref = np.zeros((B, Hq, D))
    for b in range(B):
        for h in range(Hq):
            x = kk[b, h // (Hq // H)] @ qq[b, h] * 0.25
            w = np.exp(x - x.max())
            ref[b, h] = (w / w.sum()) @ vv[b, h // (Hq // H)]
    assert np.max(np.abs(got - ref.reshape(-1))) < 1e-5
    assert O.cosine_sim(got, got) == pytest.approx(1.0, abs=1e-6)
    assert O.cosine_sim(np.zeros(4), np.zeros(4)) == 1.0


def test_oracle_guard_validates_like_the_reference():
    """guard.rs:103-127: Shape for keys/values, QueryHeads, Shape for the query."""
    g = make_oracle_guard(O.QualityPolicy.RaiseBits, 0.0, 8, 128)
    k = signal(4, 32, 1)
    with pytest.raises(O.OracleError) as e:
        g.append(k[:-1], k, 4, signal(1, 32, 3), 1, 0.5)
    assert (e.value.variant, e.value.a, e.value.b) == ("Shape", 128, 127)
    with pytest.raises(O.OracleError) as e:
        g.append(k, k, 4, signal(1, 32, 3), 0, 0.5)
    assert e.value.variant == "QueryHeads"
    with pytest.raises(O.OracleError) as e:
        g.append(k, k, 4, signal(2, 32, 3), 1, 0.5)
    assert (e.value.variant, e.value.a, e.value.b) == ("Shape", 32, 64)
    assert g.sequence_length() == 0


# ---------------------------------------------------------------- GPU: the device guard


@pytest.mark.gpu
def test_device_guard_passes_the_reference_tests():
    import kivi_cache as K

    run_reference_cases(make_device_guard, K.QualityPolicy, K.QualityUpgrade)


@pytest.mark.gpu
def test_device_guard_reference_cases_match_the_oracle():
    """The same cases, every check's cosines against the oracle's."""
    import kivi_cache as K

    cases = [
        ("RaiseBits", 0.0, 8, 128, 32, (4, 5, 6), 0.5),
        ("RaiseBits", 1.1, 4, 128, 32, (7, 8, 9), 0.5),
        ("LengthenResidual", 1.1, 8, 64, 32, (10, 11, 12), 0.25),
        ("RaiseBits", 0.0, 8, 128, 64, (13, 14, 15), 0.5),
        ("RaiseBits", 0.995, 8, 128, 32, (21, 22, 23), 1.0 / math.sqrt(32.0)),
    ]
    for pol, thr, mb, mr, seq, seeds, scale in cases:
        go = make_oracle_guard(getattr(O.QualityPolicy, pol), thr, mb, mr)
        gd = make_device_guard(getattr(K.QualityPolicy, pol), thr, mb, mr)
        args = (signal(seq, 32, seeds[0]), signal(seq, 32, seeds[1]), seq, signal(1, 32, seeds[2]),
                1, scale)
        co, cd = go.append(*args), gd.append(*args)
        assert len(co) == len(cd)
        for a, b in zip(co, cd):
            assert a.sequence_tokens == b.sequence_tokens
            assert [tuple(u) for u in a.upgrades] == [tuple(u) for u in b.upgrades]
            assert abs(a.cosine_before - b.cosine_before) < 5e-5
            assert abs(a.cosine - b.cosine) < 5e-5
        assert go.config().bits == gd.config().bits
        assert go.config().residual_length == gd.config().residual_length


@pytest.mark.gpu
@pytest.mark.parametrize("policy", ["RaiseBits", "LengthenResidual"])
def test_device_guard_multi_head_multi_flush_matches_the_oracle(policy):
    """GQA 2, head_dim 128 (the tensor-core attention path), several appends
    crossing several flushes, thresholds that force upgrades midway."""
    import kivi_cache as K

    rng = np.random.default_rng(11 if policy == "RaiseBits" else 12)
    B, H, Hq, D = 2, 2, 4, 128
    cfg_o, cfg_d = O.KiviConfig.try_new(2, 32, 64), K.KiviConfig.try_new(2, 32, 64)
    thr = 0.9995
    go = O.QualityGuard.try_new(cfg_o, B, H, D, thr, getattr(O.QualityPolicy, policy), 8, 256)
    gd = K.QualityGuard.try_new(cfg_d, B, H, D, thr, getattr(K.QualityPolicy, policy), 8, 256)
    chs = np.exp(rng.standard_normal((H, D))).astype(np.float32)
    q = rng.standard_normal(B * Hq * D).astype(np.float32)
    for n in (50, 100, 130, 40):
        k = (rng.standard_normal((B, H, n, D)) * chs[None, :, None, :]).astype(np.float32)
        v = rng.standard_normal((B, H, n, D)).astype(np.float32)
        co = go.append(k, v, n, q, Hq, 1.0 / math.sqrt(D))
        cd = gd.append(k, v, n, q, Hq, 1.0 / math.sqrt(D))
        assert len(co) == len(cd)
        for a, b in zip(co, cd):
            assert a.sequence_tokens == b.sequence_tokens
            assert [tuple(u) for u in a.upgrades] == [tuple(u) for u in b.upgrades]
            assert abs(a.cosine_before - b.cosine_before) < 5e-5, (a, b)
            assert abs(a.cosine - b.cosine) < 5e-5, (a, b)
    assert gd.sequence_length() == go.sequence_length() == 320
    assert (gd.config().bits, gd.config().residual_length) == (go.config().bits,
                                                                go.config().residual_length)
    st_o, st_d = go.cache(), gd.cache()
    assert st_d.quantized_key_tokens() == st_o.quantized_key_tokens()
    assert st_d.key_residual_len() == st_o.key_residual_len()
