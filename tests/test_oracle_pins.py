"""Pins the CPU oracle to the reference's own known-answer tests.

Each test restates one test of bieli/kivi-cache-rs (file:line cited) against
``oracle`` (the C restatement).  Passing them is what makes the oracle a
trustworthy checker for the GPU path.  CPU only.
"""
import numpy as np
import pytest

import oracle as O
from helpers import (
    concat_head_major,
    dense_attend,
    document,
    fill,
    fill_wide,
    golden_tensor,
    max_abs,
    packed_word,
    slice_tokens,
    token_mean,
)


# ---------------------------------------------------------------- quant.rs tests


def test_pytorch_pack_matches_the_published_word_layout():
    """tests/quant.rs:13-41 and examples/pytorch_golden.rs:16-67"""
    dim, seq = 32, 64
    data = golden_tensor(seq, dim)
    kc, kp = O.quantize(True, data, 1, 1, seq, dim, 2, 32)
    vc, vp = O.quantize(False, data, 1, 1, seq, dim, 2, 32)
    key_codes = O.pytorch_codes(True, kc, 1, 1, seq, dim, 2, 32)
    value_codes = O.pytorch_codes(False, vc, 1, 1, seq, dim, 2, 32)
    assert key_codes.size == (seq // 16) * dim
    assert value_codes.size == seq * (dim // 16)
    rows = key_codes.reshape(-1, dim)
    assert (rows == rows[0]).all()
    assert key_codes[0] == 0xE4E4E4E4
    assert key_codes[1] == 0x39393939
    assert key_codes[2] == 0x4E4E4E4E
    assert key_codes[3] == 0x93939393
    assert value_codes[0] == 0xE4E4E4E4
    assert value_codes[1] == 0xE4E4E4E4
    assert value_codes[2] == 0x39393939
    # examples/pytorch_golden.rs:79-96: full golden vectors
    golden_keys = np.array([packed_word(d % 4) for d in range(dim)] * (seq // 16), np.uint32)
    golden_values = np.array([packed_word(t % 4) for t in range(seq) for _ in range(2)], np.uint32)
    assert (key_codes == golden_keys).all()
    assert (value_codes == golden_values).all()
    assert (kp.reshape(-1, 2) == [1.0, 0.0]).all()
    assert (vp.reshape(-1, 2) == [1.0, 0.0]).all()
    assert (O.dequantize_packed(True, kc, kp, 1, 1, seq, dim, 2, 32) == data).all()
    assert (O.dequantize_packed(False, vc, vp, 1, 1, seq, dim, 2, 32) == data).all()


def test_pytorch_golden_attention_is_exactly_1_5():
    """examples/pytorch_golden.rs:48-65"""
    data = golden_tensor(64, 32)
    cache = O.KiviCache(O.KiviConfig.try_new(2, 32, 32), 1, 1, 32)
    cache.append(data, data, 64)
    got = cache.attention(np.ones(32, np.float32), 1, 1.0 / np.sqrt(np.float32(32)))
    assert (got == np.float32(1.5)).all()
    assert cache.quantized_key_tokens() == 64
    assert cache.quantized_value_tokens() == 32


def test_four_bit_half_ties_round_to_even():
    """tests/quant.rs:43-66"""
    data = np.zeros(16, np.float32)
    data[[0, 1, 2, 3, 4, 5, 6, 15]] = [0.0, 0.5, 1.5, 2.5, 3.5, 1.2, 1.6, 15.0]
    c, p = O.quantize(False, data, 1, 1, 1, 16, 4, 16)
    out = O.dequantize_packed(False, c, p, 1, 1, 1, 16, 4, 16)
    assert list(out[[0, 1, 2, 3, 4, 5, 6, 15]]) == [0.0, 0.0, 2.0, 2.0, 4.0, 1.0, 2.0, 15.0]


def _pattern_token():
    v = np.ones(16, np.float32)
    v[:5] = [0.0, 0.5, 1.5, 2.5, 3.0]
    return v


EXPECT_HALF_EVEN = [0.0, 0.0, 2.0, 2.0, 3.0] + [1.0] * 11


def test_per_token_half_even_and_endpoints():
    """tests/quant.rs:68-77"""
    c, p = O.quantize(False, _pattern_token(), 1, 1, 1, 16, 2, 16)
    assert list(O.dequantize_packed(False, c, p, 1, 1, 1, 16, 2, 16)) == EXPECT_HALF_EVEN


def test_per_channel_half_even_on_one_channel():
    """tests/quant.rs:79-97"""
    data = np.zeros((16, 16), np.float32)
    data[:, 0] = _pattern_token()
    c, p = O.quantize(True, data, 1, 1, 16, 16, 2, 16)
    out = O.dequantize_packed(True, c, p, 1, 1, 16, 16, 2, 16).reshape(16, 16)
    assert list(out[:, 0]) == EXPECT_HALF_EVEN
    assert (out[:, 1:] == 0).all()


def test_negative_channel_endpoints_are_exact():
    """tests/quant.rs:99-116"""
    data = np.zeros((16, 16), np.float32)
    data[:4, 0] = [-2.0, -1.0, 0.0, 1.0]
    c, p = O.quantize(True, data, 1, 1, 16, 16, 2, 16)
    out = O.dequantize_packed(True, c, p, 1, 1, 16, 16, 2, 16).reshape(16, 16)
    assert list(out[:4, 0]) == [-2.0, -1.0, 0.0, 1.0]
    assert (out[4:, 0] == 0).all()


def test_constant_group_reconstructs_exactly():
    """tests/quant.rs:118-129"""
    data = np.full(2 * 3 * 32 * 16, 0.25, np.float32)
    for per_channel in (True, False):
        c, p = O.quantize(per_channel, data, 2, 3, 32, 16, 4, 16)
        assert (O.dequantize_packed(per_channel, c, p, 2, 3, 32, 16, 4, 16) == data).all()


def test_reconstruction_error_is_bounded_by_half_scale():
    """tests/quant.rs:131-168"""
    tokens = dim = 32
    data = fill_wide(tokens * dim)
    c, p = O.quantize(True, data, 1, 1, tokens, dim, 2, 32)
    out = O.dequantize_packed(True, c, p, 1, 1, tokens, dim, 2, 32).reshape(tokens, dim)
    x = data.reshape(tokens, dim)
    mn, mx = x.min(0), x.max(0)
    scale = np.where(mx == mn, 0, (mx - mn) / np.float32(3))
    assert (np.abs(out - x) <= scale * 0.5 + 1e-4).all()


def test_per_channel_keys_keep_quiet_channels():
    """tests/quant.rs:170-211"""
    tokens = dim = 32
    data = np.zeros((tokens, dim), np.float32)
    data[:, 0] = 100.0
    data[:, 1:] = (np.arange(1, dim, dtype=np.float32) / np.float32(dim))[None, :]
    pc = O.dequantize_packed(True, *O.quantize(True, data, 1, 1, tokens, dim, 2, 32),
                             1, 1, tokens, dim, 2, 32).reshape(tokens, dim)
    pt = O.dequantize_packed(False, *O.quantize(False, data, 1, 1, tokens, dim, 2, 32),
                             1, 1, tokens, dim, 2, 32).reshape(tokens, dim)
    assert np.abs(pc[:, 1:] - data[:, 1:]).mean() < 1e-5
    assert np.abs(pt[:, 1:] - data[:, 1:]).mean() > 0.2


def test_rejects_bad_shapes():
    """tests/quant.rs:213-228"""
    data = np.zeros(8, np.float32)
    with pytest.raises(O.OracleError) as e:
        O.quantize(True, data, 1, 1, 8, 1, 3, 32)
    assert e.value.variant == "InvalidBits" and e.value.a == 3
    with pytest.raises(O.OracleError) as e:
        O.quantize(True, data, 1, 1, 7, 1, 2, 32)
    assert e.value.variant == "TokenGroup"
    with pytest.raises(O.OracleError) as e:
        O.quantize(False, data, 1, 1, 4, 2, 2, 32)
    assert e.value.variant == "HeadDim"


def test_round_half_even_scalar():
    """quant.rs:474-485"""
    for x, r in [(0.5, 0.0), (1.5, 2.0), (2.5, 2.0), (3.5, 4.0), (2.4999998, 2.0), (7.0, 7.0)]:
        assert O.round_half_even(x) == r


# ---------------------------------------------------------------- cache.rs tests


def _cfg16():
    return O.KiviConfig.try_new(2, 16, 32)


def _append_chunks(cache, keys, values, total, chunks):
    off = 0
    for n in chunks:
        cache.append(slice_tokens(keys, cache.batch, cache.heads, total, cache.head_dim, off, n),
                     slice_tokens(values, cache.batch, cache.heads, total, cache.head_dim, off, n), n)
        off += n


def test_streaming_boundaries_match_algorithm_1():
    """tests/cache.rs:59-76"""
    dim = 16
    cache = O.KiviCache(_cfg16(), 2, 3, dim)
    steps = [10, 20, 5, 100]
    total = sum(steps)
    n = 2 * 3 * total * dim
    _append_chunks(cache, fill(n, 1), fill(n, 2), total, steps)
    r = 32
    assert cache.sequence_length() == total
    assert cache.key_residual_len() == total % r
    assert cache.value_residual_len() == min(r, total)
    assert cache.quantized_key_tokens() == total - total % r
    assert cache.quantized_value_tokens() == total - min(r, total)


def test_chunked_appends_match_token_by_token():
    """tests/cache.rs:78-104"""
    dim, batch, heads, total = 16, 2, 3, 70
    n = batch * heads * total * dim
    keys, values = fill(n, 7), fill(n, 9)
    streamed = O.KiviCache(_cfg16(), batch, heads, dim)
    _append_chunks(streamed, keys, values, total, [1] * total)
    chunked = O.KiviCache(_cfg16(), batch, heads, dim)
    _append_chunks(chunked, keys, values, total, [1, 50, 7, 12])
    once = O.KiviCache(_cfg16(), batch, heads, dim)
    once.append(keys, values, total)
    sk, sv = streamed.dequantize()
    ck, cv = chunked.dequantize()
    ok, ov = once.dequantize()
    assert (sk == ck).all() and (sv == cv).all() and (sk == ok).all() and (sv == ov).all()


def test_quantized_prefix_matches_one_shot_and_residual_is_exact():
    """tests/cache.rs:106-130"""
    dim, total = 16, 80
    keys, values = fill(total * dim, 3), fill(total * dim, 4)
    cache = O.KiviCache(_cfg16(), 1, 1, dim)
    cache.append(keys, values, total)
    kq, vq = cache.quantized_key_tokens(), cache.quantized_value_tokens()
    k_hat, v_hat = cache.dequantize()
    k_ref = O.dequantize_packed(True, *O.quantize(True, keys[:kq * dim], 1, 1, kq, dim, 2, 16),
                                1, 1, kq, dim, 2, 16)
    assert (k_hat[:kq * dim] == k_ref).all()
    assert (k_hat[kq * dim:] == keys[kq * dim:]).all()
    v_ref = O.dequantize_packed(False, *O.quantize(False, values[:vq * dim], 1, 1, vq, dim, 2, 16),
                                1, 1, vq, dim, 2, 16)
    assert (v_hat[:vq * dim] == v_ref).all()
    assert (v_hat[vq * dim:] == values[vq * dim:]).all()


def test_empty_append_and_shape_errors():
    """tests/cache.rs:132-145"""
    cache = O.KiviCache(_cfg16(), 1, 1, 16)
    cache.append(np.zeros(0), np.zeros(0), 0)
    assert cache.sequence_length() == 0
    with pytest.raises(O.OracleError) as e:
        cache.append(np.zeros(4), np.zeros(16), 1)
    assert (e.value.variant, e.value.a, e.value.b) == ("Shape", 16, 4)


def test_config_rejects_residual_that_is_not_a_group_multiple():
    """tests/cache.rs:147-158"""
    with pytest.raises(O.OracleError) as e:
        O.KiviConfig.try_new(2, 32, 100)
    assert e.value.variant == "ResidualLength"
    O.KiviCache(O.KiviConfig(), 1, 1, 96)
    with pytest.raises(O.OracleError) as e:
        O.KiviCache(O.KiviConfig(), 1, 1, 40)
    assert e.value.variant == "HeadDim"


def test_same_prompt_builds_the_same_cache_twice():
    """tests/cache.rs:160-194"""
    cfg = O.KiviConfig.try_new(2, 32, 32)
    keys = fill(64 * 32, 4)
    values = fill(64 * 32, 5)
    keys[3:6] = [0.5, 1.5, 2.5]
    qa, qb = fill(32, 8), fill(32, 9)
    first = O.KiviCache(cfg, 1, 1, 32)
    second = O.KiviCache(cfg, 1, 1, 32)
    first.append(keys, values, 64)
    second.append(keys, values, 64)
    for x, y in zip(first.dequantize(), second.dequantize()):
        assert (x == y).all()
    a = first.attention(qa, 1, 0.25)
    b = first.attention(qb, 1, 0.25)
    assert (a == second.attention(qa, 1, 0.25)).all()
    assert (b == second.attention(qb, 1, 0.25)).all()
    assert not (a == b).all()
    keys[0] = 50.0
    edited = O.KiviCache(cfg, 1, 1, 32)
    edited.append(keys, values, 64)
    assert not (first.dequantize()[0] == edited.dequantize()[0]).all()


def test_long_sequence_beats_fp16_footprint():
    """tests/cache.rs:196-207"""
    cache = O.KiviCache(O.KiviConfig.try_new(2, 32, 64), 1, 2, 64)
    n = 2 * 512 * 64
    cache.append(fill(n, 11), fill(n, 13), 512)
    m = cache.memory()
    compressed = sum(m[k] for k in ("key_code_bytes", "key_metadata_bytes", "value_code_bytes",
                                    "value_metadata_bytes", "key_residual_bytes",
                                    "value_residual_bytes"))
    assert m["fp16_baseline_bytes"] / compressed > 2.0
    assert m["key_residual_bytes"] == 0


# ---------------------------------------------------------------- attention.rs tests


def _assert_matches_dequantized(bits, group, residual, dim, seq):
    cache = O.KiviCache(O.KiviConfig.try_new(bits, group, residual), 1, 1, dim)
    cache.append(fill(seq * dim, 21), fill(seq * dim, 22), seq)
    k_hat, v_hat = cache.dequantize()
    q = fill(dim, 23)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(dim)))
    got = cache.attention(q, 1, scale)
    expect = dense_attend(k_hat, v_hat, q, 1, 1, 1, seq, dim, scale)
    assert max_abs(got, expect) < 1e-4


def test_generic_kernel_matches_dequantized_attention():
    """tests/attention.rs:61-65"""
    _assert_matches_dequantized(2, 16, 32, 16, 40)
    _assert_matches_dequantized(4, 32, 64, 32, 70)


def test_fast_2bit_group32_kernel_matches_dequantized_attention():
    """tests/attention.rs:67-70"""
    _assert_matches_dequantized(2, 32, 64, 64, 100)


def test_grouped_query_attention_repeats_kv_heads():
    """tests/attention.rs:72-101"""
    dim, batch, kv, qh, seq = 32, 2, 2, 4, 48
    cache = O.KiviCache(O.KiviConfig.try_new(2, 32, 64), batch, kv, dim)
    cache.append(fill(batch * kv * seq * dim, 31), fill(batch * kv * seq * dim, 32), seq)
    k_hat, v_hat = cache.dequantize()
    q = fill(batch * qh * dim, 33)
    got = cache.attention(q, qh, 0.125)
    expect = dense_attend(k_hat, v_hat, q, batch, kv, qh, seq, dim, 0.125)
    assert max_abs(got, expect) < 1e-4


def test_empty_cache_attention_is_zero():
    """tests/attention.rs:103-108"""
    cache = O.KiviCache(O.KiviConfig(), 1, 2, 128)
    assert (cache.attention(np.full(256, 0.2, np.float32), 2, 1.0) == 0).all()


def test_rejects_query_head_count_that_is_not_a_multiple():
    """tests/attention.rs:110-114"""
    cache = O.KiviCache(O.KiviConfig.try_new(2, 16, 32), 1, 2, 16)
    with pytest.raises(O.OracleError):
        cache.attention(np.zeros(48, np.float32), 3, 1.0)


# ---------------------------------------------------------------- runtime.rs tests


def test_runtime_decode_matches_direct_cache():
    """tests/runtime.rs:13-52 (RuntimeKv::decode = append(1) + attention, runtime.rs:46-56)"""
    cfg = O.KiviConfig.try_new(2, 32, 32)
    batch, kv, qh, dim, prompt = 1, 2, 4, 32, 40
    scale = float(np.float32(1.0) / np.sqrt(np.float32(dim)))
    keys = fill(batch * kv * prompt * dim, 3)
    values = fill(batch * kv * prompt * dim, 4)
    cache = O.KiviCache(cfg, batch, kv, dim)
    cache.append(keys, values, prompt)
    previous = None
    for step in range(3):
        k = fill(batch * kv * dim, 10 + step)
        v = fill(batch * kv * dim, 20 + step)
        q = fill(batch * qh * dim, 30 + step)
        cache.append(k, v, 1)
        got = cache.attention(q, qh, scale)
        if previous is not None:
            assert not (got == previous).all()
        previous = got
    assert cache.sequence_length() == prompt + 3


# ---------------------------------------------------------------- prefix.rs tests


def _share(cfg, batch, heads, dim, seq):
    keys, values = document(batch, heads, seq, dim)
    cache = O.KiviCache(cfg, batch, heads, dim)
    cache.append(keys, values, seq)
    return cache, cache.share_prefix()


def test_empty_question_matches_cache_attention():
    """tests/prefix.rs:112-124"""
    cache, prefix = _share(O.KiviConfig.try_new(2, 32, 64), 1, 2, 64, 96)
    q = np.full(4 * 64, 0.3, np.float32)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(64)))
    assert (prefix.session().attention(q, 4, scale) == cache.attention(q, 4, scale)).all()


def test_question_attention_matches_dense_prefix_plus_suffix():
    """tests/prefix.rs:126-160"""
    batch, heads, dim, doc, qlen = 1, 2, 64, 96, 4
    cache, prefix = _share(O.KiviConfig.try_new(2, 32, 64), batch, heads, dim, doc)
    dk, dv = cache.dequantize()
    s = prefix.session()
    qk, qv = document(batch, heads, qlen, dim)
    s.append(qk, qv, qlen)
    q = np.full(batch * heads * dim, 0.15, np.float32)
    got = s.attention(q, heads, 0.25)
    expect = dense_attend(concat_head_major(dk, qk, batch, heads, doc, qlen, dim),
                          concat_head_major(dv, qv, batch, heads, doc, qlen, dim),
                          q, batch, heads, heads, doc + qlen, dim, 0.25)
    assert max_abs(got, expect) < 1e-4


def test_constant_keys_make_suffix_attention_the_value_mean():
    """tests/prefix.rs:243-273"""
    batch, heads, dim, doc, qlen = 1, 2, 32, 96, 4
    cfg = O.KiviConfig.try_new(2, 32, 64)
    keys = np.zeros(batch * heads * doc * dim, np.float32)
    values = document(batch, heads, doc, dim)[1]
    cache = O.KiviCache(cfg, batch, heads, dim)
    cache.append(keys, values, doc)
    assert cache.key_residual_len() == doc % 64 and cache.value_residual_len() == 64
    s = cache.share_prefix().session()
    qv = document(batch, heads, qlen, dim)[1]
    s.append(np.zeros(batch * heads * qlen * dim, np.float32), qv, qlen)
    dk, dv = cache.dequantize()
    assert (dk == 0).all()
    expect = token_mean(concat_head_major(dv, qv, batch, heads, doc, qlen, dim), batch, heads,
                        doc + qlen, dim)
    got = s.attention(np.ones(batch * heads * dim, np.float32), heads, 3.5)
    assert max_abs(got, expect) < 1e-5


def test_four_bit_suffix_matches_dense_attention():
    """tests/prefix.rs:275-307"""
    batch, heads, dim, doc, qlen = 1, 1, 64, 90, 6
    cache, prefix = _share(O.KiviConfig.try_new(4, 32, 64), batch, heads, dim, doc)
    assert cache.key_residual_len() == 26 and cache.value_residual_len() == 64
    dk, dv = cache.dequantize()
    s = prefix.session()
    qk, qv = document(batch, heads, qlen, dim)
    s.append(qk, qv, qlen)
    q = document(batch, heads, 1, dim)[0]
    scale = float(np.float32(1.0) / np.sqrt(np.float32(dim)))
    got = s.attention(q, heads, scale)
    expect = dense_attend(concat_head_major(dk, qk, batch, heads, doc, qlen, dim),
                          concat_head_major(dv, qv, batch, heads, doc, qlen, dim),
                          q, batch, heads, heads, doc + qlen, dim, scale)
    assert max_abs(got, expect) < 1e-4


def test_grouped_query_batch_suffix_matches_dense_attention():
    """tests/prefix.rs:309-340"""
    batch, kv, qh, dim, doc, qlen = 2, 2, 6, 32, 48, 3
    cache, prefix = _share(O.KiviConfig.try_new(2, 32, 32), batch, kv, dim, doc)
    dk, dv = cache.dequantize()
    s = prefix.session()
    qk, qv = document(batch, kv, qlen, dim)
    s.append(qk, qv, qlen)
    q = document(batch, qh, 1, dim)[0]
    got = s.attention(q, qh, 0.5)
    expect = dense_attend(concat_head_major(dk, qk, batch, kv, doc, qlen, dim),
                          concat_head_major(dv, qv, batch, kv, doc, qlen, dim),
                          q, batch, kv, qh, doc + qlen, dim, 0.5)
    assert max_abs(got, expect) < 1e-4


def test_chunked_question_append_matches_one_shot():
    """tests/prefix.rs:342-366"""
    batch, heads, dim, doc = 2, 2, 32, 40
    _, prefix = _share(O.KiviConfig.try_new(2, 32, 32), batch, heads, dim, doc)
    qk, qv = document(batch, heads, 7, dim)
    chunked = prefix.session()
    chunked.append(slice_tokens(qk, batch, heads, 7, dim, 0, 2),
                   slice_tokens(qv, batch, heads, 7, dim, 0, 2), 2)
    chunked.append(slice_tokens(qk, batch, heads, 7, dim, 2, 5),
                   slice_tokens(qv, batch, heads, 7, dim, 2, 5), 5)
    once = prefix.session()
    once.append(qk, qv, 7)
    q = np.full(batch * heads * dim, 0.4, np.float32)
    assert (chunked.attention(q, heads, 1.25) == once.attention(q, heads, 1.25)).all()


def test_matching_suffix_key_dominates_the_softmax():
    """tests/prefix.rs:368-386"""
    dim, doc = 32, 40
    cache = O.KiviCache(O.KiviConfig.try_new(2, 32, 32), 1, 1, dim)
    cache.append(np.full(doc * dim, 0.01, np.float32), np.zeros(doc * dim, np.float32), doc)
    s = cache.share_prefix().session()
    s.append(np.ones(dim, np.float32), np.full(dim, 5.0, np.float32), 1)
    got = s.attention(np.ones(dim, np.float32), 1, 20.0)
    assert max_abs(got, np.full(dim, 5.0)) < 1e-3


def test_question_only_session_matches_dense_attention():
    """tests/prefix.rs:388-401"""
    cache = O.KiviCache(O.KiviConfig.try_new(2, 32, 64), 1, 2, 64)
    s = cache.share_prefix().session()
    qk, qv = document(1, 2, 5, 64)
    s.append(qk, qv, 5)
    q = np.full(2 * 64, 0.2, np.float32)
    got = s.attention(q, 2, 0.7)
    assert max_abs(got, dense_attend(qk, qv, q, 1, 2, 2, 5, 64, 0.7)) < 1e-5


def test_bad_query_shape_and_head_count_are_rejected():
    """tests/prefix.rs:459-479"""
    _, prefix = _share(O.KiviConfig.try_new(2, 32, 64), 1, 2, 64, 32)
    s = prefix.session()
    with pytest.raises(O.OracleError) as e:
        s.attention(np.zeros(64, np.float32), 3, 1.0)
    assert (e.value.variant, e.value.a, e.value.b) == ("QueryHeads", 3, 2)
    with pytest.raises(O.OracleError) as e:
        s.attention(np.zeros(8, np.float32), 2, 1.0)
    assert (e.value.variant, e.value.a, e.value.b) == ("Shape", 128, 8)


# ---------------------------------------------------------------- budget.rs tests


def test_planner_bytes_match_live_cache():
    """tests/budget.rs:68-82"""
    cfg = O.KiviConfig()
    for seq in [1, 32, 127, 128, 129, 512, 2048]:
        cache = O.KiviCache(cfg, 1, 8, 128)
        n = 8 * seq * 128
        cache.append(np.full(n, 0.1, np.float32), np.full(n, 0.1, np.float32), seq)
        m = cache.memory()
        live = sum(m[k] for k in ("key_code_bytes", "key_metadata_bytes", "value_code_bytes",
                                  "value_metadata_bytes", "key_residual_bytes",
                                  "value_residual_bytes"))
        assert O.layer_kv_bytes(cfg, 8, 128, seq) == live


def test_marginal_rate_matches_one_key_flush_cycle():
    """tests/budget.rs:84-91, budget.rs:349-364 (1024 B for 8 heads at d=128, the reference README.md:176)"""
    cfg = O.KiviConfig()
    start = 128 * 40
    delta = O.layer_kv_bytes(cfg, 8, 128, start + 128) - O.layer_kv_bytes(cfg, 8, 128, start)
    assert delta // 128 == O.marginal_bytes_per_layer(cfg, 8, 128) == 1024
