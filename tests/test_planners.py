"""Budget and economics planners (budget.rs:157-314 MixedPrecisionBudget,
econ.rs): the reference's own tests (tests/budget.rs:127-236, tests/econ.rs)
against the host mirror, with the live-cache byte checks against the oracle's
memory() on the CPU and the device cache's memory() on the GPU.
"""
import numpy as np
import pytest

import kivi_cache as K
import oracle as O


def compressed(m):
    keys = ("key_code_bytes", "key_metadata_bytes", "value_code_bytes", "value_metadata_bytes",
            "key_residual_bytes", "value_residual_bytes")
    if isinstance(m, dict):
        return sum(m[k] for k in keys)
    return m.compressed_bytes()


# ---------------------------------------------------------------- budget.rs


def test_mixed_precision_sums_wide_and_narrow_layers():
    """tests/budget.rs:127-150"""
    tokens, heads, dim = 200_000, 8, 128
    mixed = K.MixedPrecisionBudget.early_wide(32, 8, 4, 2, 32, 128, heads, dim)
    assert mixed.num_layers() == 32
    assert mixed.layer_bits(0) == 4 and mixed.layer_bits(7) == 4
    assert mixed.layer_bits(8) == 2 and mixed.layer_bits(31) == 2
    assert mixed.layer_bits(32) is None
    wide = K.AgentMemoryBudget.try_new(K.KiviConfig.try_new(4, 32, 128), 8, heads, dim)
    narrow = K.AgentMemoryBudget.try_new(K.KiviConfig.try_new(2, 32, 128), 24, heads, dim)
    assert mixed.bytes_for_context(tokens) == wide.bytes_for_context(tokens) + narrow.bytes_for_context(tokens)
    assert mixed.bytes_for_layer(0, tokens) > mixed.bytes_for_layer(31, tokens)


def test_mixed_layer_bytes_match_live_oracle_caches():
    """tests/budget.rs:152-167 with the oracle's caches (pinned to the reference's memory())."""
    plan = K.MixedPrecisionBudget.early_wide(2, 1, 4, 2, 32, 128, 4, 64)
    seq, total = 300, 0
    for layer, bits in ((0, 4), (1, 2)):
        cache = O.KiviCache(O.KiviConfig.try_new(bits, 32, 128), 1, 4, 64)
        n = 4 * seq * 64
        cache.append(np.full(n, 0.15, np.float32), np.full(n, -0.2, np.float32), seq)
        live = compressed(cache.memory())
        assert plan.bytes_for_layer(layer, seq) == live
        total += live
    assert plan.bytes_for_context(seq) == total


@pytest.mark.gpu
def test_mixed_layer_bytes_match_live_device_caches():
    """tests/budget.rs:152-167 with the device caches."""
    plan = K.MixedPrecisionBudget.early_wide(2, 1, 4, 2, 32, 128, 4, 64)
    seq, total = 300, 0
    for layer, bits in ((0, 4), (1, 2)):
        cache = K.KiviCache(K.KiviConfig.try_new(bits, 32, 128), 1, 4, 64)
        n = 4 * seq * 64
        cache.append(np.full(n, 0.15, np.float32), np.full(n, -0.2, np.float32), seq)
        live = compressed(cache.memory())
        assert plan.bytes_for_layer(layer, seq) == live
        total += live
    assert plan.bytes_for_context(seq) == total


def test_mixed_precision_sits_between_uniform_budgets():
    """tests/budget.rs:169-191"""
    heads, dim, tokens = 8, 128, 8_192
    mixed = K.MixedPrecisionBudget.early_wide(32, 8, 4, 2, 32, 128, heads, dim)
    all2 = K.AgentMemoryBudget.try_new(K.KiviConfig.try_new(2, 32, 128), 32, heads, dim)
    all4 = K.AgentMemoryBudget.try_new(K.KiviConfig.try_new(4, 32, 128), 32, heads, dim)
    one = mixed.bytes_for_context(tokens)
    assert all4.bytes_for_context(tokens) > one > all2.bytes_for_context(tokens)
    budget = one * 3
    assert mixed.max_agents(budget, tokens) == 3
    assert mixed.fits(budget, 3, tokens) and not mixed.fits(budget, 4, tokens)
    assert all4.max_agents(budget, tokens) < mixed.max_agents(budget, tokens)
    assert all2.max_agents(budget, tokens) >= mixed.max_agents(budget, tokens)
    assert mixed.bytes_for_agents(3, tokens) == one * 3


def test_mixed_marginal_matches_one_flush_cycle():
    """tests/budget.rs:192-204"""
    plan = K.MixedPrecisionBudget.early_wide(4, 1, 4, 2, 32, 64, 2, 64)
    cycle = plan.residual_length()
    start = cycle * 40
    delta = plan.bytes_for_context(start + cycle) - plan.bytes_for_context(start)
    assert delta // cycle == plan.marginal_bytes_per_token()
    assert plan.next_token_bytes(start) == plan.bytes_for_context(start + 1) - plan.bytes_for_context(start)


def test_uniform_bit_schedule_matches_agent_budget():
    """tests/budget.rs:205-220"""
    cfg = K.KiviConfig.try_new(2, 32, 128)
    mixed = K.MixedPrecisionBudget.early_wide(16, 0, 4, 2, 32, 128, 8, 128)
    plan = K.AgentMemoryBudget.try_new(cfg, 16, 8, 128)
    assert mixed.layer_bits(0) == 2
    assert mixed.bytes_for_context(4096) == plan.bytes_for_context(4096)
    assert mixed.fp16_bytes_for_agents(2, 4096) == plan.fp16_bytes_for_agents(2, 4096)
    ratio = mixed.fp16_bytes_for_agents(2, 4096) / mixed.bytes_for_agents(2, 4096)
    assert abs(mixed.compression_ratio_vs_fp16(2, 4096) - ratio) < 1e-12


def test_mixed_precision_rejects_bad_schedules():
    """tests/budget.rs:221-235"""
    with pytest.raises(K.KiviError) as e:
        K.MixedPrecisionBudget.early_wide(8, 9, 4, 2, 32, 128, 8, 128)
    assert (e.value.variant, e.value.a, e.value.b) == ("EarlyLayers", 9, 8)
    with pytest.raises(K.KiviError) as e:
        K.MixedPrecisionBudget.try_from_bits([], 32, 128, 8, 128)
    assert e.value.variant == "ZeroDimension" and e.value.name == "num_layers"
    with pytest.raises(K.KiviError) as e:
        K.MixedPrecisionBudget.early_wide(4, 2, 4, 2, 8, 32, 1, 32)
    assert e.value.variant == "MisalignedGroup"


# ---------------------------------------------------------------- econ.rs (tests/econ.rs)


def test_parse_context_suffixes():
    assert K.parse_context_tokens("128k") == 128_000
    assert K.parse_context_tokens("1.5m") == 1_500_000
    assert K.parse_context_tokens("4096") == 4096
    assert K.parse_context_tokens(" 200_K ") == 200_000
    for bad in ("", "abc", "-1k"):
        with pytest.raises(ValueError):
            K.parse_context_tokens(bad)


def test_wider_gpu_fits_more_agents_than_fp16():
    preset = K.ModelPreset.by_id("llama3-8b")
    inputs = preset.to_inputs(K.KiviConfig.default(), 128_000, 16,
                              K.kv_budget_bytes(80.0, preset.weight_gib), 1.10)
    report = K.compute_report(inputs)
    assert report.kv_saved_gib > 0.0
    assert report.compression_ratio > 2.0
    assert report.max_agents_on_gpu >= report.max_agents_fp16_on_gpu


def test_cli_example_llama3_16_agents_128k():
    preset = K.ModelPreset.by_id("llama3-8b")
    inputs = preset.to_inputs(K.KiviConfig.try_new(2, 32, 128), K.parse_context_tokens("128k"), 16,
                              K.kv_budget_bytes(24.0, preset.weight_gib), 1.10)
    report = K.compute_report(inputs)
    assert report.kv_saved_gib > 1.0
    assert report.compression_ratio > 2.0
    assert report.agents == 16
    assert report.context_tokens == 128_000


def test_pretrain_bill_uses_gpu_count_and_planned_hours():
    preset = K.ModelPreset.by_id("llama3-8b")
    hours, rate = 8.0, 2.40
    budget = K.kv_budget_bytes(24.0, preset.weight_gib)
    inputs = preset.to_inputs(K.KiviConfig.try_new(2, 32, 128), 32_768, 4, budget, rate)
    report = K.compute_report(inputs)
    est = K.estimate_pretrain(inputs, hours)
    assert est.context_tokens == 32_768 and est.batch == 4
    assert abs(est.kivi_kv_gib - report.kivi_kv_gib) < 1e-12
    assert abs(est.fp16_kv_gib - report.fp16_kv_gib) < 1e-12
    assert est.kivi_gpus < est.fp16_gpus
    assert abs(est.kivi_usd - est.kivi_gpus * rate * hours) < 1e-9
    assert abs(est.fp16_usd - est.fp16_gpus * rate * hours) < 1e-9
    assert est.saved_usd() > 0.0
    assert K.estimate_pretrain(inputs, 0.0).kivi_usd == 0.0


def test_long_context_pretrain_needs_fewer_gpus_than_fp16():
    preset = K.ModelPreset.by_id("llama3-8b")
    budget = K.kv_budget_bytes(24.0, preset.weight_gib)
    for tokens in (32_768, 131_072):
        inputs = preset.to_inputs(K.KiviConfig.default(), tokens, 4, budget, 2.40)
        est = K.estimate_pretrain(inputs, 8.0)
        assert est.kivi_kv_gib < est.fp16_kv_gib
        assert est.kivi_gpus >= 1
        assert est.kivi_gpus < est.fp16_gpus
        assert est.kivi_usd < est.fp16_usd


def test_custom_shape_via_inputs():
    inputs = K.EconInputs("custom", 32, 8, 128, 16.0, K.KiviConfig.default(), 4096, 4,
                          K.kv_budget_bytes(48.0, 16.0), 2.0)
    report = K.compute_report(inputs)
    assert report.model_id == "custom"


def test_presets_and_sentinels():
    """econ.rs:107-115, 255-281: lookup by id, the zero-budget sentinel, the
    floored KV budget."""
    assert K.ModelPreset.by_id("LLAMA3_8B").id == "llama3-8b"
    assert K.ModelPreset.by_id("nope") is None
    assert len(K.ModelPreset.all()) == 6
    assert K.gpus_for_kv(0, 0) == 0
    assert K.gpus_for_kv(1, 0) == (1 << 64) - 1
    assert K.gpus_for_kv(10, 4) == 3
    assert K.kv_budget_bytes(8.0, 16.0) == 0
    assert K.kv_budget_bytes(24.0, 16.0) == 8 * 1024 ** 3
