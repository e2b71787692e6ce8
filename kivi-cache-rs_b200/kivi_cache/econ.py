"""Context economics (econ.rs): KV memory and rough cost estimates for agent
deployments, host arithmetic over the layer byte math (AgentMemoryBudget,
budget.rs:11-155), which equals a live cache's memory().compressed_bytes().

Names, fields, the preset table and every formula follow econ.rs so that a
caller of the reference finds the same numbers; Rust's usize::MAX sentinel is
2^64 - 1 here and f64 infinity stays float("inf").
"""
from __future__ import annotations

import math
from dataclasses import dataclass

_USIZE_MAX = (1 << 64) - 1
GIB = 1024.0 * 1024.0 * 1024.0  # econ.rs:315


def _bytes_to_gib(n):
    return n / GIB


@dataclass(frozen=True)
class ModelPreset:
    """econ.rs:7-18: KV geometry of a known model (weights in fp16 GiB)."""

    id: str
    display_name: str
    num_layers: int
    num_kv_heads: int
    head_dim: int
    weight_gib: float

    @staticmethod
    def all():
        return _PRESETS

    @staticmethod
    def by_id(id):
        """econ.rs:112-115: case-insensitive, '_' read as '-'."""
        key = id.lower().replace("_", "-")
        for p in _PRESETS:
            if p.id == key:
                return p
        return None

    def to_inputs(self, config, context_tokens, agents, kv_budget_bytes, usd_per_hour,
                  weight_gib=None):
        """econ.rs:117-138"""
        return EconInputs(self.id, self.num_layers, self.num_kv_heads, self.head_dim,
                          self.weight_gib if weight_gib is None else weight_gib, config,
                          context_tokens, agents, kv_budget_bytes, usd_per_hour)


# econ.rs:55-104 (the reference's preset table; callers look presets up by id)
_PRESETS = (
    ModelPreset("llama2-7b", "Llama-2-7B (MHA)", 32, 32, 128, 13.0),
    ModelPreset("llama2-13b", "Llama-2-13B (MHA)", 40, 40, 128, 24.0),
    ModelPreset("llama3-8b", "Llama-3-8B (GQA)", 32, 8, 128, 16.0),
    ModelPreset("mistral-7b", "Mistral-7B (GQA)", 32, 8, 128, 14.0),
    ModelPreset("falcon-7b", "Falcon-7B (MQA)", 32, 1, 64, 14.0),
    ModelPreset("longchat-7b-32k", "LongChat-7B-v1.5-32K", 32, 32, 128, 13.0),
)


@dataclass
class EconInputs:
    """econ.rs:20-34"""

    model_id: str
    num_layers: int
    num_kv_heads: int
    head_dim: int
    weight_gib: float
    config: object  # KiviConfig
    context_tokens: int
    agents: int
    kv_budget_bytes: int
    usd_per_hour: float

    def plan(self):
        """econ.rs:141-150"""
        from . import AgentMemoryBudget

        return AgentMemoryBudget.try_new(self.config, self.num_layers, self.num_kv_heads,
                                         self.head_dim)


@dataclass
class EconReport:
    """econ.rs:36-53"""

    model_id: str
    context_tokens: int
    agents: int
    bits: int
    kivi_kv_gib: float
    fp16_kv_gib: float
    kv_saved_gib: float
    compression_ratio: float
    max_agents_on_gpu: int
    max_agents_fp16_on_gpu: int
    fits_requested: bool
    usd_per_hour: float
    cost_per_agent_hour: float
    kv_savings_usd_per_hour: float


def _max_agents_fp16(plan, budget_bytes, tokens):
    """econ.rs:305-311"""
    per = plan.fp16_bytes_for_agents(1, tokens)
    return _USIZE_MAX if per == 0 else budget_bytes // per


def compute_report(inputs):
    """econ.rs:153-200"""
    plan = inputs.plan()
    agents, tokens = inputs.agents, inputs.context_tokens
    kivi_bytes = plan.bytes_for_agents(agents, tokens)
    fp16_bytes = plan.fp16_bytes_for_agents(agents, tokens)
    usd = inputs.usd_per_hour
    kv_share = kivi_bytes / fp16_bytes if fp16_bytes > 0 else 1.0
    return EconReport(
        model_id=inputs.model_id,
        context_tokens=tokens,
        agents=agents,
        bits=inputs.config.bits,
        kivi_kv_gib=_bytes_to_gib(kivi_bytes),
        fp16_kv_gib=_bytes_to_gib(fp16_bytes),
        kv_saved_gib=max(0, fp16_bytes - kivi_bytes) / GIB,
        compression_ratio=plan.compression_ratio_vs_fp16(agents, tokens),
        max_agents_on_gpu=plan.max_agents(inputs.kv_budget_bytes, tokens),
        max_agents_fp16_on_gpu=_max_agents_fp16(plan, inputs.kv_budget_bytes, tokens),
        fits_requested=plan.fits(inputs.kv_budget_bytes, agents, tokens),
        usd_per_hour=usd,
        cost_per_agent_hour=usd / agents if agents > 0 else 0.0,
        kv_savings_usd_per_hour=usd * (1.0 - kv_share),
    )


@dataclass
class PretrainEstimate:
    """econ.rs:202-223"""

    context_tokens: int
    batch: int
    hours: float
    usd_per_gpu_hour: float
    kivi_kv_gib: float
    fp16_kv_gib: float
    kivi_gpus: int
    fp16_gpus: int
    kivi_usd: float
    fp16_usd: float

    def saved_usd(self):
        """fp16_usd - kivi_usd, floored at zero."""
        return max(self.fp16_usd - self.kivi_usd, 0.0)


def gpus_for_kv(kv_bytes, kv_budget_bytes):
    """econ.rs:255-268: GPUs of kv_budget_bytes KV room that hold kv_bytes."""
    if kv_bytes == 0:
        return 0
    if kv_budget_bytes == 0:
        return _USIZE_MAX
    return (kv_bytes + kv_budget_bytes - 1) // kv_budget_bytes


def _job_usd(gpus, usd_per_gpu_hour, hours):
    """econ.rs:270-275"""
    if gpus == _USIZE_MAX:
        return math.inf
    return gpus * usd_per_gpu_hour * hours


def estimate_pretrain(inputs, hours):
    """econ.rs:225-253"""
    plan = inputs.plan()
    hours = max(hours, 0.0) if math.isfinite(hours) else 0.0
    rate = max(inputs.usd_per_hour, 0.0) if math.isfinite(inputs.usd_per_hour) else 0.0
    kivi_bytes = plan.bytes_for_agents(inputs.agents, inputs.context_tokens)
    fp16_bytes = plan.fp16_bytes_for_agents(inputs.agents, inputs.context_tokens)
    kivi_gpus = gpus_for_kv(kivi_bytes, inputs.kv_budget_bytes)
    fp16_gpus = gpus_for_kv(fp16_bytes, inputs.kv_budget_bytes)
    return PretrainEstimate(
        context_tokens=inputs.context_tokens,
        batch=inputs.agents,
        hours=hours,
        usd_per_gpu_hour=rate,
        kivi_kv_gib=_bytes_to_gib(kivi_bytes),
        fp16_kv_gib=_bytes_to_gib(fp16_bytes),
        kivi_gpus=kivi_gpus,
        fp16_gpus=fp16_gpus,
        kivi_usd=_job_usd(kivi_gpus, rate, hours),
        fp16_usd=_job_usd(fp16_gpus, rate, hours),
    )


def kv_budget_bytes(gpu_gib, weight_gib):
    """econ.rs:277-281: GPU memory minus weights (floored at zero), in bytes
    (float -> u64 cast: truncation, saturating)."""
    kv = max(gpu_gib - weight_gib, 0.0) * GIB
    if kv != kv:  # NaN casts to 0
        return 0
    return min(int(kv), _USIZE_MAX) if kv < math.inf else _USIZE_MAX


def parse_context_tokens(raw):
    """econ.rs:283-303: '128k', '200K', '1.5m' or plain counts; raises
    ValueError with the reference's message on bad input."""
    s = raw.strip().lower().replace("_", "")
    if not s:
        raise ValueError("context length must not be empty")
    if s.endswith("k"):
        num, suffix = s[:-1], 1_000
    elif s.endswith("m"):
        num, suffix = s[:-1], 1_000_000
    else:
        num, suffix = s, 1
    try:
        if num.strip() != num or not num:
            raise ValueError
        base = float(num)
    except ValueError:
        raise ValueError(f"invalid context token count: {raw}") from None
    if base < 0.0:
        raise ValueError(f"context must be non-negative: {raw}")
    value = base * suffix
    if value > float(_USIZE_MAX):
        raise ValueError(f"context too large: {raw}")
    if value != value:  # NaN casts to 0
        return 0
    return int(value)


__all__ = [
    "ModelPreset", "EconInputs", "EconReport", "PretrainEstimate", "compute_report",
    "estimate_pretrain", "gpus_for_kv", "kv_budget_bytes", "parse_context_tokens",
]
