"""C-ABI checks that need no GPU: the library loads, exports every symbol
declared in include/kivi_gpu.h, and its host-only logic (config validation,
error payloads, budget byte math, PyTorch word layout) matches the oracle."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as O
from helpers import golden_tensor

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kivi_gpu.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kivi_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import kivi_cache as K

    lib = K.lib()
    names = declared_functions()
    assert len(names) >= 40
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", K.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (kivi_[a-z0-9_]+)$", out, flags=re.M))
    assert set(names) <= exported, set(names) - exported


def test_config_errors_match_reference():
    """config.rs:31-55, tests/cache.rs:147-158"""
    import kivi_cache as K

    assert K.KiviConfig.default() == K.KiviConfig(2, 32, 128)
    for args, variant, a, b in [((3, 32, 128), "InvalidBits", 3, 0),
                                ((2, 8, 32), "MisalignedGroup", 8, 2),
                                ((2, 32, 100), "ResidualLength", 100, 32),
                                ((4, 0, 32), "MisalignedGroup", 0, 4)]:
        with pytest.raises(K.KiviError) as e:
            K.KiviConfig.try_new(*args)
        assert (e.value.variant, e.value.a, e.value.b) == (variant, a, b)
        with pytest.raises(O.OracleError) as eo:
            O.KiviConfig.try_new(*args)
        assert eo.value.variant == variant
    assert "must be a positive multiple of group_size 32" in str(
        pytest.raises(K.KiviError, K.KiviConfig.try_new, 2, 32, 100).value)


def test_cache_new_validation_runs_before_any_device_work():
    """cache.rs:93-104: errors come from argument checks alone."""
    import kivi_cache as K

    cfg = K.KiviConfig()
    for args, variant in [((0, 1, 128), "ZeroDimension"), ((1, 0, 128), "ZeroDimension"),
                          ((1, 1, 40), "HeadDim"), ((1, 1, 0), "HeadDim")]:
        with pytest.raises(K.KiviError) as e:
            K.KiviCache(cfg, *args)
        assert e.value.variant == variant
    with pytest.raises(K.KiviError) as e:
        K.KiviCache(cfg, 0, 1, 128)
    assert e.value.name == "batch"
    with pytest.raises(K.KiviError) as e:
        K.KiviCache(cfg, 1, 0, 128)
    assert e.value.name == "num_kv_heads"


def test_quantize_argument_errors_match_reference():
    """tests/quant.rs:213-228 through the C ABI (checked before any device work)."""
    import kivi_cache as K

    data = np.zeros(8, np.float32)
    with pytest.raises(K.KiviError) as e:
        K.quantize_per_channel(data, 1, 1, 8, 1, 3, 32)
    assert e.value.variant == "InvalidBits" and e.value.a == 3
    with pytest.raises(K.KiviError) as e:
        K.quantize_per_channel(data, 1, 1, 7, 1, 2, 32)
    assert e.value.variant == "TokenGroup"
    with pytest.raises(K.KiviError) as e:
        K.quantize_per_token(data, 1, 1, 4, 2, 2, 32)
    assert e.value.variant == "HeadDim"


@pytest.mark.parametrize("bits,group,residual", [(2, 32, 128), (4, 32, 128), (2, 16, 32),
                                                 (8, 32, 64), (4, 8, 16)])
def test_budget_byte_math_matches_oracle(bits, group, residual):
    """budget.rs:316-364 == memory().compressed_bytes() (tests/budget.rs:68-91)"""
    import kivi_cache as K

    cfg = K.KiviConfig(bits, group, residual)
    ocfg = O.KiviConfig(bits, group, residual)
    for heads, dim in [(8, 128), (2, 64), (1, 32)]:
        if dim % group:
            continue
        for tokens in [0, 1, group, residual - 1, residual, residual + 1, 5 * residual + 7, 200_000]:
            assert K.layer_kv_bytes(cfg, heads, dim, tokens) == O.layer_kv_bytes(ocfg, heads, dim, tokens)
        assert K.marginal_bytes_per_layer(cfg, heads, dim) == O.marginal_bytes_per_layer(ocfg, heads, dim)
    assert K.marginal_bytes_per_layer(K.KiviConfig(), 8, 128) == 1024  # the reference README.md:176


def test_agent_budget_planner_matches_readme():
    """the reference README.md:176-186 figures, tests/budget.rs:47-66"""
    import kivi_cache as K

    plan = K.AgentMemoryBudget.try_new(K.KiviConfig(), 32, 8, 128)
    per_agent = plan.bytes_for_context(200_000)
    assert round(per_agent / 2**20) == 6271
    assert abs(plan.bytes_for_agents(8, 200_000) / 2**30 - 48.99) < 0.01
    assert abs(plan.fp16_bytes_for_agents(8, 200_000) / 2**30 - 195.31) < 0.01
    assert plan.max_agents(24 * 2**30, 200_000) == 3


def test_pytorch_codes_host_transform_matches_oracle():
    """quant.rs:71-112 word permutation (host code of the C ABI)."""
    import kivi_cache as K

    data = golden_tensor(64, 32)
    for axis in (0, 1):
        codes, params = O.quantize(axis == 0, data, 1, 1, 64, 32, 2, 32)
        out = np.zeros(codes.size, np.uint32)
        err = K._Err()
        rc = K.lib().kivi_pytorch_codes(axis, codes.ctypes.data_as(C.POINTER(C.c_uint32)),
                                        codes.size, 1, 1, 64, 32, 2, 32,
                                        out.ctypes.data_as(C.POINTER(C.c_uint32)), out.size,
                                        C.byref(err))
        assert rc == 0
        assert (out == O.pytorch_codes(axis == 0, codes, 1, 1, 64, 32, 2, 32)).all()


def test_product_path_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "kivi-cache-rs_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".hpp", ".cpp")):
                text = open(os.path.join(dirpath, f), errors="replace").read()
                assert "import oracle" not in text and "kivi_oracle" not in text, f
