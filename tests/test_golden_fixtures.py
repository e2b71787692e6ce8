"""The reference's literal codec known answers (tests/quant.rs, extracted as
text into tests/golden/quant_goldens.json by tests/golden/extract_reference_goldens.py)
against the C oracle on the CPU and the device codec on the GPU.
"""
import json
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "quant_goldens.json")))


def cases():
    """(name, per_channel, data, tokens, dim, bits, group, check(dequantized, words))"""
    out = []
    w = GOLDEN["pytorch_words"]
    seq, dim = w["seq"], w["dim"]
    data = np.array([(t + d) % 4 for t in range(seq) for d in range(dim)], np.float32)
    for per_channel, key in ((True, "key_codes"), (False, "value_codes")):
        want = {int(i): v for i, v in w[key].items()}

        def check(deq, words, data=data, want=want):
            assert all(int(words[i]) == v for i, v in want.items()), (words[:4], want)
            assert (deq == data).all()

        out.append(("pytorch_words_" + key, per_channel, data, seq, dim, 2, 32, check))

    t = GOLDEN["four_bit_half_ties"]
    data = np.zeros(t["len"], np.float32)
    for i, v in t["input"].items():
        data[int(i)] = v
    exp = {int(i): v for i, v in t["expect"].items()}
    out.append(("four_bit_half_ties", False, data, 1, t["len"], t["bits"], t["group"],
                lambda deq, words, exp=exp: [deq[i] for i in exp] == list(exp.values())))

    pattern = np.array(GOLDEN["pattern_token"], np.float32)
    p = GOLDEN["per_token_half_even"]
    out.append(("per_token_half_even", False, pattern, 1, 16, p["bits"], p["group"],
                lambda deq, words, e=p["expect"]: list(deq) == e))

    c = GOLDEN["per_channel_half_even"]
    data = np.zeros(16 * 16, np.float32)
    data[::16] = pattern
    out.append(("per_channel_half_even", True, data, 16, 16, c["bits"], c["group"],
                lambda deq, words, e=c["expect_ch0"]: list(deq[::16]) == e and
                (deq.reshape(16, 16)[:, 1:] == 0).all()))

    n = GOLDEN["negative_channel_endpoints"]
    data = np.zeros(16 * 16, np.float32)
    data[:16 * len(n["values"]):16] = n["values"]
    exp = {int(i): v for i, v in n["expect"].items()}
    out.append(("negative_channel_endpoints", True, data, 16, 16, n["bits"], n["group"],
                lambda deq, words, exp=exp: [deq[i] for i in exp] == list(exp.values())
                and (deq[16 * len(n["values"])::16] == 0).all()))
    return out


CASES = cases()


def _verdict(ok):
    # checks either assert inside (None) or return their verdict
    assert ok is None or bool(ok)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_goldens(case):
    name, per_channel, data, tokens, dim, bits, group, check = case
    codes, params = O.quantize(per_channel, data, 1, 1, tokens, dim, bits, group)
    deq = O.dequantize_packed(per_channel, codes, params, 1, 1, tokens, dim, bits, group)
    words = O.pytorch_codes(per_channel, codes, 1, 1, tokens, dim, bits, group)
    _verdict(check(deq, words))


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_device_codec_matches_reference_goldens(case):
    import kivi_cache as K

    name, per_channel, data, tokens, dim, bits, group, check = case
    q = (K.quantize_per_channel if per_channel else K.quantize_per_token)(
        data, 1, 1, tokens, dim, bits, group)
    _verdict(check(q.dequantize(), q.pytorch_codes()))
