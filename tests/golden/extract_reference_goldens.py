"""Extracts the literal known answers of the reference's codec tests
(bieli/kivi-cache-rs, tests/quant.rs) into quant_goldens.json beside this
script, by reading the Rust test source as text:

  pytorch_pack_matches_the_published_word_layout   (tests/quant.rs:13-41)
  four_bit_half_ties_round_to_even                 (tests/quant.rs:43-66)
  per_token_half_even_and_endpoints                (tests/quant.rs:68-77)
  per_channel_half_even_on_one_channel             (tests/quant.rs:79-97)
  negative_channel_endpoints_are_exact             (tests/quant.rs:99-117)

and pattern_token() (tests/quant.rs:3-11), which two of them use as input.

Usage: python tests/golden/extract_reference_goldens.py <reference checkout>
The tests read only the JSON this writes.
"""
import json
import os
import re
import sys


def functions(src):
    """name -> body text of every `fn name(...)` in src."""
    out = {}
    starts = [(m.group(1), m.start()) for m in re.finditer(r"\bfn\s+(\w+)\s*\(", src)]
    for i, (name, pos) in enumerate(starts):
        end = starts[i + 1][1] if i + 1 < len(starts) else len(src)
        out[name] = src[pos:end]
    return out


def num(text):
    return float(text.replace("_", ""))


def indexed_assigns(body, var):
    """var[i] = v; -> {i: v}"""
    return {int(i): num(v) for i, v in re.findall(var + r"\[(\d+)\]\s*=\s*(-?[\d._]+)\s*;", body)}


def indexed_asserts(body, var):
    """assert_eq!(var[i], v); -> {i: v}"""
    return {int(i): num(v) for i, v in
            re.findall(r"assert_eq!\(\s*" + var + r"\[(\d+)\]\s*,\s*(-?[\d._]+)\s*\)", body)}


def array_literal(body, name):
    m = re.search(r"let\s+" + name + r"\s*=\s*\[([^\]]*)\]", body)
    return [num(x) for x in m.group(1).replace("\n", " ").split(",") if x.strip()]


def main(ref):
    path = os.path.join(ref, "tests", "quant.rs")
    src = open(path).read()
    fns = functions(src)

    pat = fns["pattern_token"]
    fill = re.search(r"\[\s*(-?[\d.]+)\s*;\s*(\d+)\s*\]", pat)
    pattern = [num(fill.group(1))] * int(fill.group(2))
    for i, v in indexed_assigns(pat, "values").items():
        pattern[i] = v

    words = fns["pytorch_pack_matches_the_published_word_layout"]
    hexes = lambda var: {int(i): int(v.replace("_", ""), 16) for i, v in re.findall(
        r"assert_eq!\(\s*" + var + r"\[(\d+)\]\s*,\s*(0x[0-9A-Fa-f_]+)\s*\)", words)}
    dims = re.search(r"let dim = (\d+);", words).group(1), re.search(r"let seq = (\d+);", words).group(1)

    ties = fns["four_bit_half_ties_round_to_even"]
    tok = fns["per_token_half_even_and_endpoints"]
    chan = fns["per_channel_half_even_on_one_channel"]
    neg = fns["negative_channel_endpoints_are_exact"]
    neg_values = array_literal(neg, "values")

    out = {
        "source": "tests/quant.rs of bieli/kivi-cache-rs, read as text by extract_reference_goldens.py",
        "pattern_token": pattern,
        "pytorch_words": {
            "dim": int(dims[0]), "seq": int(dims[1]),
            "data": "(t + d) % 4 at [t][d]",
            "key_codes": hexes("key_codes"), "value_codes": hexes("value_codes"),
        },
        "four_bit_half_ties": {
            "len": 16, "bits": 4, "group": 16,
            "input": indexed_assigns(ties, "data"), "expect": indexed_asserts(ties, "out"),
        },
        "per_token_half_even": {"bits": 2, "group": 16, "expect": array_literal(tok, "expect")},
        "per_channel_half_even": {"bits": 2, "group": 16, "expect_ch0": array_literal(chan, "expect_ch0")},
        "negative_channel_endpoints": {
            "bits": 2, "group": 16, "values": neg_values, "expect": indexed_asserts(neg, "out"),
        },
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_goldens.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
