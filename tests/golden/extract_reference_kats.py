"""Extract the reference's own known-answer vectors into a JSON fixture.

Reads the Rust test source of qx-consensus-math as TEXT (the Rust toolchain
is absent, so nothing is compiled or run) and writes
tests/golden/consensus_math_kats.json. The fixture travels with the repo;
this script is only re-run where the reference tree is present.

Sources (paths within blasrodri/qx):
  crates/qx-consensus-math/src/lib.rs:267-295  exp / rsqrt golden bits
  crates/qx-consensus-math/src/lib.rs:314-330  RoPE sin/cos golden bits
  crates/qx-consensus-math/src/lib.rs:28-61    inverse-frequency table
  crates/qx-consensus-math/src/lib.rs:217-311  error-bound limits
  crates/qx-runtime-v2/src/lib.rs:7203-7221    KV byte accounting
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference tree: the first argument, else $QX_REFERENCE
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("QX_REFERENCE", "")


def _hexes(text):
    return [int(h.replace("_", ""), 16) for h in re.findall(r"0x([0-9a-fA-F_]+)", text)]


def main():
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: extract_reference_kats.py <path of the blasrodri/qx tree> (or set QX_REFERENCE)")
    math_src = open(os.path.join(REF, "crates/qx-consensus-math/src/lib.rs")).read()
    lines = math_src.splitlines()

    def span(a, b):  # 1-based inclusive line span
        return "\n".join(lines[a - 1 : b])

    table = _hexes(span(28, 61))
    assert len(table) == 32, len(table)

    gold = span(267, 295)
    exp_cases = [float(x) for x in re.search(r"exp_cases = \[([^\]]*)\]", gold).group(1)
                 .replace("_f32", "").split(",")]
    exp_bits = _hexes(gold[gold.index("exp_bits"):gold.index("rsqrt_cases")])
    rsqrt_cases = [float(x) for x in re.search(r"rsqrt_cases = \[([^\]]*)\]", gold).group(1)
                   .replace("_f32", "").split(",")]
    rsqrt_bits = _hexes(gold[gold.index("rsqrt_bits"):])
    assert len(exp_bits) == len(exp_cases) == 7 and len(rsqrt_bits) == len(rsqrt_cases) == 5

    rope = span(314, 330)
    calls = re.findall(r"granite_rope_sin_cos\((\d+),\s*(\d+)\)", rope)
    bits = _hexes(rope)
    rope_cases = [
        {"position": int(p), "pair": int(q), "sine_bits": bits[2 * i], "cosine_bits": bits[2 * i + 1]}
        for i, (p, q) in enumerate(calls)
    ]
    assert len(rope_cases) == 4

    bounds = {
        "exp_worst_relative": float(re.search(r"worst_relative <= ([0-9.e-]+)", span(217, 236)).group(1)),
        "rsqrt_worst_relative": float(re.search(r"worst_relative <= ([0-9.e-]+)", span(239, 254)).group(1)),
        "rope_worst_absolute": float(re.search(r"worst <= ([0-9.e-]+)", span(298, 311)).group(1)),
    }

    v2 = open(os.path.join(REF, "crates/qx-runtime-v2/src/lib.rs")).read().splitlines()
    kv = "\n".join(v2[7202:7221])
    kv_bytes = {name: int(val.replace("_", "")) for name, val in
                re.findall(r"assert_eq!\((\w+)\.kv_bytes, ([0-9_]+)\)", kv)}

    out = {
        "source": "blasrodri/qx test literals, extracted as text by extract_reference_kats.py",
        "granite_inverse_frequency_bits": table,
        "exp": {"inputs": exp_cases, "bits": exp_bits},
        "rsqrt": {"inputs": rsqrt_cases, "bits": rsqrt_bits},
        "granite_rope_sin_cos": rope_cases,
        "error_bounds": bounds,
        "kv_bytes_context_512": kv_bytes,
    }
    path = os.path.join(HERE, "consensus_math_kats.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    sys.exit(main())
