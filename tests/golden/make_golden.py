"""Extract the reference's golden vectors for the quantized-projection path.

Run once in a checkout that has the reference tree (it is not needed, and
not present, on the GPU box):

    python tests/golden/make_golden.py /path/to/prism-inference

It reads the reference's own fixtures, captured from the pinned upstream C
ggml functions, and writes the records for the two weight formats this
library serves plus the Q8_K rounding control:

* ``tests/fixtures/upstream-tquants.json``  -> ``tq2_0.json``  (TypeId 35)
* ``tests/fixtures/upstream-kquants.json``  -> ``q2_k.json``   (TypeId 10)
* ``tests/fixtures/swift-q8k-parity.{json,bin}`` -> ``q8k_parity.json``

Field meaning (hex strings are little-endian byte dumps):
  OutputHex      packed weight blocks
  InputHex       the f32 row the weights were quantized from (optional)
  ActivationsHex Q8_K blocks, 292 B each (f32 scale, 256 x i8, 16 x i16)
  DecodedHex     the f32 row decoded from the packed blocks
  GenericDotHex  the f32 dot of the packed row and the activations, as the
                 upstream generic C kernel computes it (the reference's
                 tests/tquants.rs:15-77 and tests/kquants.rs:14-72 assert
                 exactly this value)
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
KEEP = ("Name", "TypeId", "Count", "OutputHex", "InputHex", "ActivationsHex",
        "DecodedHex", "GenericDotHex")


def _cases(path, type_id):
    with open(path) as f:
        fixture = json.load(f)
    out = []
    for case in fixture["Cases"]:
        if case["TypeId"] == type_id:
            out.append({k: case[k] for k in KEEP if k in case})
    return {
        "source": os.path.join("tests/fixtures", os.path.basename(path)),
        "upstream_commit": fixture.get("UpstreamCommit"),
        "generic_dot_reference": fixture.get("GenericDotReference"),
        "cases": out,
    }


def main(ref_root):
    fixtures = os.path.join(ref_root, "tests", "fixtures")
    tq = _cases(os.path.join(fixtures, "upstream-tquants.json"), 35)
    kq = _cases(os.path.join(fixtures, "upstream-kquants.json"), 10)
    with open(os.path.join(fixtures, "swift-q8k-parity.json")) as f:
        q8k_meta = json.load(f)
    with open(os.path.join(fixtures, "swift-q8k-parity.bin"), "rb") as f:
        q8k_bin = f.read()
    assert hashlib.sha256(q8k_bin).hexdigest() == q8k_meta["fixture_sha256"]
    q8k = {
        "source": "tests/fixtures/swift-q8k-parity.json + .bin",
        "layout": q8k_meta["layout"],
        "input_layout": q8k_meta["input_layout"],
        "cases": [
            {
                "input_bits": c["input_bits"],
                "inverse_scale_bits": c["inverse_scale_bits"],
                "native_code_at_1": c["native_code_at_1"],
                "source_code_at_1": c["source_code_at_1"],
                # the pinned (fused-rounding) block captured from the native DLL
                "native_block_hex": q8k_bin[i * 292:(i + 1) * 292].hex(),
            }
            for i, c in enumerate(q8k_meta["cases"])
        ],
    }
    for name, obj in (("tq2_0.json", tq), ("q2_k.json", kq), ("q8k_parity.json", q8k)):
        with open(os.path.join(HERE, name), "w") as f:
            json.dump(obj, f, indent=1)
            f.write("\n")
        print("wrote", name, len(obj["cases"]), "cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
