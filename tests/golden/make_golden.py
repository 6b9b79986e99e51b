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

and the native captures that pin the reference's pinned (Swift) GDN,
attention and RoPE arithmetic, into ``pinned.json``:

* ``swift-gdn-parity.{json,bin}``   GDN dot and row-update cases
* ``swift-attention-dot.json``      attention dots and one weighted value
* ``swift-attention-softmax.json``  masked softmax rows
* ``swift-attention-rope.json`` + ``swift-rope-basis.json``
                                    out-of-place RoPE with native cos/sin
* ``swift-rope-inplace.{json,bin}`` in-place RoPE and one binary16 boundary

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
    more = {"tq1_0.json": _cases(os.path.join(fixtures, "upstream-tquants.json"), 34)}
    for type_id, name in ((11, "q3_k"), (12, "q4_k"), (13, "q5_k"), (14, "q6_k")):
        more[name + ".json"] = _cases(os.path.join(fixtures, "upstream-kquants.json"), type_id)
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
    pinned = pinned_fixtures(fixtures)
    ptq = ptq_fixture(fixtures)
    kvq = kvq_fixture(ref_root)
    for name, obj in (("tq2_0.json", tq), ("q2_k.json", kq), ("q8k_parity.json", q8k),
                      ("pinned.json", pinned), ("ptq_reference.json", ptq),
                      ("kvq_reference.json", kvq)) + tuple(more.items()):
        with open(os.path.join(HERE, name), "w") as f:
            json.dump(obj, f, indent=1)
            f.write("\n")
        print("wrote", name, len(obj.get("cases", obj)), "records")


def kvq_fixture(ref_root):
    """The rotated scalar KV codec's published constants and known answers:
    the binary32 level tables (src/kv_quant/tables.rs), the SplitMix64 words
    of seed 0 and the little-endian packing goldens (src/kv_quant/tests.rs
    splitmix_stream_matches_independent_known_words and
    packing_matches_fixed_little_endian_goldens), read from the source text."""
    import re
    import struct
    src = os.path.join(ref_root, "src", "kv_quant")
    with open(os.path.join(src, "tables.rs")) as f:
        tables = f.read()
    with open(os.path.join(src, "tests.rs")) as f:
        tests = f.read()

    def table(name):
        body = tables.split("const %s: [f32; 16] = [" % name)[1].split("];")[0]
        vals = [float(t.replace("_", "")) for t in re.findall(r"-?[0-9][0-9_.]*", body)]
        assert len(vals) == 16
        return [struct.unpack("<I", struct.pack("<f", v))[0] for v in vals]

    def words(fn):
        body = tests.split("fn %s()" % fn)[1].split("\n}\n")[0]
        return body

    sm = words("splitmix_stream_matches_independent_known_words")
    splitmix = [int(w.replace("_", ""), 16) for w in re.findall(r"0x([0-9a-f_]{16,})", sm)]
    pk = words("packing_matches_fixed_little_endian_goldens")
    packs = [[int(b, 16) for b in re.findall(r"0x([0-9a-f]{2})", arr)]
             for arr in re.findall(r"\[(0x[0-9a-f]{2}(?:, 0x[0-9a-f]{2})*)\]", pk)]
    assert len(splitmix) == 3 and [len(p) for p in packs] == [3, 8]
    return {
        "source": "src/kv_quant/tables.rs THREE and FOUR; src/kv_quant/tests.rs known words",
        "three_bits": table("THREE"),
        "four_bits": table("FOUR"),
        "splitmix_seed0": splitmix,
        "pack3": packs[0],
        "pack4": packs[1],
    }


def ptq_fixture(fx):
    """The native C++ PQ2/PTQ codec capture (tests/fixtures/ptq-reference.bin,
    layout in tools/ternary/tests/fixtures/README.md): binary16 conversions,
    then per case the same rows as PQ2 blocks and as PTQ blocks."""
    import struct
    with open(os.path.join(fx, "ptq-reference.bin"), "rb") as f:
        buf = f.read()
    assert hashlib.sha256(buf).hexdigest() == \
        "de86d0ff0e31037635ae5f607bcb68d4e62ee7cb5d1b5db5e739ef900114fd79"
    assert buf[:8] == b"PTPAR001"
    off = 8
    (nconv,) = struct.unpack_from("<I", buf, off)
    off += 4
    conversions = []
    for _ in range(nconv):
        h, bits = struct.unpack_from("<HI", buf, off)
        conversions.append([h, bits])
        off += 6
    (ncases,) = struct.unpack_from("<I", buf, off)
    off += 4
    cases = []
    for _ in range(ncases):
        rows, bpr = struct.unpack_from("<II", buf, off)
        off += 8
        n = rows * bpr
        pq2 = buf[off:off + 34 * n]
        off += 34 * n
        ptq = buf[off:off + 28 * n]
        off += 28 * n
        cases.append({"rows": rows, "blocks_per_row": bpr, "pq2_hex": pq2.hex(),
                      "ptq_hex": ptq.hex()})
    assert off == len(buf)
    return {"source": "tests/fixtures/ptq-reference.bin (native C++ PQ2/PTQ codec capture)",
            "half_conversions": conversions, "cases": cases}


def pinned_fixtures(fx):
    """The pinned-arithmetic captures, as plain u32 bit lists."""
    import struct

    def words(buf, off, n):
        return list(struct.unpack_from("<%dI" % n, buf, off)), off + 4 * n

    out = {"source": "reference tests/fixtures swift-* native captures (ggml-cpu sha256 "
                     "701b354a38b25e5c6dc57a1559f71cd26b2d0f8d69c1576a0e77a59a4273d2ab)"}
    # GDN: PGDN001\0, u32 dots, u32 rows; dot: width, native, x[w], y[w];
    # row: width, v, native out, q[w], k[w], state[w], native updated state[w]
    with open(os.path.join(fx, "swift-gdn-parity.bin"), "rb") as f:
        b = f.read()
    assert b[:8] == b"PGDN001\0"
    (nd, nr), off = words(b, 8, 2)
    dots, rows = [], []
    for _ in range(nd):
        (w, native), off = words(b, off, 2)
        x, off = words(b, off, w)
        y, off = words(b, off, w)
        dots.append({"native": native, "x": x, "y": y})
    for _ in range(nr):
        (w, v, native), off = words(b, off, 3)
        q, off = words(b, off, w)
        k, off = words(b, off, w)
        st, off = words(b, off, w)
        upd, off = words(b, off, w)
        rows.append({"v": v, "native_out": native, "q": q, "k": k, "state": st,
                     "native_state": upd})
    assert off == len(b)
    out["gdn"] = {"dots": dots, "rows": rows}
    with open(os.path.join(fx, "swift-attention-dot.json")) as f:
        d = json.load(f)
    out["attention_dot"] = {
        "cases": [{"name": c["name"], "first": c["first_bits"], "second": c["second_bits"],
                   "native": c["native_bits"]} for c in d["cases"]],
        "weighted_value": d["weighted_value"]}
    with open(os.path.join(fx, "swift-attention-softmax.json")) as f:
        d = json.load(f)
    out["softmax"] = [{"input": c["input_bits"], "native": c["native_bits"]} for c in d["cases"]]
    with open(os.path.join(fx, "swift-attention-rope.json")) as f:
        d = json.load(f)
    with open(os.path.join(fx, "swift-rope-basis.json")) as f:
        basis = json.load(f)
    rope = {"head": d["head"], "rotary": d["rotary_dimensions"], "input": d["input_bits"],
            "cases": []}
    for c, k in zip(d["cases"], basis["cases"]):
        assert c["position"] == k["position"]
        rope["cases"].append({"position": c["position"], "cos": k["cosine_bits"],
                              "sin": k["sine_bits"], "native_out_of_place": c["native_bits"]})
    with open(os.path.join(fx, "swift-rope-inplace.bin"), "rb") as f:
        b = f.read()
    assert b[:8] == b"SWROPIP1"
    (n,), off = words(b, 8, 1)
    for i in range(n):
        (pos,), off = words(b, off, 1)
        nat, off = words(b, off, 64)
        assert pos == rope["cases"][i]["position"]
        rope["cases"][i]["native_in_place_first64"] = nat
    bw, off = words(b, off, 11)
    assert off == len(b)
    rope["boundary"] = dict(zip(["position", "pair", "first", "second", "cos", "sin",
                                 "in_place_0", "in_place_1", "out_of_place_0",
                                 "out_of_place_1", "half_words"], bw))
    out["rope"] = rope
    return out


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
