"""Extracts the MDX23C golden forward into `mdx23c_tiny.json` (run in a checkout that has the
reference project; the committed output is what the tests read).

The source fixture, crates/ancha-models/tests/fixtures/mdx23c-tiny.json, holds a PyTorch (UVR
tfc_tdf_v3) forward of a two-scale, two-head TFC-TDF network on a synthetic spectrum. Its
weights and input are not stored: the reference test regenerates them from closed formulas
(tests/support/mdx23c.rs:27-78), restated in `oracle/mdx23c.py` (`fixture_weights`,
`fixture_input`). This script keeps the config, the tensor names and shapes, the shapes of
input and output, and the expected output, and records the source file's SHA-256.
"""
import hashlib
import json
import os
import sys

SRC = "crates/ancha-models/tests/fixtures/mdx23c-tiny.json"


def main(reference_root: str) -> None:
    path = os.path.join(reference_root, SRC)
    raw = open(path, "rb").read()
    d = json.loads(raw)
    out = {
        "source": SRC,
        "source_file_sha256": hashlib.sha256(raw).hexdigest(),
        "scope": d.get("scope"),
        "source_revision": d.get("source_revision"),
        "torch": d.get("torch"),
        "config": d["config"],
        "weights": [{"name": w["name"], "shape": w["shape"]} for w in d["weights"]],
        "input_shape": d["input_shape"],
        "output_shape": d["output_shape"],
        "expected": d["expected"],
    }
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mdx23c_tiny.json")
    with open(dst, "w") as f:
        json.dump(out, f, separators=(",", ":"))
    print(dst, len(out["expected"]), "values")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_mdx23c_tiny.py <reference project root>")
    main(sys.argv[1])
