"""Regenerate the golden fixtures in this directory from the reference checkout.

half_vectors.json: the 138 f32 -> binary16 / bfloat16 roundings LYTH measured on a device
(reference: fixtures/half_vectors.json, written by tools/half_probe.py and checked by
crates/lyth/tests/half_rounding.rs). Only the vectors are kept, with their provenance.

Run in a checkout that has the reference at $LYTH_REFERENCE (default /root/reference); the
tests read only the committed JSON, never the reference.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> int:
    ref = os.environ.get("LYTH_REFERENCE", "/root/reference")
    src = os.path.join(ref, "fixtures", "half_vectors.json")
    with open(src) as f:
        data = json.load(f)
    out = {
        "source": "QuantumDrizzy/LYTH fixtures/half_vectors.json",
        "device": data.get("device"),
        "meaning": "f32 bit pattern -> the binary16 and bfloat16 bits a device produced with RNE",
        "vectors": [{"f32": v["f32"], "f16": v["f16"], "bf16": v["bf16"]} for v in data["vectors"]],
    }
    with open(os.path.join(HERE, "half_vectors.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"{len(out['vectors'])} vectors")
    return 0


if __name__ == "__main__":
    sys.exit(main())
