"""Regenerate the golden fixtures in this directory from a checkout of the reference.

Usage: python tests/golden/make_golden.py /path/to/LYTH   (or LYTH_REFERENCE=/path/to/LYTH)

* half_vectors.json: the 138 f32 -> binary16 / bfloat16 roundings LYTH measured on a device
  (reference: fixtures/half_vectors.json, written by tools/half_probe.py and checked by
  crates/lyth/tests/half_rounding.rs). Only the vectors are kept, with their provenance.
* ncu/*.csv: the reference's `ncu --csv` captures (fixtures/ncu), verbatim: dots group the
  digits (a Spanish-locale ncu), which is what the locale-safe parser is pinned on.
* machine/*.json: the reference's machine files and measurements (fixtures/machine): the honest
  sm_120 file with its measurement, a file that lies about its bandwidth, and one whose stored
  ridge is stale -- what machine-check must pass and refuse.

The tests read only the committed files, never the reference.
"""
import json
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
NCU = ["k_integrate-sm_120-2026-09-14.csv", "k_propagate-sm_120-2026-09-14.csv",
       "rmsnorm_fused_block-sm_120-2026-09-14.csv", "saxpy-lyth-sm_120-2026-09-14.csv"]
MACHINE = ["sm_120.json", "meas-sm_120-2026-09-14.json", "sm_120-lie.json", "sm_120-stale-ridge.json"]


def main(argv) -> int:
    ref = argv[1] if len(argv) > 1 else os.environ.get("LYTH_REFERENCE")
    if not ref:
        print(__doc__.strip().splitlines()[2], file=sys.stderr)
        return 2
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
    for sub, names in (("ncu", NCU), ("machine", MACHINE)):
        os.makedirs(os.path.join(HERE, sub), exist_ok=True)
        for n in names:
            shutil.copyfile(os.path.join(ref, "fixtures", sub, n), os.path.join(HERE, sub, n))
    print(f"{len(out['vectors'])} vectors, {len(NCU)} ncu captures, {len(MACHINE)} machine files")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
