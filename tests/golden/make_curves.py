"""Copy the loss curves that the reference's own test suite recorded into a
small fixture.

Run in a container that has the reference checkout (it is not needed, and not
present, where the tests run):

    python tests/golden/make_curves.py /path/to/reference

The reference's tests galore/tests/test_galore_theorem_38.rs and
test_galore_scale_independence.rs train a toy transformer with the galore
crate's optimizer and write their per-step losses to
aethelStream/galore/pyref/galore_theorem_38_curves.json and
galore_scale_independence_curves.json.  This script keeps the first STEPS
losses of the four GaLore runs (and of the AdamW baseline, for reference) in
galore_curves.json; tests/test_oracle_reference_curves.py pins the oracle's
GaLore restatement against them.
"""
from __future__ import annotations

import json
import os
import sys

STEPS = 32


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETH_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_curves.py <reference checkout> (or set AETH_REFERENCE_ROOT)")
    pyref = os.path.join(root, "aethelStream", "galore", "pyref")
    out = {}
    for fname, prefix in (("galore_theorem_38_curves.json", "theorem_38"),
                          ("galore_scale_independence_curves.json", "scale_independence")):
        with open(os.path.join(pyref, fname)) as f:
            curves = json.load(f)
        for name, losses in curves.items():
            out[f"{prefix}/{name}"] = losses[:STEPS]
    out["_source"] = ("first %d losses of the curves in aethelStream/galore/pyref (written by the reference's "
                      "galore/tests/test_galore_theorem_38.rs and test_galore_scale_independence.rs)" % STEPS)
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "galore_curves.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=0)
    print(dst)


if __name__ == "__main__":
    main()
