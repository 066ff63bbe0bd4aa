"""Writes tests/golden/nerf_h_layout.json: struct sizes/offsets and enum values
of the reference's nerf.h (Xayah-Graphics/NeRF), measured by compiling a probe
against it.  Run where the reference checkout is available:
    python tests/golden/make_layout_golden.py /path/to/reference
"""
import json
import pathlib
import sys

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[1]))
from layout_probe import probe  # noqa: E402

if len(sys.argv) < 2:
    sys.exit("usage: make_layout_golden.py <reference checkout>")
ref = sys.argv[1]
out = pathlib.Path(__file__).with_name("nerf_h_layout.json")
out.write_text(json.dumps(probe(ref), indent=1, sort_keys=True) + "\n")
print(f"wrote {out}")
