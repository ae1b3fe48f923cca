"""Writes ici_model.json: outputs of the reference's analytical interconnect
model (src/orthocache/ici_bandwidth_model.py, pure Python + numpy) for a few
configurations, to pin orthocache_b200.nvlink_model's restatement.  Run in a
container that has the reference checkout:

    python tests/golden/make_ici_golden.py /path/to/orthocache
"""
import importlib.util
import json
import os
import sys

ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ORTHOCACHE_REFERENCE", ".")
spec = importlib.util.spec_from_file_location("ici", os.path.join(ref, "src/orthocache/ici_bandwidth_model.py"))
R = importlib.util.module_from_spec(spec)
spec.loader.exec_module(R)
CASES = [(80, 131072, 128, 8, 8, 0.75), (50, 65536, 256, 4, 8, 0.688), (1, 512, 64, 1, 1, 0.0),
         (126, 1000003, 128, 8, 16, 0.9), (60, 131072, 256, 16, 8, 1.0)]
out = {"per_step": [[list(c), R.ici_bytes_per_step(*c)] for c in CASES],
       "table": [[[80, 131072, 128, 8, 8], R.ici_bandwidth_table(80, 131072, 128, 8, 8)],
                 [[60, 131072, 256, 16, 8], R.ici_bandwidth_table(60, 131072, 256, 16, 8, 2, [0.0, 0.25, 0.75])]]}
with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "ici_model.json"), "w") as f:
    json.dump(out, f, indent=1)
