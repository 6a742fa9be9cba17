"""Record the reference's calibration-hook values for every golden case.

Run in a container that holds the reference checkout, named by
FFTS_REFERENCE_ROOT:

    python tests/golden/make_collector_golden.py

For each case of make_golden.CASES it sets ``_sparsity_collector`` on the
reference module (as calibrate_from_qk does,
eval/efficiency/benchmark_attention_multilayer.py:179-262), runs the
reference's ``myattn_prefill`` on the CPU once per sequence (oracle/ref_import.py,
lowest-index tie-breaking) and stores the recorded "corr" and "final" kept
fractions (my_attn_v7.py:713-720) in collector.json.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

from make_golden import CASES, case_inputs  # noqa: E402


def main():
    from oracle.ref_import import load_reference, run_reference

    mod = load_reference()
    out = {}
    for name, spec in CASES.items():
        kw = dict(spec["kw"], block_size=spec.get("bs", 128))
        q, k, v = case_inputs(spec)
        mod._sparsity_collector = {"corr": [], "final": []}
        try:
            for b in range(q.shape[0]):
                run_reference(q[b:b + 1], k[b:b + 1], v[b:b + 1], stable_topk=True, **kw)
            out[name] = dict(mod._sparsity_collector)
        finally:
            del mod._sparsity_collector
        print(name, out[name], flush=True)
    with open(os.path.join(HERE, "collector.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
