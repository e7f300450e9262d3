"""Writes the golden fixtures under tests/golden/ from the reference's own records.

Run where the reference is mounted (``python tests/golden/make_fixtures.py
/path/to/reference``).  The fixtures are data the reference recorded, copied
unchanged in content:

* ``cases_torch.json``: golden/cases.json (112 graphs, inputs, cotangents) with
  golden/torch.json's float64 PyTorch answers (outputs + gradients) beside
  each case; pinned by test/golden.test.js:23-46 at metric v2 (1e-12) with
  random-9 the one recorded exception.
* ``cases_m3_torch.json``: golden/cases-m3.json + golden/torch-m3.json (the
  sqrt cases).
* ``pins.json``: golden/measurements.json's m4.fusion and m4.semantics.model
  structure counts, and golden/spec-m3b.json's first golden config.
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref):
    g = os.path.join(ref, "golden")
    load = lambda name: json.load(open(os.path.join(g, name)))
    cases = load("cases.json")["cases"]
    torch = load("torch.json")
    by = {c["name"]: c for c in torch["cases"]}
    out = {"source": "golden/cases.json + golden/torch.json", "torch": torch["torch"], "dtype": torch["dtype"],
           "cases": [dict(c, torch=by[c["name"]]) for c in cases]}
    json.dump(out, open(os.path.join(HERE, "cases_torch.json"), "w"), separators=(",", ":"))
    cm3 = load("cases-m3.json")
    tm3 = load("torch-m3.json")
    json.dump({"source": "golden/cases-m3.json + golden/torch-m3.json", "cases": cm3, "torch": tm3},
              open(os.path.join(HERE, "cases_m3_torch.json"), "w"), separators=(",", ":"))
    m = load("measurements.json")["m4"]
    spec = load("spec-m3b.json")
    g0 = spec["golden"][0]
    pins = {"source": "golden/measurements.json m4; golden/spec-m3b.json golden[0]",
            "fusion": m["fusion"], "semanticsModel": m["semantics"]["model"],
            "corpusByPattern": m["semantics"]["corpus"]["byPattern"],
            "corpus": {k: m["semantics"]["corpus"][k] for k in ("programs", "graphs", "withFused", "identical",
                                                                "compared", "fusedNodes", "byPattern")},
            "gpuFuzz": {k: m["gpu"]["fuzz"][k] for k in ("programs", "skipped", "runs", "fusedRuns", "unfusedPassed",
                                                         "fusedPassed", "bitwiseSame")}
            if "fuzz" in m.get("gpu", {}) else None,
            "goldenConfig": {k: g0[k] for k in ("name", "seed", "V", "batch")},
            "gpuLaunches": m["gpu"].get("teacherForced", {}).get("launches")}
    json.dump(pins, open(os.path.join(HERE, "pins.json"), "w"), indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
