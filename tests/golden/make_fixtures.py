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
* ``train_m3.json`` + ``train_m3_params.npz``: golden/train-spec-m3.json (the
  MLP 8 -> 16 -> 4 step's dims, synthetic training set, the 8 runs' optimizer,
  initial parameters and batch schedule) and golden/torch-train-m3.json's
  float64 PyTorch losses and parameters after every step; pinned by
  src/train/verify-cpu.js at metric v2 1e-8.  (The optdigits demo is left out:
  it needs a dataset.)
* ``m3b.json`` + ``m3b_blob.npz``: golden/spec-m3b.json (the transformer's
  config, parameter order, synthetic set, the 4 golden runs' seeds and
  schedules, the init and projection hashes) with golden/torch-m3b.json's
  losses and parameter projections, and from golden/torch-m3b.f64 the logits
  at initialisation of every golden run, the gradients at initialisation of
  golden-seed1 and its parameters after 20 steps; pinned by
  src/m3b/verify-cpu.js:11-12 at TAU1 = 1e-10 (init) and TAU2 = 1e-8 (training).
  (The text case is left out: it needs the book it was drawn from.)
"""
import json
import os
import sys

import numpy as np

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

    # the MLP training goldens (milestone 3)
    ts = load("train-spec-m3.json")
    tt = load("torch-train-m3.json")
    assert [c["name"] for c in tt["configs"]] == [c["name"] for c in ts["configs"]]
    json.dump({"source": "golden/train-spec-m3.json (dims, synthetic.train, configs) + golden/torch-train-m3.json losses",
               "torch": tt["torch"], "dtype": tt["dtype"], "dims": ts["dims"], "synthetic": {"train": ts["synthetic"]["train"]},
               "configs": ts["configs"], "losses": [c["losses"] for c in tt["configs"]]},
              open(os.path.join(HERE, "train_m3.json"), "w"), separators=(",", ":"))
    order = ("W1", "b1", "W2", "b2")
    params = {p: np.array([[step[p] for step in c["params"]] for c in tt["configs"]], dtype=np.float64) for p in order}
    np.savez_compressed(os.path.join(HERE, "train_m3_params.npz"), **params)

    # the transformer goldens (milestone 3b), synthetic runs only
    sp = load("spec-m3b.json")
    tb = load("torch-m3b.json")
    blob = np.fromfile(os.path.join(g, tb["blob"]["file"]), dtype="<f8")
    idx = tb["blob"]["index"]
    at = lambda key: blob[idx[key][0]:idx[key][0] + idx[key][1]]
    names = [p["name"] for p in sp["paramOrder"]]
    golden = sp["golden"]
    arrays = {}
    for gc in golden:
        arrays[f"init/{gc['name']}/logits"] = at(f"init/{gc['name']}/logits")
    g0 = golden[0]["name"]
    for n in names:
        arrays[f"init/{g0}/grad/{n}"] = at(f"init/{g0}/grad/{n}")
        arrays[f"train/{g0}/final/{n}"] = at(f"train/{g0}/final/{n}")
    np.savez_compressed(os.path.join(HERE, "m3b_blob.npz"), **arrays)
    init = [c for c in tb["init"] if c["name"] in {gc["name"] for gc in golden}]
    json.dump({"source": "golden/spec-m3b.json + golden/torch-m3b.json (+ arrays of golden/torch-m3b.f64 in m3b_blob.npz)",
               "torch": tb["torch"], "config": sp["config"], "optimizer": sp["optimizer"],
               "paramOrder": sp["paramOrder"], "synthetic": {k: sp["synthetic"][k] for k in ("seed", "vocab", "period", "train")},
               "golden": golden, "projections": sp["projections"],
               "init": init, "training": tb["training"]},
              open(os.path.join(HERE, "m3b.json"), "w"), separators=(",", ":"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_fixtures.py /path/to/reference")
    main(sys.argv[1])
