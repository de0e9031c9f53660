"""Helpers to load the committed golden fixtures (produced by tests/golden/make_golden.py from the
reference itself)."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MODEL_CASES = ["cfg1", "cfg1_spline", "cfg2", "cfg3_small", "cfg4_small", "cfg5_small"]


def load(name):
    d = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    if "meta" in d:
        d["meta"] = json.loads(str(d["meta"]))
    return d


def case_inputs(name):
    """(structures, model spec, pme options, golden dict) for a model case."""
    from face_b200 import systems
    d = load(name)
    m = d["meta"]
    structs = systems.config_structures(m["cfg"], seed=m["seed"], scale=m["scale"])
    pos = np.concatenate([s.positions for s in structs])
    assert np.array_equal(pos, d["pos"]), "structure generator drifted from the committed fixture"
    pme = dict(m["pme"])
    if "mesh" in pme and pme["mesh"] is not None:
        pme["mesh"] = tuple(pme["mesh"])
    return structs, m["spec"], pme, d
