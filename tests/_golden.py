"""Helpers to load the committed golden fixtures (produced by tests/golden/make_golden.py from the
reference itself)."""
import hashlib
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SMALL_CASES = ["cfg1", "cfg1_spline", "cfg2", "cfg3_small", "cfg4_small", "cfg5_small"]
# cfg3 at full size (15,590 atoms), a 16,384-atom cfg4 box (the full 32,768-atom box does not fit the reference's
# evaluation on the host that made the fixtures) and a 37,044-atom cfg5 sub-box
FULL_CASES = ["cfg3", "cfg4_16k", "cfg5_37k"]
# physics terms: ZBL and dispersion (the latter needs the 10 A long-range list, rc_long below)
TERM_CASES = ["zbl_mol", "disp_mol", "disp_nacl"]
RC_LONG = 10.0
# the CP form and the non-factorised MomentBlock
FORM_CASES = ["cp_small", "cp_mol", "cp_spline", "moment_small", "moment_mol"]
MODEL_CASES = SMALL_CASES + FULL_CASES + TERM_CASES + FORM_CASES


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
    pos = np.ascontiguousarray(np.concatenate([s.positions for s in structs]), np.float64)
    if "pos" in d:
        assert np.array_equal(pos, d["pos"]), "structure generator drifted from the committed fixture"
    else:
        digest = hashlib.sha256(pos.tobytes()).hexdigest()
        assert digest == str(d["pos_sha256"]), "structure generator drifted from the committed fixture"
    pme = dict(m["pme"])
    if "mesh" in pme and pme["mesh"] is not None:
        pme["mesh"] = tuple(pme["mesh"])
    return structs, m["spec"], pme, d
