"""The oracle restatement against fixtures produced by the reference itself
(its own model sources compiled for CPU/FP32, see tests/golden/make_golden.py)."""
import json
import os

import numpy as np
import pytest

from yalama_b200 import synth
from oracle.model import OracleModel, OK, KV_CACHE_EXCEEDED
from oracle import sampler

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# the model fixtures of make_golden.py (the sampler fixture has its own test)
CASES = sorted(f[:-4] for f in os.listdir(GOLDEN)
               if f.endswith(".npz") and "spec" in np.load(os.path.join(GOLDEN, f)).files)


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    kw = json.loads(str(z["spec"]))
    flags = json.loads(str(z["flags"]))
    return z, synth.tiny_spec(**kw), flags


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    z, spec, flags = load(name)
    kv = "--nokv" not in flags
    kvgb = int(flags[flags.index("--kvgb") + 1]) if "--kvgb" in flags else 1
    m = OracleModel(spec, synth.model_weights(spec, 0), mode="f32", kv_gb=kvgb, kv_enabled=kv)
    m.begin_infer()
    ids = list(z["prompt"])
    ref_logits, ref_ids = z["logits"], z["ids"]
    for step in range(len(ref_ids)):
        st, lg = m.infer(ids)
        assert st == OK
        # FP32 on both sides; only summation order differs
        np.testing.assert_allclose(lg, ref_logits[step], rtol=0, atol=2e-5)
        assert sampler.greedy(lg) == ref_ids[step]
        nxt = int(ref_ids[step])
        ids = [nxt] if kv else list(m.ids) + [nxt]
    if int(z["error"]) != 0:
        st, _ = m.infer(ids)
        assert st == int(z["error"]) == KV_CACHE_EXCEEDED
