"""The RWKV-7 (config 5) float64 oracle pinned to the reference's own harness (CPU).

fhessm.rwkv7.step restates the x070 forward of results/vector-d-20261104/harness/rwkv7_model.py
(:329-392, the wkv recurrence :277-298) one token at a time.  tests/golden/rwkv7_small.npz holds
the harness's logits and last-block outputs for two 10-token sequences at a small shape (written
by tests/golden/make_rwkv7_golden.py from the harness itself, which computes in float32); the
recurrent step must reproduce them to float32 accuracy.  Where the reference is present the
comparison is also made live.  The polynomial sites of the circuit (Chebyshev series on fitted
intervals, Newton 1/sqrt from linear seeds) must track the exact sites."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_rwkv7_golden as gold  # noqa: E402

REF_ROOT = os.environ.get("FHESSM_REFERENCE", os.path.join(os.sep, "root", "reference"))
HARNESS = os.path.join(REF_ROOT, "results", "vector-d-20261104", "harness", "rwkv7_model.py")


def recurrent(sh, w, ids, sites=None):
    from fhessm.rwkv7 import new_state, step
    st = new_state(sh, ids.shape[0])
    lg, hid = [], []
    for t in range(ids.shape[1]):
        h = []
        lg.append(step(sh, w, ids[:, t], st, sites, hidden=h))
        hid.append(h[-1])
    return np.stack(lg, 1), np.stack(hid, 1)


def rel(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_recurrent_step_matches_harness_golden():
    g = np.load(os.path.join(ROOT, "tests", "golden", "rwkv7_small.npz"))
    sh, w, ids = gold.small_model()
    assert (ids == g["ids"]).all()
    lg, hid = recurrent(sh, w, ids)
    assert rel(lg, g["logits"]) < 2e-5      # the harness runs in float32
    assert rel(hid, g["hidden"]) < 2e-5
    assert (lg.argmax(-1) == g["logits"].argmax(-1)).mean() == 1.0


@pytest.mark.skipif(not os.path.exists(HARNESS), reason="the reference is not present on this machine")
def test_recurrent_step_matches_harness_live():
    ref_lg, ref_hid = gold.reference_logits(REF_ROOT)
    sh, w, ids = gold.small_model()
    lg, hid = recurrent(sh, w, ids)
    assert rel(lg, ref_lg) < 2e-5
    assert rel(hid, ref_hid) < 2e-5


def test_polynomial_sites_track_exact():
    from fhessm.rwkv7 import Sites, fit_sites
    sh, w, ids = gold.small_model()
    cal = [np.random.default_rng(11).integers(0, sh.vocab_size, 16) for _ in range(6)]
    fits = fit_sites(sh, w, cal, degree=23)
    assert all(len(f) == 3 for f in fits.values())
    lg_exact, _ = recurrent(sh, w, ids)
    lg_poly, _ = recurrent(sh, w, ids, Sites(fits))
    assert rel(lg_poly, lg_exact) < 1e-2
    assert (lg_poly.argmax(-1) == lg_exact.argmax(-1)).mean() >= 0.9
