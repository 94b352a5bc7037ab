"""The float64 model oracle pinned to the reference's own forward (CPU).

fhessm.model.plain_step restates the reference's _fwd_np (ml-eval/train_fhe_native_ssm.py:
829-890) in recurrent form: one token per call, with the scan state s and the shift-mix input
carried.  tests/golden/fwd_np_small.npz holds _fwd_np's logits for a 12-token sequence at a
small shape (written by tests/golden/make_fwd_np_golden.py from the reference itself); running
plain_step token by token on the same weights must give the same logits to 1e-10 relative.
Where the reference is importable, the comparison is also made live against _fwd_np itself."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_fwd_np_golden as gold  # noqa: E402

REF_ROOT = os.environ.get("FHESSM_REFERENCE", os.path.join(os.sep, "root", "reference"))


def recurrent_logits(cfg, w, ids):
    from fhessm.model import plain_step
    state, out = None, []
    for t in ids:
        y, state = plain_step(cfg, w, w["emb"][[t]], state)
        out.append((y @ w["emb"].T)[0])
    return np.array(out)


def rel(a, b):
    return float(np.sqrt(np.mean((a - b) ** 2)) / np.sqrt(np.mean(b ** 2)))


def test_plain_step_matches_reference_fwd_np_golden():
    g = np.load(os.path.join(ROOT, "tests", "golden", "fwd_np_small.npz"))
    cfg, w, ids = gold.small_weights()
    assert (ids == g["ids"]).all()
    got = recurrent_logits(cfg, w, ids)
    assert got.shape == g["logits"].shape
    assert rel(got, g["logits"]) < 1e-10
    assert np.abs(got - g["logits"]).max() < 1e-10 * np.abs(g["logits"]).max()
    assert (got.argmax(-1) == g["logits"].argmax(-1)).all()


@pytest.mark.skipif(not os.path.exists(os.path.join(REF_ROOT, "ml-eval", "train_fhe_native_ssm.py")),
                    reason="the reference is not present on this machine")
def test_plain_step_matches_reference_fwd_np_live():
    ids, ref = gold.reference_logits(REF_ROOT)
    cfg, w, _ = gold.small_weights()
    assert rel(recurrent_logits(cfg, w, ids), ref) < 1e-10
