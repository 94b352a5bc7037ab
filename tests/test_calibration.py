"""Newton-seed calibration (CPU): the per-site windows, the bootstrap gains and the seeded
float64 model on conversations outside the calibration set.

calibrate_seeds fits a linear 1/sqrt seed per norm site and picks the Newton iteration count
that reaches the tolerance over the window (the reference's fhe_circuit_sim.py:125-160 recipe,
window [0.8 m, 1.25 M]).  A conversation whose mean square leaves the window is not refreshed
by the Newton steps; these tests pin the window arithmetic and that a wider upper margin keeps
held-out conversations on the exact model."""
import os
import sys

import numpy as np

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import make_fwd_np_golden as gold  # noqa: E402


def _newton(a, b, x, n):
    y = a + b * x
    for _ in range(n):
        y = 1.5 * y - 0.5 * x * y ** 3
    return y


def _capture(cfg, w, lanes, steps, seed):
    from fhessm.model import plain_step
    rng = np.random.default_rng(seed)
    cap, state = {}, None
    for _ in range(steps):
        _, state = plain_step(cfg, w, w["emb"][rng.integers(0, cfg.vocab, lanes)], state, None, cap)
    return cap


def test_window_reaches_tolerance_over_asymmetric_margin():
    from fhessm.model import calibrate_seeds
    cfg, w, _ = gold.small_weights()
    tol = 1e-4
    seeds = calibrate_seeds(cfg, w, steps=3, lanes=32, tol=tol, ms_margin=(1.25, 4.0))
    cap = _capture(cfg, w, 32, 3, 7)
    sites = [t for t in cap if not t.startswith("peak:")]
    assert sites
    for tag in sites:
        arr = np.array(cap[tag])
        m, M = arr[:, 0].min(), arr[:, 1].max()
        a, b, n = seeds[tag]
        x = np.geomspace(m / 1.25, 4.0 * M, 400)
        err = np.abs(_newton(a, b, x, n) * np.sqrt(x) - 1.0)
        assert err.max() <= tol, tag
        assert a + b * (4.0 * M) > 0.0   # the seed stays in the Newton basin at the top


def test_gains_do_not_depend_on_newton_window():
    from fhessm.model import calibrate_seeds
    cfg, w, _ = gold.small_weights()
    s0 = calibrate_seeds(cfg, w, steps=2, lanes=32)
    s1 = calibrate_seeds(cfg, w, steps=2, lanes=32, ms_margin=(1.25, 4.0))
    gains = [k for k in s0 if k.startswith("gain:")]
    assert gains
    for k in gains:
        assert s0[k] == s1[k], k
    # the asymmetric window is wider above, so it never needs fewer iterations
    for k in s0:
        if not k.startswith("gain:"):
            assert s1[k][2] >= s0[k][2] - 1, k


def test_seeded_model_tracks_exact_model_on_held_out_conversations():
    from fhessm.model import calibrate_seeds, plain_step, rel_err_rms
    cfg, w, _ = gold.small_weights()
    seeds = calibrate_seeds(cfg, w, steps=3, lanes=64, ms_margin=(1.25, 4.0))
    E = w["emb"]
    for tok_seed in (100, 101, 102):
        rng = np.random.default_rng(tok_seed)
        s_exact = s_newton = None
        for _ in range(6):
            x = E[rng.integers(0, cfg.vocab, 64)]
            ya, s_exact = plain_step(cfg, w, x, s_exact)
            yb, s_newton = plain_step(cfg, w, x, s_newton, seeds)
            la, lb = ya @ E.T, yb @ E.T
            assert rel_err_rms(lb, la) < 1e-4
            assert np.mean(la.argmax(-1) == lb.argmax(-1)) >= 0.98
