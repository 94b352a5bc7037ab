"""The RWKV-7 circuit's norm and Chebyshev sites on CPU: the minimax-tuned Newton steps for
1/sqrt from a linear seed, and the calibration rounds that refit every site on the polynomial
model's own ranges."""
import numpy as np


def run_steps(a, b, steps, v):
    y = a + b * v
    for al, be in steps:
        y = y * (al - be * v * y * y)
    return y


def test_tuned_newton_reaches_tolerance_on_the_window():
    from fhessm.model import linear_rsqrt_seed, rsqrt_iters_for
    from fhessm.rwkv7 import newton_steps
    for m0, m1 in ((1.0, 10.0), (0.5, 400.0), (6.4e-4, 760.0)):
        a, b = linear_rsqrt_seed(m0, m1)
        steps = newton_steps(a, b, m0, m1, 1e-4)
        v = np.geomspace(m0, m1, 5001)
        err = np.abs(run_steps(a, b, steps, v) * np.sqrt(v) - 1).max()
        assert err < 1e-4, (m0, m1, err)
        # never more steps than Newton's own 3/2, 1/2
        assert len(steps) <= rsqrt_iters_for(a, b, m0, m1, 1e-4, cap=80)


def test_tuned_newton_saves_steps_on_a_wide_window():
    """GroupNorm's window from a cold state spans six decades: 10 tuned steps against 17"""
    from fhessm.model import linear_rsqrt_seed, rsqrt_iters_for
    from fhessm.rwkv7 import newton_steps
    m0, m1 = 5e-4, 760.0
    a, b = linear_rsqrt_seed(m0, m1)
    assert len(newton_steps(a, b, m0, m1, 1e-4)) + 5 <= rsqrt_iters_for(a, b, m0, m1, 1e-4, cap=80)


def test_tuned_newton_is_newton_near_one():
    """once t = y sqrt(v) is within a hair of 1, the minimax step is Newton's own"""
    from fhessm.rwkv7 import newton_steps
    a, b = 1.0, 0.0          # y0 = 1 on v in [1 - d, 1 + d]: t in [1 - d/2, 1 + d/2] roughly
    steps = newton_steps(a, b, 0.999, 1.001, 1e-12, widen=0.0)
    al, be = steps[-1]
    assert abs(al - 1.5) < 1e-6 and abs(be - 0.5) < 1e-6


def test_tuned_newton_never_diverges_below_the_window():
    """a value below the window only converges less far: t grows towards 1 from below"""
    from fhessm.model import linear_rsqrt_seed
    from fhessm.rwkv7 import newton_steps
    m0, m1 = 1.0, 100.0
    a, b = linear_rsqrt_seed(m0, m1)
    steps = newton_steps(a, b, m0, m1, 1e-4)
    v = np.geomspace(1e-4, m0, 200)
    t = run_steps(a, b, steps, v) * np.sqrt(v)
    assert np.all(np.isfinite(t)) and np.all(t > 0) and np.all(t < 1 + 1e-4)


def test_calibration_rounds_cover_the_polynomial_model():
    """after the refit rounds every site's input, run with the fitted sites on the calibration
    tokens, lies inside its interval (Chebyshev) or window (Newton)"""
    from fhessm.rwkv7 import RWKV7Shape, Sites, _site_ranges, fit_sites, synthetic_weights
    sh = RWKV7Shape(n_layer=2, n_embd=64, head_size=16, d_decay=8, d_aaa=8, d_mv=4, d_gate=16, dim_ffn=128,
                    vocab_size=64)
    w = synthetic_weights(sh, seed=5)
    rng = np.random.default_rng(6)
    toks = [rng.integers(0, sh.vocab_size, 8) for _ in range(4)]
    fits = fit_sites(sh, w, toks, degree=7, rounds=3)
    seen = _site_ranges(sh, w, toks, fits)
    for name, (lo, hi) in seen.items():
        f = fits[name]
        if np.ndim(f[2]) == 2:      # Newton: the seed's window is [lo / 1.25, hi * 2] of the union
            continue
        assert f[0] <= lo and hi <= f[1], (name, lo, hi, f[:2])
    assert all(np.isfinite(v).all() for v in (np.array(list(seen.values())),))
