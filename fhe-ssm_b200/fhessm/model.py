"""fhessm.model -- the polynomial SSM language model on the encrypted engine.

Client/model-preparation side of the hot path:
  * ``ModelConfig`` and ``synthetic_weights``: the architecture of
    ml-eval/train_fhe_native_ssm.py (build_model :149-362) with seeded random weights
    (the trained bundle is not shipped with the reference; the benchmark uses synthetic
    weights of the same shapes);
  * ``plain_step``: the float64 recurrent step (one token per conversation) with the exact
    semantics of ``_fwd_np`` (train_fhe_native_ssm.py:829-890) written in recurrent form, with
    either the exact 1/sqrt or the circuit's seeded Newton rsqrt;
  * ``calibrate_seeds``: per-site linear Newton seeds fitted on the calibration ranges, as
    ``cmd_export`` does (train_fhe_native_ssm.py:1068-1089, fhe_circuit_sim.py:125-160);
  * ``pack_lanes`` / ``unpack_lanes``: the block layout with complex packing;
  * ``EncryptedModel``: uploads the weights to the engine (C-ABI fhe_model_*) and runs the
    encrypted step.
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import FheError, Ciphertext, _check, _VP, _DP, lib


@dataclass
class ModelConfig:
    d: int = 1024
    dff: int = 4096
    n_layer: int = 24
    vocab: int = 50304
    D: int = 1024          # block width (d padded to a power of two)
    b1: int = 32           # BSGS baby steps
    a_min: float = 0.90
    a_max: float = 0.9995
    alpha: float = 1.0
    eps: float = 1e-5
    shift_mix: bool = True


CONFIG_405M = ModelConfig(b1=64)   # double-hoisted BSGS: 127 babies, 30 giants per 1024x1024 block


def synthetic_weights(cfg: ModelConfig, seed: int = 1234):
    """Seeded random weights of the model's shapes: matrices N(0, 0.02); polynomial
    coefficients U[-1, 1]; decays in [a_min, a_max]; norm gains 1; mix U[0, 1]; readout
    c, dd U[-1, 1]; tied embedding N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    d, dff = cfg.d, cfg.dff
    w = {"emb": rng.normal(0, 0.02, (cfg.vocab, d)), "g_out": np.ones(d), "layers": []}
    for _ in range(cfg.n_layer):
        a = rng.uniform(cfg.a_min, cfg.a_max, d)
        L = {
            "win": rng.normal(0, 0.02, (d, d)), "wout": rng.normal(0, 0.02, (d, d)),
            "wk": rng.normal(0, 0.02, (dff, d)), "wr": rng.normal(0, 0.02, (dff, d)),
            "wv": rng.normal(0, 0.02, (d, dff)),
            "decay": a, "b": 1.0 - a, "g1": np.ones(d), "mix": rng.uniform(0, 1, d),
            "c": rng.uniform(-1, 1, d), "dd": rng.uniform(-1, 1, d),
            "p0": rng.uniform(-1, 1, d), "p1": rng.uniform(-1, 1, d), "p2": rng.uniform(-1, 1, d),
            "g2": np.ones(d),
        }
        for i in range(4):
            L[f"q{i}"] = rng.uniform(-1, 1, dff)
        for i in range(3):
            L[f"r{i}"] = rng.uniform(-1, 1, dff)
        w["layers"].append(L)
    return w


# ------------------------------------------------------------------------ plaintext ----
def _peak(cap, tag, v):
    if cap is not None:
        cap.setdefault("peak:" + tag, []).append(float(np.max(np.abs(v))))


def _rms(x, g, eps, seed=None, cap=None, tag=None):
    ms = (x * x).mean(-1, keepdims=True) + eps
    if cap is not None:
        cap.setdefault(tag, []).append([float(ms.min()), float(ms.max())])
        _peak(cap, tag + ".x", x)
    if seed is None:
        return x / np.sqrt(ms) * g
    a, b, iters = seed
    y = a + b * ms
    for _ in range(int(iters)):
        y = 1.5 * y - 0.5 * ms * y * y * y
    return x * y * g


def plain_step(cfg: ModelConfig, w, h, state, seeds=None, cap=None, hidden=False):
    """One recurrent step for a batch of lanes: h (lanes, d) embedded tokens; state is a
    list per layer of (s_prev, u_prev) or None (cold start).  Returns (y, new_state) with
    y = rmsnorm(h_final, g_out) (hidden=True: h_final itself, before the output norm).
    seeds: None = exact 1/sqrt (the _fwd_np reference), else the circuit's Newton rsqrt with
    the per-site seeds."""
    new_state = []
    H = h.astype(np.float64)
    for i, L in enumerate(w["layers"]):
        sd = seeds[f"L{i}.tm"] if seeds else None
        u = _rms(H, L["g1"], cfg.eps, sd, cap, f"L{i}.tm")
        sp, up = state[i] if state else (None, None)
        un = u
        if cfg.shift_mix:
            us = up if up is not None else np.zeros_like(u)
            u = u * L["mix"] + us * (1.0 - L["mix"])
        _peak(cap, f"L{i}.u", u)
        x = u @ L["win"].T
        s = L["b"] * x + (L["decay"] * sp if sp is not None else 0.0)
        _peak(cap, f"L{i}.s", s)
        z = L["c"] * s + L["dd"] * x
        _peak(cap, f"L{i}.z", z)
        g = z * (L["p0"] + L["p1"] * z + L["p2"] * z * z)
        _peak(cap, f"L{i}.g", g)
        H = H + cfg.alpha * (g @ L["wout"].T)
        sd = seeds[f"L{i}.cm"] if seeds else None
        u2 = _rms(H, L["g2"], cfg.eps, sd, cap, f"L{i}.cm")
        _peak(cap, f"L{i}.v", u2)
        k = u2 @ L["wk"].T
        r = u2 @ L["wr"].T
        act = L["q0"] + L["q1"] * k + L["q2"] * k * k + L["q3"] * k * k * k
        gate = L["r0"] + L["r1"] * r + L["r2"] * r * r
        _peak(cap, f"L{i}.f", act * gate)
        H = H + (act * gate) @ L["wv"].T
        new_state.append((s, un))
    if hidden:
        return H, new_state
    sd = seeds["ln_out"] if seeds else None
    return _rms(H, w["g_out"], cfg.eps, sd, cap, "ln_out"), new_state


def linear_rsqrt_seed(m, M):
    """Linear seed y0 = a + b v for 1/sqrt(v) on [m, M], relative least squares on a log grid
    (fhe_circuit_sim.py:125-136)."""
    grid = np.geomspace(m, M, 64)
    tgt = 1.0 / np.sqrt(grid)
    A = np.stack([np.ones_like(grid), grid], axis=1) / tgt[:, None]
    sol, *_ = np.linalg.lstsq(A, np.ones_like(grid), rcond=None)
    return float(sol[0]), float(sol[1])


def rsqrt_iters_for(a, b, lo, hi, tol=1e-4, cap=14):
    """Newton iterations for relative error <= tol over [lo, hi] (fhe_circuit_sim.py:138-160
    checks [0.8 m, 1.25 M]); raises when the seed leaves the convergence basin."""
    grid = np.geomspace(lo, hi, 256)
    y = a + b * grid
    if np.any(grid * y * y >= 3.0) or np.any(y <= 0.0):
        raise ValueError("linear seed outside the Newton basin")
    for n in range(cap + 1):
        if np.max(np.abs(y * np.sqrt(grid) - 1.0)) <= tol:
            return n
        y = 1.5 * y - 0.5 * grid * y ** 3
    raise ValueError("Newton rsqrt did not converge")


def calibrate_seeds(cfg, w, steps=2, lanes=64, seed=7, tol=1e-4, margin=2.0, inputs=None, ms_margin=None):
    """Per-site (a, b, iters) from the ranges of mean(x^2)+eps over a calibration run: the
    linear seed is fitted on [m / lo, M * hi] with (lo, hi) = ms_margin (default (margin,
    margin)) and the iteration count verified there (the reference uses [0.8 m, 1.25 M]; a
    wider window keeps conversations whose state drifts past the calibration tokens inside the
    Newton basin, at the cost of about one iteration).  The tails are one-sided: conversations
    outside the calibration range reach mean squares a few times the calibrated maximum but
    stay within about 10 % of the minimum, so an asymmetric ms_margin such as (1.25, 3) covers
    them at about the iteration count of the symmetric (2, 2).  Beyond the window's top the
    linear seed falls towards zero and Newton's iteration, which multiplies a small relative
    seed by only about 1.5 per step there, leaves that lane's norm wrong.  The bootstrap gains use
    [m / margin, M * margin] in either case.
    The run feeds embeddings of random tokens, or the given input batches (lanes, d) in turn."""
    rng = np.random.default_rng(seed)
    cap, state = {}, None
    batches = inputs if inputs is not None else [w["emb"][rng.integers(0, cfg.vocab, lanes)] for _ in range(steps)]
    for x in batches:
        _, state = plain_step(cfg, w, x, state, None, cap)
    seeds = {}
    for tag, rows in cap.items():
        if tag.startswith("peak:"):
            seeds["gain:" + tag[5:]] = boot_gain(margin * max(rows))
            continue
        arr = np.array(rows)
        m, M = float(arr[:, 0].min()), float(arr[:, 1].max())
        mlo, mhi = ms_margin if ms_margin is not None else (margin, margin)
        lo, hi = m / mlo, M * mhi
        a, b = linear_rsqrt_seed(lo, hi)
        seeds[tag] = (a, b, rsqrt_iters_for(a, b, lo, hi, tol))
        seeds["gain:" + tag + ".ms"] = boot_gain(M * margin)
        seeds["gain:" + tag + ".y"] = boot_gain(1.0 / np.sqrt(m / margin))
    return seeds


def boot_gain(peak, target=2.0):
    """Power-of-two gain bringing a site's peak magnitude to <= target before a bootstrap."""
    if peak <= 0:
        return 1.0
    return float(2.0 ** np.floor(np.log2(target / peak)))


def layer_seed_array(seeds, i):
    """The 18 per-layer values of fhe_model_set_layer: Newton seeds of both norms, then the
    bootstrap gains tm.x, tm.ms, u, s, g, cm.x, cm.ms, v, f, tm.y, cm.y, z."""
    g = lambda k: seeds.get("gain:" + k, 1.0)
    return np.array(list(seeds[f"L{i}.tm"]) + list(seeds[f"L{i}.cm"]) +
                    [g(f"L{i}.tm.x"), g(f"L{i}.tm.ms"), g(f"L{i}.u"), g(f"L{i}.s"), g(f"L{i}.g"),
                     g(f"L{i}.cm.x"), g(f"L{i}.cm.ms"), g(f"L{i}.v"), g(f"L{i}.f"),
                     g(f"L{i}.tm.y"), g(f"L{i}.cm.y"), g(f"L{i}.z")], dtype=np.float64)


# -------------------------------------------------------------------------- packing ----
def pack_lanes(x, D, slots):
    """(lanes, width <= D) -> complex slot vector: lane r in block r mod R (R = slots / D),
    real part for r < R, imaginary part for R <= r < 2R."""
    R = slots // D
    if x.shape[0] > 2 * R:
        raise ValueError("more lanes than 2 * slots / D")
    z = np.zeros(slots, dtype=np.complex128)
    xr = x[:R]
    z.reshape(R, D)[: xr.shape[0], : x.shape[1]] += xr
    xi = x[R:]
    z.reshape(R, D)[: xi.shape[0], : x.shape[1]] += 1j * xi
    return z


def unpack_lanes(z, D, lanes, width):
    R = len(z) // D
    blocks = z.reshape(R, D)[:, :width]
    out = np.concatenate([blocks.real, blocks.imag], axis=0)
    return out[:lanes]


# -------------------------------------------------------------------- encrypted model ----
class ModelCfgC(C.Structure):
    _fields_ = [("d", C.c_int), ("dff", C.c_int), ("n_layer", C.c_int), ("D", C.c_int), ("b1", C.c_int),
                ("a_min", C.c_double), ("a_max", C.c_double), ("alpha", C.c_double), ("eps", C.c_double),
                ("shift_mix", C.c_int)]


def _sigs():
    h = lib()
    for name, res, args in [
        ("fhe_model_create", C.c_int, [_VP, C.POINTER(ModelCfgC), C.POINTER(_VP)]),
        ("fhe_model_free", None, [_VP]),
        ("fhe_model_set_layer", C.c_int, [_VP, C.c_int] + [_DP] * 7),
        ("fhe_model_set_output", C.c_int, [_VP, _DP, _DP]),
        ("fhe_model_keygen", C.c_int, [_VP]),
        ("fhe_model_reset", C.c_int, [_VP]),
        ("fhe_model_step", C.c_int, [_VP, _VP, C.POINTER(_VP)]),
        ("fhe_model_stats", C.c_int, [_VP, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
        ("fhe_model_probe", C.c_int, [_VP, C.c_int]),
        ("fhe_server_step", C.c_int, [_VP, C.POINTER(_VP), C.c_int, C.POINTER(_VP), C.POINTER(C.c_int), C.c_int]),
    ]:
        f = getattr(h, name)
        f.restype = res
        f.argtypes = args
    return h


def _dp(a):
    a = np.ascontiguousarray(a, dtype=np.float64)
    return a, a.ctypes.data_as(_DP)


class EncryptedModel:
    """The model uploaded to one engine context."""

    def __init__(self, ctx, cfg: ModelConfig, w, seeds):
        self.ctx, self.cfg = ctx, cfg
        h = _sigs()
        c = ModelCfgC(cfg.d, cfg.dff, cfg.n_layer, cfg.D, cfg.b1, cfg.a_min, cfg.a_max, cfg.alpha, cfg.eps,
                      1 if cfg.shift_mix else 0)
        mh = _VP()
        _check(h.fhe_model_create(ctx.h, C.byref(c), C.byref(mh)))
        self.h = mh
        for i, L in enumerate(w["layers"]):
            vecs = np.concatenate([L[k] for k in ("decay", "b", "g1", "mix", "c", "dd", "p0", "p1", "p2", "g2")] +
                                  [L[f"q{j}"] for j in range(4)] + [L[f"r{j}"] for j in range(3)])
            sd = layer_seed_array(seeds, i)
            keep = [_dp(L[k]) for k in ("win", "wout", "wk", "wr", "wv")] + [_dp(vecs), _dp(sd)]
            _check(h.fhe_model_set_layer(self.h, i, *[p for _, p in keep]))
        g, gp = _dp(w["g_out"])
        so, sop = _dp(np.array(list(seeds["ln_out"]) + [seeds.get("gain:ln_out.x", 1.0),
                                                         seeds.get("gain:ln_out.ms", 1.0),
                                                         seeds.get("gain:ln_out.y", 1.0)], dtype=np.float64))
        _check(h.fhe_model_set_output(self.h, gp, sop))

    def keygen(self):
        _check(lib().fhe_model_keygen(self.h))

    def reset(self):
        _check(lib().fhe_model_reset(self.h))

    def step(self, ct):
        out = _VP()
        _check(lib().fhe_model_step(self.h, ct.h, C.byref(out)))
        return Ciphertext(self.ctx, out)

    def probe(self, k):
        """Diagnostics: make step() return the layer-0 intermediate k (0 = off)."""
        _check(lib().fhe_model_probe(self.h, k))

    def stats(self):
        b, s = C.c_longlong(), C.c_longlong()
        _check(lib().fhe_model_stats(self.h, C.byref(b), C.byref(s)))
        return {"bootstraps": b.value, "steps": s.value}

    def rot_contract(self):
        """The rotation-index contract ("fhe-ssm-rot-indices-v1") a client keygen must satisfy."""
        import json
        h = lib()
        h.fhe_model_rot_contract.restype = C.c_int
        h.fhe_model_rot_contract.argtypes = [_VP, C.c_char_p, C.c_int]
        buf = C.create_string_buffer(1 << 16)
        _check(h.fhe_model_rot_contract(self.h, buf, len(buf)))
        return json.loads(buf.value.decode())

    REFRESH_SITES = ("norm.x", "norm.ms", "norm.y", "norm.m", "norm.tail", "shift.xn", "shift.up", "u", "s.prev",
                     "s.new", "z", "g", "v", "f")

    def refresh_census(self):
        """Bootstraps per refresh site since the model was created."""
        n = len(self.REFRESH_SITES)
        arr = (C.c_longlong * n)()
        h = lib()
        h.fhe_model_refresh_census.restype = C.c_int
        h.fhe_model_refresh_census.argtypes = [C.c_void_p, C.POINTER(C.c_longlong), C.c_int]
        _check(h.fhe_model_refresh_census(self.h, arr, n))
        return dict(zip(self.REFRESH_SITES, list(arr)))

    def __del__(self):
        try:
            if getattr(self, "h", None) and getattr(self.ctx, "h", None):
                lib().fhe_model_free(self.h)
            self.h = None
        except (TypeError, AttributeError):   # module globals already torn down at interpreter exit
            pass


def rel_err_rms(enc, ref):
    """relErrRms = rms(enc - ref) / rms(ref) (spec_decode/fidelity_tick.py:298-307)."""
    return float(np.sqrt(np.mean((enc - ref) ** 2)) / np.sqrt(np.mean(ref ** 2)))
