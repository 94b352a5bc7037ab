"""Config 1 of the baseline at its own shapes: one encrypted recurrent step of a single
polynomial-SSM block (the config's own chain holds the time-mix half without bootstrapping).

N = 2^16, q0 60 bits and 45-bit scaling primes, K = 4 x 60-bit special primes, alpha = 4
(dnum = 5 at 20 limbs), HW-192 secret, sigma 3.19.  Block: d = 256 (4 heads x 64 diagonal-decay
channels), dff = 1024 (4 d), 64 conversations packed across the slots.  Weights N(0, 0.02),
polynomial coefficients U[-1, 1] (degree-3 gate and activation), inputs N(0, 1), all seeded;
Newton seeds calibrated on other N(0, 1) draws over the reference's window [0.8 m, 1.25 M].

Levels.  A whole block (two rmsnorms with two Newton iterations each, shift-mix, W_in, the scan
and readout, the degree-3 gate, W_out, then W_k/W_r, the activation and gate polynomials, W_v)
uses about 31 levels, more than the 19 of the config's 20-limb chain.  A longer chain of 45-bit
primes with one scale anchor does not help: the FLEXIBLEAUTO recursion Delta_{l-1} = Delta_l^2 / q_l
doubles the relative drift of the scale at every level, so 30 levels below the anchor the scales
leave the 61-bit range.  So:
  * the time-mix half (rmsnorm .. W_out and the residual) runs on the config's own 20-limb chain
    with no bootstrap (the context has no bootstrap keys; the refresh census stays zero);
  * the whole block runs on the bootstrapping chain of the 405M model (q0, 13 x 45-bit user primes,
    14 x 58-bit primes for the bootstrap), refreshing where the levels run out.
Decrypted block outputs must match the float64 model (exact 1/sqrt) within relErrRms <= 1e-3, and
the top-1 of a readout through a seeded tied embedding must agree on >= 98 % of the lanes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LANES = 64


def run_block(L, probe, boot_primes=0):
    import fhessm
    from fhessm.model import (EncryptedModel, ModelConfig, calibrate_seeds, pack_lanes, plain_step, rel_err_rms,
                              synthetic_weights, unpack_lanes)
    cfg = ModelConfig(d=256, dff=1024, n_layer=1, vocab=4096, D=256, b1=16)
    w = synthetic_weights(cfg, seed=41)
    cal = np.random.default_rng(42)
    seeds = calibrate_seeds(cfg, w, margin=1.25, inputs=[cal.normal(0, 1, (LANES, cfg.d)) for _ in range(4)])
    cx = fhessm.CryptoContext(logN=16, L=L, K=4, alpha=4, hw=192, boot_primes=boot_primes)
    try:
        cx.KeyGen(seed=43)
        if boot_primes:
            cx.EvalBootstrapSetup(24.0, 31, 4)
        m = EncryptedModel(cx, cfg, w, seeds)
        m.keygen()
        m.probe(probe)
        x = np.random.default_rng(44).normal(0, 1, (LANES, cfg.d))
        ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(pack_lanes(x, cfg.D, cx.slots)))
        out = m.step(ct)
        y = unpack_lanes(cx.Decrypt(out), cfg.D, LANES, cfg.d)
        levels_used = out.level
        boots = m.stats()["bootstraps"]
        assert boot_primes or (boots == 0 and not any(m.refresh_census().values()))
    finally:
        cx.close()
    if probe == 11:
        ref, _ = plain_step(cfg, w, x, None, hidden=True)
    else:   # probe 7: h + W_out g, the residual after the time mix: a copy of the model up to there
        ref = time_mix_reference(cfg, w, x)
    lg, lr = y @ w["emb"].T, ref @ w["emb"].T
    return rel_err_rms(y, ref), rel_err_rms(lg, lr), float(np.mean(lg.argmax(-1) == lr.argmax(-1))), levels_used, boots


def time_mix_reference(cfg, w, x):
    """h + W_out g of layer 0 on a cold start (the first half of plain_step)."""
    L = w["layers"][0]
    ms = (x * x).mean(-1, keepdims=True) + cfg.eps
    u = x / np.sqrt(ms) * L["g1"]
    u = u * L["mix"]                      # shift-mix with a zero previous token
    xx = u @ L["win"].T
    s = L["b"] * xx                       # scan from a zero state
    z = L["c"] * s + L["dd"] * xx
    g = z * (L["p0"] + L["p1"] * z + L["p2"] * z * z)
    return x + cfg.alpha * (g @ L["wout"].T)


def test_config1_time_mix_on_the_20_limb_chain():
    e, el, top1, lv, _ = run_block(20, 7)
    print(f"time mix, L=20: relErrRms {e:.2e}, logits {el:.2e}, top-1 {top1:.3f}, output level {lv} "
          f"({lv} of 19 levels used)")
    assert e <= 1e-3 and el <= 1e-3 and top1 >= 0.98


def test_config1_whole_block_with_refreshes():
    e, el, top1, lv, boots = run_block(28, 11, boot_primes=14)
    print(f"block, bootstrapping chain: relErrRms {e:.2e}, logits {el:.2e}, top-1 {top1:.3f}, "
          f"{boots} bootstraps")
    assert e <= 1e-3 and el <= 1e-3 and top1 >= 0.98
