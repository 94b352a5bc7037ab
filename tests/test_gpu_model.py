"""GPU test of the encrypted model step against the float64 plaintext model.

A reduced configuration in the spirit of harness/cpu_real_model.cpp (d = 48, deliberately not
a power of two; dff = 128 chunked by D = 64; 2 layers) run for two steps (cold start, then
with the carried state) over 128 distinct lanes, with real bootstrapping.  The decrypted
outputs must match the plaintext model (exact 1/sqrt) within relErrRms <= 1e-3 and the
logits' top-1 must agree (baseline acceptance: relErrRms <= 1e-3, top-1 >= 0.98).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_model_two_steps_small():
    import fhessm
    from fhessm.model import (EncryptedModel, ModelConfig, calibrate_seeds, pack_lanes, plain_step, rel_err_rms,
                              synthetic_weights, unpack_lanes)
    cfg = ModelConfig(d=48, dff=128, n_layer=2, vocab=512, D=64, b1=8)
    w = synthetic_weights(cfg, seed=5)
    seeds = calibrate_seeds(cfg, w, steps=3, lanes=128)
    cx = fhessm.CryptoContext(logN=13, L=28, K=4, alpha=4, hw=192, boot_primes=14)
    cx.KeyGen(seed=9)
    cx.EvalBootstrapSetup(24.0, 59)
    m = EncryptedModel(cx, cfg, w, seeds)
    m.keygen()
    lanes = 2 * cx.slots // cfg.D
    rng = np.random.default_rng(3)
    state_exact, state_newton = None, None
    for step in range(2):
        ids = rng.integers(0, cfg.vocab, lanes)
        x = w["emb"][ids]
        ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(pack_lanes(x, cfg.D, cx.slots)))
        out = m.step(ct)
        y = unpack_lanes(cx.Decrypt(out), cfg.D, lanes, cfg.d)
        ref, state_exact = plain_step(cfg, w, x, state_exact)
        refn, state_newton = plain_step(cfg, w, x, state_newton, seeds)
        e_exact, e_newton = rel_err_rms(y, ref), rel_err_rms(y, refn)
        lg, lr = y @ w["emb"].T, ref @ w["emb"].T
        top1 = float(np.mean(lg.argmax(-1) == lr.argmax(-1)))
        print(f"step {step}: relErrRms vs exact {e_exact:.2e}, vs Newton circuit {e_newton:.2e}, "
              f"logits {rel_err_rms(lg, lr):.2e}, top1 {top1:.3f}, {m.stats()}")
        assert e_newton < 1e-3
        assert e_exact < 1e-3
        assert rel_err_rms(lg, lr) < 1e-3
        assert top1 >= 0.98


def test_model_served_through_request_files(tmp_path):
    """The same small model behind the native serve loop: two requests of one session (the first
    with req.0.reset), answered with the carried state; outputs decrypt to the plaintext model."""
    import threading

    import fhessm
    from fhessm import serve as sv
    from fhessm.model import (EncryptedModel, ModelConfig, calibrate_seeds, pack_lanes, plain_step, rel_err_rms,
                              synthetic_weights, unpack_lanes)
    cfg = ModelConfig(d=48, dff=128, n_layer=2, vocab=512, D=64, b1=8)
    w = synthetic_weights(cfg, seed=6)
    seeds = calibrate_seeds(cfg, w, steps=3, lanes=128)
    cx = fhessm.CryptoContext(logN=13, L=28, K=4, alpha=4, hw=192, boot_primes=14)
    cx.KeyGen(seed=10)
    cx.EvalBootstrapSetup(24.0, 59)
    m = EncryptedModel(cx, cfg, w, seeds)
    m.keygen()
    d = str(tmp_path)
    served = {}
    th = threading.Thread(target=lambda: served.setdefault("n", sv.serve_model(m, d, timeout_ms=120000,
                                                                               max_requests=2)))
    th.start()
    lanes = 2 * cx.slots // cfg.D
    rng = np.random.default_rng(4)
    state = None
    for n in range(2):
        x = w["emb"][rng.integers(0, cfg.vocab, lanes)]
        ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(pack_lanes(x, cfg.D, cx.slots)))
        sv.submit(d, n, [(ct.level, ct.scale, ct.words())], reset=(n == 0), lanes=lanes, tokensReal=1)
        (resp, meta) = sv.wait_response(d, n, timeout=300)
        level, scale, words = resp[0]
        y = unpack_lanes(cx.Decrypt(cx.ct_from_words(words, level, scale)), cfg.D, lanes, cfg.d)
        ref, state = plain_step(cfg, w, x, state)
        assert rel_err_rms(y, ref) < 1e-3, n
        assert meta["reset"] is (n == 0)
    th.join(60)
    assert served.get("n") == 2
