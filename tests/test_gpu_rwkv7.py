"""RWKV-7 (config 5's model) on the engine against the float64 recurrence of fhessm.rwkv7
(itself pinned to the reference harness, tests/test_rwkv7_reference.py): the wkv state update
alone, one block, and whole models of several blocks, heads and conversations, with the same
polynomial sites and Newton seeds on both sides."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_wkv_state_update_matches_float64():
    """Four head blocks (two conversations of two heads, N = 64) in the row-stacked layout: the
    state as 64 row ciphertexts at N = 2^14, two steps of S <- S diag(w) + (S a) b^T + v k^T and
    y = S r with a = -kk, b = kk * a (kk a unit vector per head).  Decrypted state and readout
    must match to 1e-4 of their largest entry."""
    import fhessm
    from fhessm.rwkv7 import EncryptedWkv
    N, blocks = 64, 4
    cx = fhessm.CryptoContext(logN=14, L=18, K=3, alpha=3, hw=64)
    try:
        cx.KeyGen(seed=21)
        cx.EvalRotateKeyGen(EncryptedWkv.rotations(N))
        wkv = EncryptedWkv(cx, N, blocks)
        rng = np.random.default_rng(4)
        S = 0.3 * rng.normal(size=(blocks, N, N))
        enc = lambda z: cx.Encrypt(cx.MakeCKKSPackedPlaintext(z))
        S_ct = [enc(z) for z in wkv.pack_state(S)]
        for step in range(2):
            w = rng.uniform(0.5, 1.0, (blocks, N))
            kk = rng.normal(size=(blocks, N))
            kk /= np.linalg.norm(kk, axis=1, keepdims=True)
            a_rate = rng.uniform(0.0, 1.0, (blocks, N))
            a, b = -kk, kk * a_rate
            k = rng.normal(0.0, 0.3, (blocks, N))
            r = rng.normal(0.0, 0.3, (blocks, N))
            v = rng.normal(size=(blocks, N))
            # float64 reference (rwkv7_model.py:290-296)
            Sa = np.einsum("bij,bj->bi", S, a)
            S = S * w[:, None, :] + Sa[:, :, None] * b[:, None, :] + v[:, :, None] * k[:, None, :]
            y = np.einsum("bij,bj->bi", S, r)
            # encrypted
            cts = [enc(wkv.pack_channel(t)) for t in (w, a, b, k, r, v)]
            S_ct, y_ct = wkv.step(S_ct, *cts)
            S_dec = wkv.unpack_state([cx.Decrypt(c) for c in S_ct])
            y_dec = wkv.unpack_channel(cx.Decrypt(y_ct))
            es = np.abs(S_dec - S).max() / np.abs(S).max()
            ey = np.abs(y_dec - y).max() / np.abs(y).max()
            print(f"step {step}: state err {es:.2e}, readout err {ey:.2e}, state level {S_ct[0].level}, "
                  f"readout level {y_ct.level}")
            assert es < 1e-4 and ey < 1e-4
    finally:
        cx.close()


def test_rwkv7_block_matches_polynomial_model():
    """One RWKV-7 block (layer 0: time mix with the wkv state, channel mix) on the engine for one
    head of 64 channels, two tokens, against the float64 block with the same polynomial sites and
    Newton seeds.  N = 2^13 with the bootstrapping chain (q0 60 bits, 19 x 45-bit user primes,
    14 x 58-bit bootstrap primes, K = 4): a correctness test of the circuit, not a secure
    parameter set at this ring size."""
    import fhessm
    from fhessm.rwkv7 import (EncryptedRWKV7, EncryptedRWKV7Block, RWKV7Shape, Sites, _ln, block_step, fit_sites,
                              new_state, synthetic_weights)
    sh = RWKV7Shape(n_layer=1, n_embd=64, head_size=64, d_decay=16, d_aaa=16, d_mv=8, d_gate=32, dim_ffn=256,
                    vocab_size=256)
    w = synthetic_weights(sh, seed=9)
    fits = fit_sites(sh, w, [np.random.default_rng(12).integers(0, sh.vocab_size, 32) for _ in range(4)], degree=15)
    sites = Sites(fits)
    cx = fhessm.CryptoContext(logN=13, L=34, K=4, alpha=4, hw=64, boot_primes=14)
    try:
        cx.KeyGen(seed=23)
        EncryptedRWKV7.keygen(cx, sh)
        cx.EvalBootstrapSetup(24.0, 31, 4)
        blk = EncryptedRWKV7Block(cx, sh, w, 0, fits)
        st = new_state(sh, 1)
        toks = np.random.default_rng(13).integers(0, sh.vocab_size, 2)
        for t, tok in enumerate(toks):
            x = _ln(sites, "blocks.0.ln0", w["emb.weight"][[tok]], w["blocks.0.ln0.weight"], w["blocks.0.ln0.bias"])
            ref, _ = block_step(sh, w, 0, x.copy(), st[0], None, sites, ln0=False)
            z = np.zeros(cx.slots)
            z[:64] = x[0]
            out, _ = blk.step(cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, level=14)))   # the user region's top
            got = np.asarray(cx.Decrypt(out)).real[:64]
            err = np.abs(got - ref[0]).max() / np.abs(ref[0]).max()
            print(f"token {t}: block output rel err {err:.2e} (level {out.level})")
            assert err < 1e-3
    finally:
        cx.close()


def test_rwkv7_two_layers_logits_match_polynomial_model():
    """Two blocks (the value residual of block 1 on block 0's value), four tokens, logits after the
    client's output norm and head against the float64 model with the same sites."""
    import fhessm
    from fhessm.rwkv7 import EncryptedRWKV7, RWKV7Shape, Sites, fit_sites, new_state, step, synthetic_weights
    sh = RWKV7Shape(n_layer=2, n_embd=64, head_size=64, d_decay=16, d_aaa=16, d_mv=8, d_gate=32, dim_ffn=256,
                    vocab_size=256)
    w = synthetic_weights(sh, seed=10)
    fits = fit_sites(sh, w, [np.random.default_rng(14).integers(0, sh.vocab_size, 32) for _ in range(4)], degree=15)
    sites = Sites(fits)
    cx = fhessm.CryptoContext(logN=13, L=34, K=4, alpha=4, hw=64, boot_primes=14)
    try:
        cx.KeyGen(seed=24)
        EncryptedRWKV7.keygen(cx, sh)
        cx.EvalBootstrapSetup(24.0, 31, 4)
        model = EncryptedRWKV7(cx, sh, w, fits)
        st = new_state(sh, 1)
        for t, tok in enumerate(np.random.default_rng(15).integers(0, sh.vocab_size, 4)):
            ref = step(sh, w, [tok], st, sites)
            z = np.zeros(cx.slots)
            z[:64] = model.client_input([tok])[0]
            out = model.step(cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, level=14)))
            hid = np.asarray(cx.Decrypt(out)).real[:64][None]
            lg = model.client_logits(hid)
            err = np.abs(lg - ref).max() / np.abs(ref).max()
            print(f"token {t}: logits rel err {err:.2e}, top-1 {lg.argmax() == ref.argmax()}")
            assert err < 1e-3 and lg.argmax() == ref.argmax()
    finally:
        cx.close()


def test_rwkv7_multi_head_conversations_logits():
    """Two heads of 64 (C = 128), two blocks, two conversations at N = 2^14 (four head blocks in
    every state row ciphertext); logits of both conversations over three tokens."""
    import fhessm
    from fhessm.rwkv7 import EncryptedRWKV7, RWKV7Shape, Sites, fit_sites, new_state, step, synthetic_weights
    sh = RWKV7Shape(n_layer=2, n_embd=128, head_size=64, d_decay=16, d_aaa=16, d_mv=8, d_gate=32, dim_ffn=256,
                    vocab_size=256)
    w = synthetic_weights(sh, seed=11)
    rng = np.random.default_rng(16)
    seqs = [rng.integers(0, sh.vocab_size, 2) for _ in range(3)]
    cal = [np.concatenate([s, rng.integers(0, sh.vocab_size, 30)]) for s in seqs]
    fits = fit_sites(sh, w, cal, degree=15)
    sites = Sites(fits)
    cx = fhessm.CryptoContext(logN=14, L=34, K=4, alpha=4, hw=64, boot_primes=14)
    try:
        cx.KeyGen(seed=25)
        EncryptedRWKV7.keygen(cx, sh)
        cx.EvalBootstrapSetup(24.0, 31, 4)
        model = EncryptedRWKV7(cx, sh, w, fits, convs=2)
        st = new_state(sh, 2)
        for t, toks in enumerate(seqs):
            ref = step(sh, w, toks, st, sites)
            out = model.step(cx.Encrypt(cx.MakeCKKSPackedPlaintext(model.pack(model.client_input(toks)), level=14)))
            lg = model.client_logits(model.unpack(cx.Decrypt(out)))
            err = np.abs(lg - ref).max() / np.abs(ref).max()
            top1 = (lg.argmax(-1) == ref.argmax(-1)).all()
            print(f"token {t}: logits rel err {err:.2e}, top-1 {top1}")
            assert err < 1e-3 and top1
    finally:
        cx.close()
