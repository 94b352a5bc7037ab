"""The encrypted RWKV-7 circuit (fhessm.rwkv7.EncryptedRWKV7) on the plaintext slot simulator
(CPU): several heads, several conversations and several head blocks per state ciphertext, so
that every move between the contiguous channel layout and the wkv state blocks (the rotation,
the bit steps, the per-block transpose of the readout) and the level bookkeeping run.  With
exact slot arithmetic the circuit must reproduce the float64 model with the same polynomial
sites to round-off."""
import numpy as np
import pytest

from sim_engine import SimContext


def run(shape, slots, convs, tokens, seed=3):
    from fhessm.rwkv7 import EncryptedRWKV7, RWKV7Shape, Sites, fit_sites, new_state, step, synthetic_weights
    sh = RWKV7Shape(**shape)
    w = synthetic_weights(sh, seed=seed)
    rng = np.random.default_rng(seed + 1)
    seqs = [rng.integers(0, sh.vocab_size, convs) for _ in range(tokens)]
    fits = fit_sites(sh, w, seqs, degree=7)   # sites fitted on the run itself: every input inside
    cx = SimContext(slots)
    EncryptedRWKV7.keygen(cx, sh)
    model = EncryptedRWKV7(cx, sh, w, fits, convs=convs)
    st = new_state(sh, convs)
    sites = Sites(fits)
    errs = []
    for toks in seqs:
        ref = step(sh, w, toks, st, sites)
        x = model.client_input(toks)
        out = model.step(cx.Encrypt(cx.MakeCKKSPackedPlaintext(model.pack(x), level=14)))
        lg = model.client_logits(model.unpack(cx.Decrypt(out)))
        errs.append(np.abs(lg - ref).max() / np.abs(ref).max())
        # nothing outside the conversations in use
        assert np.abs(cx.Decrypt(out)[convs * sh.n_embd:]).max() < 1e-9 if convs * sh.n_embd < slots else True
    return errs, model, cx


@pytest.mark.parametrize("convs", [1, 3])
def test_heads_and_conversations(convs):
    """head size 16, 4 heads, 1024 slots: 4 or 12 head blocks in every state row ciphertext"""
    shape = dict(n_layer=2, n_embd=64, head_size=16, d_decay=8, d_aaa=8, d_mv=4, d_gate=16, dim_ffn=128,
                 vocab_size=64)
    errs, model, cx = run(shape, 1024, convs, 3)
    assert model.blocks[0].wkv.blocks == 4 * convs
    assert max(errs) < 1e-9, errs


def test_full_slots():
    """every slot in use: 2 heads x 4 conversations of 32 channels at 256 slots"""
    shape = dict(n_layer=1, n_embd=32, head_size=16, d_decay=8, d_aaa=8, d_mv=4, d_gate=16, dim_ffn=64,
                 vocab_size=64)
    errs, model, cx = run(shape, 256, 8, 2)
    assert max(errs) < 1e-9, errs


@pytest.mark.parametrize("blocks", [1, 5, 16])
def test_wkv_step_alone(blocks):
    """EncryptedWkv's row-stacked update and its readout from the old rows, two steps on random
    state and inputs (head size 16, 256 slots), against S <- S diag(w) + (S a) b^T + v k^T,
    y = S' r (rwkv7_model.py:290-296)"""
    from fhessm.rwkv7 import EncryptedWkv
    N = 16
    cx = SimContext(256, L=34)
    cx.EvalRotateKeyGen(EncryptedWkv.rotations(N))
    wkv = EncryptedWkv(cx, N, blocks)
    rng = np.random.default_rng(blocks)
    S = rng.normal(size=(blocks, N, N))
    rows = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(z)) for z in wkv.pack_state(S)]
    for _ in range(2):
        w, a, b, k, r, v = (rng.normal(size=(blocks, N)) for _ in range(6))
        S = S * w[:, None, :] + np.einsum("bij,bj->bi", S, a)[:, :, None] * b[:, None, :] + v[:, :, None] * k[:, None, :]
        y = np.einsum("bij,bj->bi", S, r)
        cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(wkv.pack_channel(t))) for t in (w, a, b, k, r, v)]
        rows, y_ct = wkv.step(rows, *cts)
        assert np.abs(wkv.unpack_state([cx.Decrypt(c) for c in rows]) - S).max() < 1e-9 * np.abs(S).max()
        assert np.abs(wkv.unpack_channel(cx.Decrypt(y_ct)) - y).max() < 1e-9 * np.abs(y).max()
        assert rows[0].level == y_ct.level    # a row and the readout both spend 3 levels a step
