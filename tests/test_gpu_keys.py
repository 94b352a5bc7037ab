"""The key material path on the GPU: seeded part files and the rotation-index contract.

A client context holds the secret; a server context with the same chain holds none.  The client
reads the server model's rotation-index contract, mints exactly its automorphism indices, and
writes them with the relinearisation key to a seeded part file (FSSMSKY1: b words plus the
32-byte seeds of the a-halves).  The server loads the file (a-halves re-expanded on its GPU),
sets up bootstrapping and the model without any key generation, and runs a model step on the
client's ciphertext; the client decrypts it.  Checked: the loaded keys equal the client's word for
word, a file of another chain is refused, and the decrypted step matches the float64 model."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CTX = dict(logN=13, L=28, K=4, alpha=4, hw=192, boot_primes=14)


def test_part_file_round_trip_and_refusal(tmp_path):
    import fhessm
    # K = 3 special primes (180 bits) above a digit of alpha = 3 45-bit limbs: the switching noise
    # stays small; `other` has another chain on the same GPU
    a = fhessm.CryptoContext(logN=13, L=8, K=3, alpha=3, hw=64)
    b = fhessm.CryptoContext(logN=13, L=8, K=3, alpha=3, hw=64)
    other = fhessm.CryptoContext(logN=13, L=7, K=3, alpha=3, hw=64)
    try:
        a.KeyGen(seed=21)
        a.EvalRotateKeyGen([1, -2, 7], conj=True)
        idx = [0] + [a.rot_index(r) for r in (1, -2, 7)] + [2 * a.N - 1]
        path = str(tmp_path / "evalrot.part000.seeded.bin")
        a.save_keys_part(path, idx, "client")
        lay, mods, tag = fhessm.part_header(path)
        assert lay["count"] == len(idx) and tag == "client" and (mods == a.moduli).all()
        assert b.load_keys_part(path) == len(idx)
        for k in idx:
            assert (b.key_words(k) == a.key_words(k)).all(), k
        assert b.load_keys_part(path) == 0          # keys already held are kept
        with pytest.raises(fhessm.FheError, match="another context"):
            other.load_keys_part(path)
        # a rotation on the server of a client ciphertext, decrypted by the client
        z = np.random.default_rng(1).uniform(-1, 1, a.slots)
        ct = a.Encrypt(a.MakeCKKSPackedPlaintext(z, 1))
        rb = b.EvalRotate(b.ct_from_words(ct.words(), ct.level, ct.scale), 7)
        assert (rb.words() == a.EvalRotate(ct, 7).words()).all()   # loaded keys act as the minted ones
        back = a.ct_from_words(rb.words(), rb.level, rb.scale)
        assert np.abs(a.Decrypt(back).real - np.roll(z, -7)).max() < 1e-4
    finally:
        for c in (a, b, other):
            c.close()


def test_secretless_server_from_contract_and_part_file(tmp_path):
    import fhessm
    from fhessm.model import (EncryptedModel, ModelConfig, calibrate_seeds, pack_lanes, plain_step, rel_err_rms,
                              synthetic_weights, unpack_lanes)
    cfg = ModelConfig(d=48, dff=128, n_layer=1, vocab=512, D=64, b1=8)
    w = synthetic_weights(cfg, seed=15)
    seeds = calibrate_seeds(cfg, w, steps=3, lanes=128)
    server = fhessm.CryptoContext(**CTX)
    client = fhessm.CryptoContext(**CTX)
    try:
        m = EncryptedModel(server, cfg, w, seeds)
        contract = m.rot_contract()
        assert contract["contract"] == "fhe-ssm-rot-indices-v1" and contract["ring"] == server.N
        assert 2 * server.N - 1 in contract["autoIndices"]
        # the client mints the contract's indices and ships them with its relinearisation key
        client.KeyGen(seed=16)
        client.keygen_auto(contract["autoIndices"])
        path = str(tmp_path / "keys.seeded.bin")
        client.save_keys_part(path, [0] + contract["autoIndices"], "session")
        assert server.load_keys_part(path) == 1 + len(contract["autoIndices"])
        server.EvalBootstrapSetup(24.0, 59)      # every bootstrap key is in the file: no keygen
        m.keygen()                               # likewise for the model's rotations
        lanes = 2 * server.slots // cfg.D
        x = w["emb"][np.random.default_rng(3).integers(0, cfg.vocab, lanes)]
        ct = client.Encrypt(client.MakeCKKSPackedPlaintext(pack_lanes(x, cfg.D, client.slots)))
        out = m.step(server.ct_from_words(ct.words(), ct.level, ct.scale))
        y = unpack_lanes(client.Decrypt(client.ct_from_words(out.words(), out.level, out.scale)), cfg.D, lanes, cfg.d)
        ref, _ = plain_step(cfg, w, x, None)
        assert rel_err_rms(y, ref) < 1e-3
    finally:
        server.close()
        client.close()
