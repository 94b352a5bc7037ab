"""GPU parity: every integer RNS primitive of the CUDA engine, called through the C-ABI,
must equal the CPU oracle word for word (canonical residues, evaluation form).

Covers config 2 of the baseline (NTT/iNTT, HMult + relinearise + rescale, hoisted
power-of-two rotations, conjugation) at reduced ring sizes the oracle finishes in seconds,
plus the production ring N = 2^16 for the NTT and one key switch.  The key material is
also compared: the engine's seeded keygen must reproduce the oracle's keys bit for bit
(secret, public key, relinearisation and rotation keys).
"""
import numpy as np
import pytest

from oracle_lib import Oracle, derive_seed, load

pytestmark = pytest.mark.gpu

OLIB = load()


def make_pair(logN, L, K, alpha, hw=64, seed=7):
    import fhessm
    cx = fhessm.CryptoContext(logN=logN, L=L, K=K, alpha=alpha, hw=hw)
    o = Oracle(logN, cx.moduli[:L], cx.moduli[L:], alpha, OLIB)
    return cx, o


@pytest.fixture(scope="module")
def pair():
    cx, o = make_pair(13, 7, 3, 3)
    cx.KeyGen(seed=1234)
    return cx, o


def rand_poly(o, nl, rng, first=0):
    return np.stack([rng.integers(0, int(o.mods[first + i]), o.N, dtype=np.uint64) for i in range(nl)])


@pytest.mark.parametrize("logN", [12, 13, 14, 15, 16])
def test_ntt_bit_exact(logN):
    cx, o = make_pair(logN, 3, 2, 2)
    rng = np.random.default_rng(logN)
    mods = [0, 1, 2, 3, 4]
    a = np.stack([rng.integers(0, int(o.mods[m]), o.N, dtype=np.uint64) for m in mods])
    got = cx.ntt(a, mods).reshape(len(mods), o.N)
    for i, m in enumerate(mods):
        assert (got[i] == o.ntt(a[i], m)).all(), (logN, m)
    back = cx.ntt(got, mods, inverse=True).reshape(len(mods), o.N)
    assert (back == a).all()
    # inverse on random input also matches the oracle's inverse
    b = cx.ntt(a, mods, inverse=True).reshape(len(mods), o.N)
    for i, m in enumerate(mods):
        assert (b[i] == o.intt(a[i], m)).all()


def test_keygen_bit_exact(pair):
    cx, o = pair
    ms = (1234).to_bytes(8, "little") + bytes(24)
    s = o.secret(derive_seed(OLIB, ms, 0xFFFFFFF1), 64)
    assert (cx.secret_coeffs() == s).all()
    se = o.secret_eval(s)
    pk = o.keygen_public(se, derive_seed(OLIB, ms, 0xFFFFFFF0))
    assert (cx.public_key_words() == pk).all()
    s2 = np.stack([(se[m].astype(object) ** 2 % int(o.mods[m])).astype(np.uint64) for m in range(len(o.mods))])
    rlk = o.keygen_switch(s2, se, derive_seed(OLIB, ms, 2))
    assert (cx.key_words(0) == rlk).all()
    cx.EvalRotateKeyGen([1, 2, 4, -3], conj=True)
    M = 2 * o.N
    for r in (1, -3):
        k = cx.rot_index(r)
        sk = np.stack([o.automorph_eval(se[m], pow(k, -1, M)) for m in range(len(o.mods))])
        key = o.keygen_switch(se, sk, derive_seed(OLIB, ms, k))
        assert (cx.key_words(k) == key).all(), r


def test_keyswitch_bit_exact_all_levels(pair):
    cx, o = pair
    rng = np.random.default_rng(1)
    key = cx.key_words(0)
    for level in range(cx.L):
        nl = cx.L - level
        d = rand_poly(o, nl, rng)
        g0, g1 = cx.keyswitch_raw(d, level, key)
        e0, e1 = o.keyswitch(d, nl, key)
        assert (g0 == e0).all() and (g1 == e1).all(), level


def test_hmult_relin_rescale_bit_exact(pair):
    cx, o = pair
    rng = np.random.default_rng(2)
    for level in (0, 3, 5):
        nl = cx.L - level
        a = np.stack([rand_poly(o, nl, rng), rand_poly(o, nl, rng)])
        b = np.stack([rand_poly(o, nl, rng), rand_poly(o, nl, rng)])
        ca, cb = cx.ct_from_words(a, level), cx.ct_from_words(b, level)
        prod = cx.EvalMult(ca, cb)
        ref = o.ct_mul_relin(a, b, nl, cx.key_words(0))
        assert (prod.words() == ref).all(), level
        cx.RescaleInPlace(prod)
        assert (prod.words() == o.ct_rescale(ref, nl)).all(), level


def test_rotation_hoisted_and_conjugation_bit_exact(pair):
    cx, o = pair
    rng = np.random.default_rng(3)
    level = 1
    nl = cx.L - level
    a = np.stack([rand_poly(o, nl, rng), rand_poly(o, nl, rng)])
    ca = cx.ct_from_words(a, level)
    steps = [1, 2, 4, -3]
    cx.EvalRotateKeyGen(steps, conj=True)
    hoisted = cx.EvalFastRotation(ca, steps)
    for r, h in zip(steps, hoisted):
        k = cx.rot_index(r)
        ref = o.ct_automorph(a, nl, k, cx.key_words(k))
        assert (cx.EvalRotate(ca, r).words() == ref).all(), r
        assert (h.words() == ref).all(), r
    k = 2 * o.N - 1
    assert (cx.EvalConj(ca).words() == o.ct_automorph(a, nl, k, cx.key_words(k))).all()


def test_elementwise_bit_exact(pair):
    cx, o = pair
    rng = np.random.default_rng(4)
    level = 2
    nl = cx.L - level
    a = np.stack([rand_poly(o, nl, rng), rand_poly(o, nl, rng)])
    b = np.stack([rand_poly(o, nl, rng), rand_poly(o, nl, rng)])
    p = rand_poly(o, nl, rng)
    ca, cb = cx.ct_from_words(a, level), cx.ct_from_words(b, level)
    assert (cx.EvalAdd(ca, cb).words() == o.ct_add(a, b, nl)).all()
    assert (cx.EvalMult(ca, cx.pt_from_words(p, level)).words() == o.ct_mul_pt(a, p, nl)).all()


def test_encode_encrypt_bit_exact_and_decrypt(pair):
    cx, o = pair
    rng = np.random.default_rng(5)
    z = rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2)
    level = 0
    scale = cx.GetScalingFactorReal(level)
    pt = cx.MakeCKKSPackedPlaintext(z, level)
    ref = o.encode(z, scale, cx.L)
    assert (cx.pt_words(pt) == ref).all()
    ct = cx.Encrypt(pt)
    ms = (1234).to_bytes(8, "little") + bytes(24)
    se = o.secret_eval(cx.secret_coeffs())
    pk = cx.public_key_words()
    # engine encryptions draw seeds derive(master, ENCRYPT, counter); counter 0 is the first
    refct = o.encrypt(pk, ref, cx.L, derive_seed(OLIB, ms, 0xFFFFFFF2, 0))
    assert (ct.words() == refct).all()
    got = cx.Decrypt(ct)
    assert np.abs(got - z).max() < 1e-6                                   # encdec (cpu_real_model.cpp:255-260)


def test_rotate_convention_decrypted(pair):
    """EvalRotate(ct, k)[i] == x[i + k]  (harness/cpu_real_model.cpp:262-268), all power-of-two steps."""
    cx, o = pair
    rng = np.random.default_rng(6)
    z = rng.uniform(-1, 1, o.N // 2)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, 0))
    steps = [1 << i for i in range(cx.logN - 1)]
    cx.EvalRotateKeyGen(steps)
    for r, h in zip(steps, cx.EvalFastRotation(ct, steps)):
        assert np.abs(cx.Decrypt(h).real - np.roll(z, -r)).max() < 1e-4, r


def test_rotate_sum_lazy_moddown(pair):
    """sum_i rot(ct_i, k_i) with one ModDown of the summed inner products: decrypts to the
    rotated sum, within the rounding of the P-division of the one-at-a-time result."""
    cx, o = pair
    rng = np.random.default_rng(9)
    steps = [0, 3, -5, 64, 1000]
    cx.EvalRotateKeyGen([s for s in steps if s])
    zs = [rng.uniform(-1, 1, o.N // 2) + 1j * rng.uniform(-1, 1, o.N // 2) for _ in steps]
    cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, 1)) for z in zs]
    got = cx.Decrypt(cx.EvalRotateSum(cts, steps))
    want = sum(np.roll(z, -s) for z, s in zip(zs, steps))
    assert np.abs(got - want).max() < 1e-4
    one = None
    for c, s in zip(cts, steps):
        r = cx.EvalRotate(c, s) if s else c
        one = r if one is None else cx.EvalAdd(one, r)
    assert np.abs(got - cx.Decrypt(one)).max() < 1e-6


def test_production_ring_keyswitch_bit_exact():
    """N = 2^16 with the baseline's chain shape at a reduced depth: L=6, K=4, alpha=4."""
    cx, o = make_pair(16, 6, 4, 4)
    cx.KeyGen(seed=5)
    rng = np.random.default_rng(8)
    key = cx.key_words(0)
    for level in (0, 3):
        nl = cx.L - level
        d = rand_poly(o, nl, rng)
        g0, g1 = cx.keyswitch_raw(d, level, key)
        e0, e1 = o.keyswitch(d, nl, key)
        assert (g0 == e0).all() and (g1 == e1).all(), level
