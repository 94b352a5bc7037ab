"""CPU tests of the oracle (the checker): known answers and algebraic properties.

These pin the oracle before it is trusted as the reference for the CUDA engine:
  * ChaCha20 against RFC 8439 section 2.3.2 (the block-function test vector);
  * the NTT against direct evaluation at the odd powers of psi in bit-reversed order
    (the ordering of hpc_gpu_port/periodic_encode.hpp:240-260);
  * the special FFT against direct evaluation of sum_k u_k zeta^{k 5^j};
  * CKKS round trips and the reference's CPU-twin verdicts (harness/cpu_real_model.cpp
    :248-268: encdec < 1e-6, rotation convention EvalRotate(ct,k)[i] == x[i+k] < 1e-4).
"""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import Oracle, derive_seed, gen_chain, load, pd, seed_bytes

LIB = load()


def test_chacha20_rfc8439_block():
    key = (C.c_uint32 * 8)(*[int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)])
    nonce = (C.c_uint32 * 3)(0x09000000, 0x4A000000, 0)
    out = (C.c_uint32 * 16)()
    LIB.oc_chacha20_block(key, 1, nonce, out)
    expect = [0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3, 0xC7F4D1C7, 0x0368C033, 0x9AAA2204, 0x4E6CD4C3,
              0x466482D2, 0x09AA9F07, 0x05D7C214, 0xA2028BD9, 0xD19C12B5, 0xB94E16DE, 0xE883D0CB, 0x4E3C50A2]
    assert list(out) == expect


def test_chain_properties():
    for logN, L in ((12, 6), (16, 20), (16, 30)):
        q, p = gen_chain(logN, L, 60, 45, 4, 60, LIB)
        M = 2 << logN
        allm = [int(x) for x in q] + [int(x) for x in p]
        assert len(set(allm)) == len(allm)
        for x in allm:
            assert LIB.oc_is_prime(x) and x % M == 1
        assert int(q[0]).bit_length() == 60 and all(int(x).bit_length() == 60 for x in p)
        assert all(abs(int(x).bit_length() - 45.5) <= 0.5 for x in q[1:])


@pytest.fixture(scope="module")
def small():
    q, p = gen_chain(12, 5, 60, 45, 2, 60, LIB)
    return Oracle(12, q, p, 2, LIB)


def _direct_ntt(a, q, psi, logN):
    N = 1 << logN
    out = []
    for i in range(N):
        br = int(format(i, f"0{logN}b")[::-1], 2)
        r = pow(psi, 2 * br + 1, q)
        out.append(sum(int(a[k]) * pow(r, k, q) for k in range(N)) % q)
    return np.array(out, dtype=np.uint64)


def test_ntt_matches_direct_evaluation():
    q, p = gen_chain(8 + 4, 2, 60, 45, 1, 60, LIB)
    o = Oracle(12, q, p, 1, LIB)
    rng = np.random.default_rng(3)
    for m in range(3):
        mod = int(o.mods[m])
        a = rng.integers(0, mod, o.N, dtype=np.uint64)
        A = o.ntt(a, m)
        psi = int(LIB.oc_root(o.ctx, m))
        assert pow(psi, o.N, mod) == mod - 1
        # spot-check 16 evaluation points against the definition
        idx = rng.integers(0, o.N, 16)
        full = None
        for i in idx:
            br = int(format(int(i), f"0{o.logN}b")[::-1], 2)
            r = pow(psi, 2 * br + 1, mod)
            v = 0
            for k in range(o.N - 1, -1, -1):
                v = (v * r + int(a[k])) % mod
            assert v == int(A[i])
        assert (o.intt(A, m) == a).all()


def test_special_fft_matches_definition():
    n, M = 64, 256
    rng = np.random.default_rng(5)
    z = rng.standard_normal(n) + 1j * rng.standard_normal(n)
    re, im = z.real.copy(), z.imag.copy()
    LIB.oc_fft_special_fwd(pd(re), pd(im), n, M)
    zeta = np.exp(2j * np.pi / M)
    rg = [pow(5, j, M) for j in range(n)]
    direct = np.array([sum(z[k] * zeta ** ((k * rg[j]) % M) for k in range(n)) for j in range(n)])
    assert np.abs(direct - (re + 1j * im)).max() < 1e-10
    LIB.oc_fft_special_inv(pd(re), pd(im), n, M)
    assert np.abs(re + 1j * im - z).max() < 1e-12


def test_automorphism_eval_matches_coefficient_form(small):
    o = small
    rng = np.random.default_rng(7)
    a = rng.integers(0, int(o.mods[1]), o.N, dtype=np.uint64)
    for k in (5, 25, 2 * o.N - 1):
        ac = np.empty_like(a)
        LIB.oc_automorph_coeff(o.ctx, a.ctypes.data_as(C.POINTER(C.c_uint64)), ac.ctypes.data_as(C.POINTER(C.c_uint64)),
                               k, 1)
        assert (o.automorph_eval(o.ntt(a, 1), k) == o.ntt(ac, 1)).all()


def _keys(o, h=64, master=11):
    ms = seed_bytes(master)
    s = o.secret(derive_seed(LIB, ms, 0xFFFFFFF1), h)
    se = o.secret_eval(s)
    pk = o.keygen_public(se, derive_seed(LIB, ms, 0xFFFFFFF0))
    return ms, s, se, pk


def test_samplers(small):
    o = small
    ms = seed_bytes(1)
    s = o.secret(derive_seed(LIB, ms, 0xFFFFFFF1), 192)
    assert np.count_nonzero(s) == 192 and set(np.unique(s)) <= {-1, 0, 1}
    e = np.empty(1 << 16, dtype=np.int32)
    LIB.oc_sample_gauss(derive_seed(LIB, ms, 5), 0, 0, 3.19, e.ctypes.data_as(C.POINTER(C.c_int32)), e.size)
    assert abs(e.mean()) < 0.05 and abs(e.std() - 3.19) < 0.05 and np.abs(e).max() <= 20


def test_ckks_roundtrips_and_ops(small):
    """The CPU-twin verdicts of harness/cpu_real_model.cpp on the oracle."""
    o = small
    ms, s, se, pk = _keys(o)
    n = o.N // 2
    rng = np.random.default_rng(2)
    z = rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)
    w = rng.uniform(-1, 1, n)
    scale = 2.0 ** 40
    pt = o.encode(z, scale, 5)
    assert np.abs(o.decode(pt, scale) - z).max() < 1e-9
    ct = o.encrypt(pk, pt, 5, derive_seed(LIB, ms, 0xFFFFFFF2, 0))
    assert np.abs(o.decode(o.decrypt(ct, 5, se), scale) - z).max() < 1e-6            # encdec < 1e-6
    ct2 = o.encrypt(pk, o.encode(w, scale, 5), 5, derive_seed(LIB, ms, 0xFFFFFFF2, 1))
    s2 = np.stack([(se[m].astype(object) ** 2 % int(o.mods[m])).astype(np.uint64) for m in range(7)])
    rlk = o.keygen_switch(s2, se, derive_seed(LIB, ms, 2))
    prod = o.ct_rescale(o.ct_mul_relin(ct, ct2, 5, rlk), 5)
    got = o.decode(o.decrypt(prod, 4, se), scale * scale / float(o.q[4]))
    assert np.abs(got - z * w).max() < 1e-6
    M = 2 * o.N
    for r in (1, 3, -2):
        k = o.rot_index(r)
        sk = np.stack([o.automorph_eval(se[m], pow(k, -1, M)) for m in range(7)])
        key = o.keygen_switch(se, sk, derive_seed(LIB, ms, k))
        rot = o.ct_automorph(ct, 5, k, key)
        got = o.decode(o.decrypt(rot, 5, se), scale)
        assert np.abs(got - np.roll(z, -r)).max() < 1e-4                               # rotate < 1e-4
    k = M - 1
    key = o.keygen_switch(se, np.stack([o.automorph_eval(se[m], k) for m in range(7)]), derive_seed(LIB, ms, k))
    got = o.decode(o.decrypt(o.ct_automorph(ct, 5, k, key), 5, se), scale)
    assert np.abs(got - np.conj(z)).max() < 1e-4


def test_keyswitch_at_lower_levels(small):
    """A key generated at the top level switches ciphertexts at every level (partial digits)."""
    o = small
    ms, s, se, pk = _keys(o)
    k = o.rot_index(1)
    sk = np.stack([o.automorph_eval(se[m], pow(k, -1, 2 * o.N)) for m in range(7)])
    key = o.keygen_switch(se, sk, derive_seed(LIB, ms, k))
    rng = np.random.default_rng(9)
    z = rng.uniform(-1, 1, o.N // 2)
    for nl in (5, 4, 3, 2, 1):
        pt = o.encode(z, 2.0 ** 40, nl)
        ct = o.encrypt(pk, pt, nl, derive_seed(LIB, ms, 0xFFFFFFF2, nl))
        rot = o.ct_automorph(ct, nl, k, key)
        got = o.decode(o.decrypt(rot, nl, se), 2.0 ** 40)
        assert np.abs(got - np.roll(z, -1)).max() < 1e-4, nl
