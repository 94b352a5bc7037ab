"""Config 2 of the baseline at its own shapes: the CKKS primitive sweep at N = 2^16.

For L in {4, 10, 20, 30} Q limbs (a 60-bit q0 and 45-bit scaling primes) with K = 4 special
primes of 60 bits and digits of alpha = 4 limbs (dnum = 1, 3, 5, 8), every result of the
engine, called through the C-ABI, must equal the CPU oracle word for word in evaluation form:
  * HMult + relinearise + rescale of two ciphertexts with uniform residues;
  * the 15 hoisted rotations by 2^0 .. 2^14, and conjugation;
  * the forward and inverse NTT over every modulus of the chain.
At L = 30 the engine's relinearisation key and one rotation key are also compared with the
oracle's keygen from the same seed.  The oracle's key switches run on all host threads (ctypes
releases the GIL).  Bytes per primitive are in the measurement notes; this file is parity only."""
from concurrent.futures import ThreadPoolExecutor
import os

import numpy as np
import pytest

from oracle_lib import Oracle, derive_seed, load

pytestmark = pytest.mark.gpu

OLIB = load()
STEPS = [1 << i for i in range(15)]


def ctx_pair(L):
    import fhessm
    cx = fhessm.CryptoContext(logN=16, L=L, K=4, alpha=4, hw=192)
    o = Oracle(16, cx.moduli[:L], cx.moduli[L:], 4, OLIB)
    cx.KeyGen(seed=100 + L)
    return cx, o


def rand_ct(o, nl, rng):
    return np.stack([np.stack([rng.integers(0, int(o.mods[i]), o.N, dtype=np.uint64) for i in range(nl)])
                     for _ in range(2)])


@pytest.mark.parametrize("L", [4, 10, 20, 30])
def test_config2_primitives_bit_exact(L):
    cx, o = ctx_pair(L)
    try:
        rng = np.random.default_rng(L)
        nthreads = os.cpu_count() or 1
        # NTT / iNTT over the whole chain (Q and P moduli)
        mods = list(range(L + 4))
        w = np.stack([rng.integers(0, int(o.mods[m]), o.N, dtype=np.uint64) for m in mods])
        f = cx.ntt(w, mods).reshape(len(mods), o.N)
        with ThreadPoolExecutor(nthreads) as ex:
            ref = list(ex.map(lambda m: o.ntt(w[m], m), mods))
        assert all((f[m] == ref[m]).all() for m in mods)
        assert (cx.ntt(f, mods, inverse=True).reshape(len(mods), o.N) == w).all()

        # HMult + relinearise + rescale at the top level
        a, b = rand_ct(o, L, rng), rand_ct(o, L, rng)
        prod = cx.EvalMult(cx.ct_from_words(a, 0), cx.ct_from_words(b, 0))
        rlk = cx.key_words(0)
        want = o.ct_mul_relin(a, b, L, rlk)
        assert (prod.words() == want).all(), "HMult + relinearise"
        cx.RescaleInPlace(prod)
        assert (prod.words() == o.ct_rescale(want, L)).all(), "rescale"
        del rlk

        # 15 hoisted power-of-two rotations and conjugation of one ciphertext at the top level
        cx.EvalRotateKeyGen(STEPS, conj=True)
        ca = cx.ct_from_words(a, 0)
        got = [h.words() for h in cx.EvalFastRotation(ca, STEPS)]
        conj = cx.EvalConj(ca).words()
        ks = [cx.rot_index(r) for r in STEPS] + [2 * o.N - 1]
        outs = got + [conj]

        def check(i):
            k = ks[i]
            return bool((outs[i] == o.ct_automorph(a, L, k, cx.key_words(k))).all())

        with ThreadPoolExecutor(min(nthreads, 4)) as ex:   # each call holds one key (up to 272 MiB)
            ok = list(ex.map(check, range(len(ks))))
        assert all(ok), [s for s, g in zip(STEPS + ["conj"], ok) if not g]

        if L == 30:
            # the keys themselves, from the same seed
            ms = (100 + L).to_bytes(8, "little") + bytes(24)
            se = o.secret_eval(cx.secret_coeffs())
            s2 = np.stack([(se[m].astype(object) ** 2 % int(o.mods[m])).astype(np.uint64) for m in range(len(o.mods))])
            assert (cx.key_words(0) == o.keygen_switch(s2, se, derive_seed(OLIB, ms, 2))).all(), "relinearisation key"
            k = cx.rot_index(1 << 14)
            sk = np.stack([o.automorph_eval(se[m], pow(k, -1, 2 * o.N)) for m in range(len(o.mods))])
            assert (cx.key_words(k) == o.keygen_switch(se, sk, derive_seed(OLIB, ms, k))).all(), "rotation key"
    finally:
        cx.close()
