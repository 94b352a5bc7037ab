"""The oracle pinned to the reference's own code (CPU).

tests/golden/ref_vectors.json holds outputs of the reference's seeded-key expander
(hpc_gpu_port/seeded_keys.hpp:80-134: ChaCha20 block, SeedStream, fillUniformMod) and of its
periodic encoder's NTT with its root table (hpc_gpu_port/periodic_encode.hpp:102-120, :150-160,
:241-260), made by tests/golden/make_ref_vectors.py from those lines compiled where they lie in
the reference tree (oracle/ref_extract.sh).  The oracle must reproduce every word.  Where the
compiled reference is present (oracle/_ref/libref_pins.so), fresh random cases are compared
live as well.  The engine is held to the oracle by the GPU tests (keys, NTT, periodic encode),
which closes the chain reference == oracle == engine for these two pieces."""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle_lib import U64P, load, p64

GOLD = json.load(open(os.path.join(ROOT, "tests", "golden", "ref_vectors.json")))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_pins.so")
TAG_SKEY = 0x59454B53


def seed_bytes(i):
    return bytes((7 * i + 3 * k) % 256 for k in range(32))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<u8").tobytes()).hexdigest()


@pytest.fixture(scope="module")
def lib():
    return load()


def oracle_expand(lib, seed, digit, limb, q, n):
    w = np.empty(n, dtype=np.uint64)
    lib.oc_sample_uniform(seed, digit, limb, TAG_SKEY, q, p64(w), n)
    return w


def oracle_periodic_ntt(lib, q, psi, log_n, log_rep, a):
    a = np.ascontiguousarray(a, dtype=np.uint64).copy()
    lib.oc_ntt_root(log_n - log_rep, q, pow(psi, 1 << log_rep, q), p64(a))
    return a


def test_chacha_block_matches_reference(lib):
    for c in GOLD["chacha"]:
        key = (C.c_uint32 * 8)(*[int.from_bytes(seed_bytes(c["key_seed_case"])[4 * k:4 * k + 4], "little")
                                 for k in range(8)])
        o = (C.c_uint32 * 16)()
        lib.oc_chacha20_block(key, c["counter"], (C.c_uint32 * 3)(*c["nonce"]), o)
        assert list(o) == c["out"]


def test_key_a_half_expansion_matches_reference(lib):
    """Every word of the a-half stream for (seed, digit, limb) over 45-, 58- and 60-bit moduli."""
    for c in GOLD["expand"]:
        w = oracle_expand(lib, seed_bytes(c["seed_case"]), c["digit"], c["limb"], c["q"], c["n"])
        assert [int(x) for x in w[:16]] == c["head"]
        assert sha(w) == c["sha256"], f"case {c['seed_case']}: a-half words differ from the reference expander"


def test_ntt_matches_reference_periodic_encoder(lib):
    """The oracle's Cooley-Tukey transform with the reference's ordering equals the reference's own
    transform at ring 2^16 and at the small rings of the periodic encoder (root psi^REP)."""
    for c in GOLD["ntt"]:
        n = 1 << (c["logN"] - c["logRep"])
        a = np.random.default_rng(c["input_seed"]).integers(0, c["q"], n, dtype=np.uint64)
        got = oracle_periodic_ntt(lib, c["q"], c["psi"], c["logN"], c["logRep"], a)
        assert [int(x) for x in got[:16]] == c["head"]
        assert sha(got) == c["sha256"], f"q={c['q']} logRep={c['logRep']}: NTT words differ from the reference"


def test_oracle_context_ntt_is_the_pinned_transform(lib):
    """oc_ntt (the context's transform, used by every oracle routine) equals oc_ntt_root with the
    context's root, so the pin above covers the oracle's key-switch, rescale and encode paths."""
    from oracle_lib import Oracle, gen_chain
    q, p = gen_chain(16, 4, 60, 45, 1, 60, lib)
    o = Oracle(16, q, p, 4, lib)
    for m in range(len(q)):
        a = np.random.default_rng(m).integers(0, int(q[m]), 1 << 16, dtype=np.uint64)
        b = a.copy()
        lib.oc_ntt(o.ctx, p64(a), m)
        lib.oc_ntt_root(16, int(q[m]), int(lib.oc_root(o.ctx, m)), p64(b))
        assert (a == b).all()


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="the reference's code is not compiled here (oracle/_ref)")
def test_live_against_compiled_reference(lib):
    ref = C.CDLL(REF_SO)
    ref.ref_expand_a.argtypes = [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint64, U64P, C.c_size_t]
    ref.ref_periodic_ntt.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32, U64P]
    from oracle_lib import gen_chain
    q, p = gen_chain(16, 12, 60, 45, 4, 60, lib)
    mods = [int(x) for x in q] + [int(x) for x in p]
    rng = np.random.default_rng(2024)
    for _ in range(12):
        seed = bytes(rng.integers(0, 256, 32, dtype=np.uint8))
        digit, limb = int(rng.integers(0, 6)), int(rng.integers(0, len(mods)))
        qq = mods[limb]
        w = np.empty(4096, dtype=np.uint64)
        ref.ref_expand_a(seed, digit, limb, qq, w.ctypes.data_as(U64P), 4096)
        assert (oracle_expand(lib, seed, digit, limb, qq, 4096) == w).all()
    for log_rep in (0, 3, 6, 10):
        qq = mods[int(rng.integers(0, len(mods)))]
        psi = int(lib.oc_min_root(qq, 16))
        a = rng.integers(0, qq, 1 << (16 - log_rep), dtype=np.uint64)
        r = a.copy()
        ref.ref_periodic_ntt(qq, psi, 16, log_rep, r.ctypes.data_as(U64P))
        assert (oracle_periodic_ntt(lib, qq, psi, 16, log_rep, a) == r).all()
