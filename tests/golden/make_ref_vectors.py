#!/usr/bin/env python3
"""Writes tests/golden/ref_vectors.json from the reference's own code.

Runs oracle/_ref/libref_pins.so (oracle/ref_extract.sh: the reference's seeded-key expander,
hpc_gpu_port/seeded_keys.hpp:80-134, and its periodic encoder's NTT with root table,
hpc_gpu_port/periodic_encode.hpp:102-120, :150-160, :241-260, compiled where they lie in the
reference tree) on fixed inputs and records the outputs, so that tests/test_ref_pins.py can hold the
oracle to them on machines without the reference.  Moduli come from the oracle's chain rule; the
roots are the minimal primitive 2N-th roots (OpenFHE's RootOfUnity choice), given to both sides.

    python tests/golden/make_ref_vectors.py <reference root>
"""
import ctypes as C
import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
U64P = C.POINTER(C.c_uint64)


def seed_bytes(i):
    """The 32-byte seed of case i: bytes (7 i + 3 k) mod 256, k = 0..31."""
    return bytes((7 * i + 3 * k) % 256 for k in range(32))


def input_words(seed, q, n):
    return np.random.default_rng(seed).integers(0, q, n, dtype=np.uint64)


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<u8").tobytes()).hexdigest()


def moduli(lib):
    from oracle_lib import gen_chain
    q, p = gen_chain(16, 20, 60, 45, 4, 60, lib)
    qb, _ = gen_chain(16, 3, 60, 58, 1, 60, lib)
    return [int(q[0]), int(q[1]), int(q[7]), int(q[19]), int(p[0]), int(p[3]), int(qb[2])]


def main(ref_root):
    from oracle_lib import load
    lib = load()
    subprocess.run(["sh", os.path.join(ROOT, "oracle", "ref_extract.sh"), ref_root,
                    os.path.join(ROOT, "oracle", "_ref")], check=True)
    ref = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_pins.so"))
    ref.ref_expand_a.argtypes = [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint64, U64P, C.c_size_t]
    ref.ref_periodic_ntt.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32, U64P]
    ref.ref_chacha20_block.argtypes = [C.POINTER(C.c_uint32), C.c_uint32, C.POINTER(C.c_uint32),
                                       C.POINTER(C.c_uint32)]
    mods = moduli(lib)
    out = {"about": "outputs of the reference's own seeded-key expander and periodic-encoder NTT "
                    "(tests/golden/make_ref_vectors.py)", "chacha": [], "expand": [], "ntt": []}
    for i, (ctr, nonce) in enumerate([(1, (0x09000000, 0x4a000000, 0)), (7, (3, 11, 0x59454b53))]):
        key = (C.c_uint32 * 8)(*[int.from_bytes(seed_bytes(i)[4 * k:4 * k + 4], "little") for k in range(8)])
        o = (C.c_uint32 * 16)()
        ref.ref_chacha20_block(key, ctr, (C.c_uint32 * 3)(*nonce), o)
        out["chacha"].append({"key_seed_case": i, "counter": ctr, "nonce": list(nonce), "out": list(o)})
    n = 1 << 16
    for i, (digit, limb, q) in enumerate([(0, 0, mods[0]), (0, 19, mods[3]), (1, 7, mods[2]), (4, 20, mods[4]),
                                          (2, 23, mods[5]), (3, 2, mods[6]), (0, 1, mods[1])]):
        w = np.empty(n, dtype=np.uint64)
        ref.ref_expand_a(seed_bytes(i), digit, limb, q, w.ctypes.data_as(U64P), n)
        out["expand"].append({"seed_case": i, "digit": digit, "limb": limb, "q": q, "n": n,
                              "head": [int(x) for x in w[:16]], "sha256": sha(w)})
    for i, (q, log_rep) in enumerate([(mods[0], 0), (mods[3], 0), (mods[1], 5), (mods[4], 5), (mods[6], 5),
                                      (mods[2], 9)]):
        psi = int(lib.oc_min_root(q, 16))
        a = input_words(1000 + i, q, n >> log_rep)
        ref.ref_periodic_ntt(q, psi, 16, log_rep, a.ctypes.data_as(U64P))
        out["ntt"].append({"q": q, "psi": psi, "logN": 16, "logRep": log_rep, "input_seed": 1000 + i,
                           "head": [int(x) for x in a[:16]], "sha256": sha(a)})
    with open(os.path.join(HERE, "ref_vectors.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "ref_vectors.json"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FHESSM_REFERENCE", ""))
