"""ctypes view of the CPU oracle (oracle/liboracle.so) for the tests.

Test infrastructure: the oracle is the checker for the CUDA engine and is never part of
the product path.  Arrays are numpy uint64 in the layouts documented in
oracle/fhe_oracle.h ([poly][limb][N] for ciphertexts, [digit][2][nq+np][N] for keys).
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
LIB_PATH = os.path.join(ORACLE_DIR, "liboracle.so")

U64P = C.POINTER(C.c_uint64)


def _build():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


def load():
    src = os.path.join(ORACLE_DIR, "fhe_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        _build()
    lib = C.CDLL(LIB_PATH)
    sig = {
        "oc_mulmod": (C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64]),
        "oc_powmod": (C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64]),
        "oc_is_prime": (C.c_int, [C.c_uint64]),
        "oc_gen_chain": (C.c_int, [C.c_int] * 6 + [U64P, U64P]),
        "oc_min_root": (C.c_uint64, [C.c_uint64, C.c_int]),
        "oc_ctx_new": (C.c_void_p, [C.c_int, C.c_int, U64P, C.c_int, U64P, C.c_int]),
        "oc_ctx_free": (None, [C.c_void_p]),
        "oc_modulus": (C.c_uint64, [C.c_void_p, C.c_int]),
        "oc_root": (C.c_uint64, [C.c_void_p, C.c_int]),
        "oc_ntt": (None, [C.c_void_p, U64P, C.c_int]),
        "oc_intt": (None, [C.c_void_p, U64P, C.c_int]),
        "oc_ntt_root": (None, [C.c_int, C.c_uint64, C.c_uint64, U64P]),
        "oc_automorph_eval": (None, [C.c_void_p, U64P, U64P, C.c_uint64]),
        "oc_automorph_coeff": (None, [C.c_void_p, U64P, U64P, C.c_uint64, C.c_int]),
        "oc_rot_index": (C.c_uint64, [C.c_int, C.c_int64]),
        "oc_rescale": (None, [C.c_void_p, U64P, C.c_int, U64P]),
        "oc_modup": (None, [C.c_void_p, U64P, C.c_int, U64P]),
        "oc_moddown": (None, [C.c_void_p, U64P, C.c_int, U64P]),
        "oc_key_inner": (None, [C.c_void_p, U64P, C.c_int, U64P, U64P, U64P]),
        "oc_keyswitch": (None, [C.c_void_p, U64P, C.c_int, U64P, U64P, U64P]),
        "oc_ks_part_ext": (None, [C.c_void_p, U64P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, U64P]),
        "oc_ks_part_inner": (None, [C.c_void_p, U64P, C.c_int, U64P, C.c_int, C.c_int, C.c_int, C.c_int, U64P, U64P]),
        "oc_ks_part_moddown": (None, [C.c_void_p, U64P, U64P, C.c_int, C.c_int, C.c_int, U64P]),
        "oc_ct_add": (None, [C.c_void_p, U64P, U64P, C.c_int, U64P]),
        "oc_ct_mul_pt": (None, [C.c_void_p, U64P, U64P, C.c_int, U64P]),
        "oc_ct_mul_relin": (None, [C.c_void_p, U64P, U64P, C.c_int, U64P, U64P]),
        "oc_ct_rescale": (None, [C.c_void_p, U64P, C.c_int, U64P]),
        "oc_ct_automorph": (None, [C.c_void_p, U64P, C.c_int, C.c_uint64, U64P, U64P]),
        "oc_chacha20_block": (None, [C.POINTER(C.c_uint32), C.c_uint32, C.POINTER(C.c_uint32), C.POINTER(C.c_uint32)]),
        "oc_sample_uniform": (None, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, U64P, C.c_int]),
        "oc_sample_ternary_hw": (None, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_int, C.POINTER(C.c_int8), C.c_int]),
        "oc_sample_ternary": (None, [C.c_char_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_int8), C.c_int]),
        "oc_sample_gauss": (None, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_double, C.POINTER(C.c_int32), C.c_int]),
        "oc_derive_seed": (None, [C.c_char_p, C.c_uint32, C.c_uint32, C.c_char_p]),
        "oc_secret_eval": (None, [C.c_void_p, C.POINTER(C.c_int8), U64P]),
        "oc_keygen_switch": (None, [C.c_void_p, U64P, U64P, C.c_char_p, C.c_double, U64P]),
        "oc_keygen_public": (None, [C.c_void_p, U64P, C.c_char_p, C.c_double, U64P]),
        "oc_encrypt": (None, [C.c_void_p, U64P, U64P, C.c_int, C.c_char_p, C.c_double, U64P]),
        "oc_decrypt": (None, [C.c_void_p, U64P, C.c_int, U64P, U64P]),
        "oc_fft_special_inv": (None, [C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int, C.c_int]),
        "oc_fft_special_fwd": (None, [C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_int, C.c_int]),
        "oc_encode": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_double), C.c_double, C.c_int, U64P]),
        "oc_decode": (None, [C.c_void_p, U64P, C.c_double, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


def p64(a):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(U64P)


def pd(a):
    assert a.dtype == np.float64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.POINTER(C.c_double))


class Oracle:
    """A ring + moduli context of the oracle with numpy-friendly methods."""

    def __init__(self, logN, q, p, alpha, lib=None):
        self.lib = lib or load()
        self.logN, self.N = logN, 1 << logN
        self.q = np.ascontiguousarray(q, dtype=np.uint64)
        self.p = np.ascontiguousarray(p, dtype=np.uint64)
        self.nq, self.np_, self.alpha = len(self.q), len(self.p), alpha
        self.ctx = self.lib.oc_ctx_new(logN, self.nq, p64(self.q), self.np_, p64(self.p), alpha)
        self.mods = np.concatenate([self.q, self.p])

    def __del__(self):
        try:
            self.lib.oc_ctx_free(self.ctx)
        except Exception:
            pass

    def dnum(self, nl):
        return (nl + self.alpha - 1) // self.alpha

    def ntt(self, a, m):
        a = np.ascontiguousarray(a, dtype=np.uint64).copy()
        self.lib.oc_ntt(self.ctx, p64(a), m)
        return a

    def intt(self, a, m):
        a = np.ascontiguousarray(a, dtype=np.uint64).copy()
        self.lib.oc_intt(self.ctx, p64(a), m)
        return a

    def automorph_eval(self, a, k):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        out = np.empty_like(a)
        self.lib.oc_automorph_eval(self.ctx, p64(a), p64(out), k)
        return out

    def rot_index(self, r):
        return self.lib.oc_rot_index(self.logN, r)

    def rescale(self, a, nl):
        a = np.ascontiguousarray(a, dtype=np.uint64)
        out = np.empty(((nl - 1) * self.N,), dtype=np.uint64)
        self.lib.oc_rescale(self.ctx, p64(a), nl, p64(out))
        return out.reshape(nl - 1, self.N)

    def modup(self, d, nl):
        d = np.ascontiguousarray(d, dtype=np.uint64)
        out = np.empty((self.dnum(nl), nl + self.np_, self.N), dtype=np.uint64)
        self.lib.oc_modup(self.ctx, p64(d), nl, p64(out))
        return out

    def moddown(self, x, nl):
        x = np.ascontiguousarray(x, dtype=np.uint64)
        out = np.empty((nl, self.N), dtype=np.uint64)
        self.lib.oc_moddown(self.ctx, p64(x), nl, p64(out))
        return out

    def key_inner(self, ext, nl, key):
        o0 = np.empty((nl + self.np_, self.N), dtype=np.uint64)
        o1 = np.empty_like(o0)
        self.lib.oc_key_inner(self.ctx, p64(np.ascontiguousarray(ext)), nl, p64(key), p64(o0), p64(o1))
        return o0, o1

    def keyswitch(self, d, nl, key):
        o0 = np.empty((nl, self.N), dtype=np.uint64)
        o1 = np.empty_like(o0)
        self.lib.oc_keyswitch(self.ctx, p64(np.ascontiguousarray(d)), nl, p64(key), p64(o0), p64(o1))
        return o0, o1

    def ct_mul_relin(self, a, b, nl, rlk):
        out = np.empty((2, nl, self.N), dtype=np.uint64)
        self.lib.oc_ct_mul_relin(self.ctx, p64(np.ascontiguousarray(a)), p64(np.ascontiguousarray(b)), nl,
                                 p64(rlk), p64(out))
        return out

    def ct_rescale(self, a, nl):
        out = np.empty((2, nl - 1, self.N), dtype=np.uint64)
        self.lib.oc_ct_rescale(self.ctx, p64(np.ascontiguousarray(a)), nl, p64(out))
        return out

    def ct_mul_pt(self, a, pt, nl):
        out = np.empty((2, nl, self.N), dtype=np.uint64)
        self.lib.oc_ct_mul_pt(self.ctx, p64(np.ascontiguousarray(a)), p64(np.ascontiguousarray(pt)), nl, p64(out))
        return out

    def ct_add(self, a, b, nl):
        out = np.empty((2, nl, self.N), dtype=np.uint64)
        self.lib.oc_ct_add(self.ctx, p64(np.ascontiguousarray(a)), p64(np.ascontiguousarray(b)), nl, p64(out))
        return out

    def ct_automorph(self, a, nl, k, key):
        out = np.empty((2, nl, self.N), dtype=np.uint64)
        self.lib.oc_ct_automorph(self.ctx, p64(np.ascontiguousarray(a)), nl, k, p64(key), p64(out))
        return out

    # ---- keys / encryption ----
    def secret(self, seed32, h):
        s = np.empty(self.N, dtype=np.int8)
        self.lib.oc_sample_ternary_hw(seed32, 0, 0, h, s.ctypes.data_as(C.POINTER(C.c_int8)), self.N)
        return s

    def secret_eval(self, s):
        out = np.empty((self.nq + self.np_, self.N), dtype=np.uint64)
        self.lib.oc_secret_eval(self.ctx, np.ascontiguousarray(s).ctypes.data_as(C.POINTER(C.c_int8)), p64(out))
        return out

    def keygen_switch(self, s_src_eval, s_key_eval, seed32, sigma=3.19):
        out = np.empty((self.dnum(self.nq), 2, self.nq + self.np_, self.N), dtype=np.uint64)
        self.lib.oc_keygen_switch(self.ctx, p64(np.ascontiguousarray(s_src_eval)), p64(np.ascontiguousarray(s_key_eval)),
                                  seed32, sigma, p64(out))
        return out

    def keygen_public(self, s_eval, seed32, sigma=3.19):
        out = np.empty((2, self.nq, self.N), dtype=np.uint64)
        self.lib.oc_keygen_public(self.ctx, p64(np.ascontiguousarray(s_eval)), seed32, sigma, p64(out))
        return out

    def encrypt(self, pk, pt, nl, seed32, sigma=3.19):
        out = np.empty((2, nl, self.N), dtype=np.uint64)
        self.lib.oc_encrypt(self.ctx, p64(np.ascontiguousarray(pk)), p64(np.ascontiguousarray(pt)), nl, seed32, sigma,
                            p64(out))
        return out

    def decrypt(self, ct, nl, s_eval):
        out = np.empty((nl, self.N), dtype=np.uint64)
        self.lib.oc_decrypt(self.ctx, p64(np.ascontiguousarray(ct)), nl, p64(np.ascontiguousarray(s_eval[:nl])),
                            p64(out))
        return out

    def encode(self, z, scale, nl):
        z = np.asarray(z, dtype=np.complex128)
        re = np.ascontiguousarray(z.real)
        im = np.ascontiguousarray(z.imag)
        out = np.empty((nl, self.N), dtype=np.uint64)
        rc = self.lib.oc_encode(self.ctx, pd(re), pd(im), scale, nl, p64(out))
        if rc:
            raise ValueError(f"encode failed: {rc}")
        return out

    def decode(self, pt, scale):
        re = np.empty(self.N // 2)
        im = np.empty(self.N // 2)
        self.lib.oc_decode(self.ctx, p64(np.ascontiguousarray(pt[0])), scale, pd(re), pd(im))
        return re + 1j * im


def gen_chain(logN, L, q0bits=60, qbits=45, K=4, pbits=60, lib=None):
    lib = lib or load()
    q = np.zeros(L, dtype=np.uint64)
    p = np.zeros(K, dtype=np.uint64)
    rc = lib.oc_gen_chain(logN, L, q0bits, qbits, K, pbits, p64(q), p64(p))
    assert rc == 0
    return q, p


def seed_bytes(master: int) -> bytes:
    """32-byte master seed from a 64-bit integer (little-endian, zero padded)."""
    return int(master).to_bytes(8, "little") + bytes(24)


def derive_seed(lib, master32: bytes, ident: int, sub: int = 0) -> bytes:
    out = C.create_string_buffer(32)
    lib.oc_derive_seed(master32, ident, sub, out)
    return out.raw
