"""fhessm -- Python binding of the B200 CKKS evaluation engine (libfhessm.so, C-ABI in
include/fhessm.h).

The class ``CryptoContext`` mirrors the OpenFHE CryptoContext calls that the reference's
server makes on its hot path (hpc_gpu_port/gpu_real_model.cu: KeyGen/EvalMultKeyGen
:1293-1298, EvalRotateKeyGen :1299-1336, MakeCKKSPackedPlaintext :1577-1589,
Encrypt/Decrypt :2202-2221, EvalMult + RescaleInPlace :2629-2632, EvalAdd :2692-2743,
EvalRotate :2762-2765), with the same argument meaning: levels count consumed levels,
rotation k moves slot i+k to slot i.  Errors raise ``FheError`` carrying the engine's
status code and message; nothing falls back to another implementation.  The CUDA library
must be built (``python -c "import __graft_entry__ as g; g.build()"``); importing this
package on a machine without it raises.
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfhessm.so")

_U64P = C.POINTER(C.c_uint64)
_DP = C.POINTER(C.c_double)
_VP = C.c_void_p


class FheError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class Params(C.Structure):
    _fields_ = [("logN", C.c_int), ("L", C.c_int), ("K", C.c_int), ("alpha", C.c_int),
                ("q0bits", C.c_int), ("qbits", C.c_int), ("pbits", C.c_int), ("hw", C.c_int),
                ("sigma", C.c_double), ("device", C.c_int), ("boot_primes", C.c_int), ("boot_bits", C.c_int)]


_SIGS = {
    "fhe_last_error": (C.c_char_p, []),
    "fhe_ctx_create": (C.c_int, [C.POINTER(Params), C.POINTER(_VP)]),
    "fhe_ctx_destroy": (None, [_VP]),
    "fhe_ctx_moduli": (C.c_int, [_VP, _U64P]),
    "fhe_ctx_scale": (C.c_double, [_VP, C.c_int]),
    "fhe_ctx_sync": (C.c_int, [_VP]),
    "fhe_ctx_launches": (C.c_longlong, [_VP]),
    "fhe_ctx_stream": (_VP, [_VP]),
    "fhe_prof_enable": (C.c_int, [_VP, C.c_int]),
    "fhe_prof_collect": (C.c_int, [_VP, C.c_char_p, C.c_int]),
    "fhe_keygen": (C.c_int, [_VP, C.c_char_p]),
    "fhe_keygen_rotations": (C.c_int, [_VP, C.POINTER(C.c_int32), C.c_int, C.c_int]),
    "fhe_key_export": (C.c_int, [_VP, C.c_uint64, _U64P]),
    "fhe_key_import": (C.c_int, [_VP, C.c_uint64, _U64P]),
    "fhe_secret_export": (C.c_int, [_VP, C.POINTER(C.c_int8)]),
    "fhe_pubkey_export": (C.c_int, [_VP, _U64P]),
    "fhe_rot_index": (C.c_uint64, [_VP, C.c_int32]),
    "fhe_encode": (C.c_int, [_VP, _DP, _DP, C.c_int, C.c_int, C.c_double, C.POINTER(_VP)]),
    "fhe_decode": (C.c_int, [_VP, _VP, _DP, _DP]),
    "fhe_encode_periodic": (C.c_int, [_VP, _DP, _DP, C.c_int, C.c_int, C.c_int, C.c_double, _U64P]),
    "fhe_pt_free": (None, [_VP]),
    "fhe_pt_level": (C.c_int, [_VP]),
    "fhe_encrypt": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "fhe_decrypt": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "fhe_ct_free": (None, [_VP]),
    "fhe_ct_level": (C.c_int, [_VP]),
    "fhe_ct_scale": (C.c_double, [_VP]),
    "fhe_ct_copy": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "fhe_mul_ct_pt": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_mul_ct_ct_relin": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_add": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_sub": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_add_pt": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_mul_const": (C.c_int, [_VP, _VP, C.c_double, C.c_double, C.POINTER(_VP)]),
    "fhe_add_const": (C.c_int, [_VP, _VP, C.c_double, C.POINTER(_VP)]),
    "fhe_rescale": (C.c_int, [_VP, _VP]),
    "fhe_level_reduce": (C.c_int, [_VP, _VP, C.c_int]),
    "fhe_rotate": (C.c_int, [_VP, _VP, C.c_int32, C.POINTER(_VP)]),
    "fhe_rotate_hoisted": (C.c_int, [_VP, _VP, C.POINTER(C.c_int32), C.c_int, C.POINTER(_VP)]),
    "fhe_rotate_sum": (C.c_int, [_VP, C.POINTER(_VP), C.POINTER(C.c_int32), C.c_int, C.POINTER(_VP)]),
    "fhe_ctx_set_option": (C.c_int, [_VP, C.c_char_p, C.c_int]),
    "fhe_conjugate": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "fhe_mul_vec_rescale": (C.c_int, [_VP, _VP, _DP, _DP, C.c_int, C.POINTER(_VP)]),
    "fhe_align": (C.c_int, [_VP, _VP, C.c_int]),
    "fhe_mul_rescale": (C.c_int, [_VP, _VP, _VP, C.POINTER(_VP)]),
    "fhe_poly_eval": (C.c_int, [_VP, _VP, _DP, C.c_int, C.c_int, C.POINTER(_VP)]),
    "fhe_cheb_eval": (C.c_int, [_VP, _VP, _DP, C.c_int, C.POINTER(_VP)]),
    "fhe_cheb_eval_n": (C.c_int, [_VP, C.POINTER(_VP), C.c_int, _DP, C.c_int, C.POINTER(_VP)]),
    "fhe_cheb_depth": (C.c_int, [_DP, C.c_int, C.POINTER(C.c_int)]),
    "fhe_bootstrap_setup": (C.c_int, [_VP, C.c_double, C.c_int]),
    "fhe_bootstrap_setup_r": (C.c_int, [_VP, C.c_double, C.c_int, C.c_int]),
    "fhe_bootstrap": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "fhe_bootstrap_level": (C.c_int, [_VP]),
    "fhe_matvec_plan": (C.c_int, [_VP, _DP, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_VP)]),
    "fhe_mvplan_free": (None, [_VP]),
    "fhe_matvec_keygen": (C.c_int, [_VP, C.c_int, C.c_int]),
    "fhe_matvec_bsgs": (C.c_int, [_VP, _VP, C.POINTER(_VP), C.c_int, C.POINTER(_VP)]),
    "fhe_ct_import": (C.c_int, [_VP, _U64P, C.c_int, C.c_double, C.POINTER(_VP)]),
    "fhe_ct_export": (C.c_int, [_VP, _VP, _U64P]),
    "fhe_pt_import": (C.c_int, [_VP, _U64P, C.c_int, C.c_double, C.POINTER(_VP)]),
    "fhe_pt_export": (C.c_int, [_VP, _VP, _U64P]),
    "fhe_ntt_host": (C.c_int, [_VP, _U64P, C.c_int, C.POINTER(C.c_int), C.c_int]),
    "fhe_keyswitch_host": (C.c_int, [_VP, _U64P, C.c_int, _U64P, _U64P, _U64P]),
}

_lib_handle = None


def lib():
    """The loaded CUDA engine.  Raises if libfhessm.so has not been built."""
    global _lib_handle
    if _lib_handle is None:
        if not os.path.exists(LIB_PATH):
            raise FheError(-1, f"libfhessm.so not built at {LIB_PATH}: run __graft_entry__.build()")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib_handle = h
    return _lib_handle


def _check(rc):
    if rc != 0:
        raise FheError(rc, lib().fhe_last_error().decode())


def _u64(a):
    a = np.ascontiguousarray(a, dtype=np.uint64)
    return a, a.ctypes.data_as(_U64P)


class Plaintext:
    def __init__(self, ctx, h):
        self.ctx, self.h = ctx, h

    def __del__(self):
        try:
            # a handle outliving its closed context is dropped (its memory went with the context)
            if getattr(self, "h", None) and getattr(self.ctx, "h", None):
                lib().fhe_pt_free(self.h)
            self.h = None
        except (TypeError, AttributeError):   # module globals already torn down at interpreter exit
            pass

    @property
    def level(self):
        return lib().fhe_pt_level(self.h)


class Ciphertext:
    def __init__(self, ctx, h):
        self.ctx, self.h = ctx, h

    def __del__(self):
        try:
            if getattr(self, "h", None) and getattr(self.ctx, "h", None):
                lib().fhe_ct_free(self.h)
            self.h = None
        except (TypeError, AttributeError):   # module globals already torn down at interpreter exit
            pass

    @property
    def level(self):
        return lib().fhe_ct_level(self.h)

    @property
    def scale(self):
        return lib().fhe_ct_scale(self.h)

    def words(self):
        nl = self.ctx.L - self.level
        out = np.empty((2, nl, self.ctx.N), dtype=np.uint64)
        _check(lib().fhe_ct_export(self.ctx.h, self.h, out.ctypes.data_as(_U64P)))
        return out


class _MvPlan:
    def __init__(self, h, ctx=None):
        self.h, self.ctx = h, ctx

    def __del__(self):
        try:
            if getattr(self, "h", None) and (self.ctx is None or getattr(self.ctx, "h", None)):
                lib().fhe_mvplan_free(self.h)
            self.h = None
        except (TypeError, AttributeError):   # module globals already torn down at interpreter exit
            pass


def seed32(seed) -> bytes:
    """32-byte seed from an int (little-endian, zero padded) or bytes."""
    if isinstance(seed, (bytes, bytearray)):
        assert len(seed) == 32
        return bytes(seed)
    return int(seed).to_bytes(8, "little") + bytes(24)


class PartLayout(C.Structure):
    """fhe_part_layout: the header fields of a seeded key part file (FSSMSKY1)."""
    _fields_ = [(k, C.c_uint32) for k in ("version", "expander", "N", "sizeQ", "sizeP", "numPartQ", "numPerPartQ",
                                          "count")]


def part_header(path):
    """Header of a seeded key part file (no GPU needed): (layout dict, moduli, key tag)."""
    h = lib()
    h.fhe_part_header.restype = C.c_int
    h.fhe_part_header.argtypes = [C.c_char_p, C.POINTER(PartLayout), _U64P, C.c_int, C.c_char_p, C.c_int]
    lay = PartLayout()
    mods = np.zeros(256, dtype=np.uint64)
    tag = C.create_string_buffer(4097)
    _check(h.fhe_part_header(path.encode(), C.byref(lay), mods.ctypes.data_as(_U64P), 256, tag, len(tag)))
    d = {k: getattr(lay, k) for k, _ in PartLayout._fields_}
    return d, mods[:d["sizeQ"] + d["sizeP"]].copy(), tag.value.decode()


def write_part_words(path, layout, moduli, tag, indices, seeds, b):
    """A seeded key part file from caller-held words (no GPU needed): layout dict (N, sizeQ, sizeP,
    numPartQ, numPerPartQ), indices (count,), seeds (count, 32) uint8, b (count, numPartQ,
    sizeQ + sizeP, N) uint64."""
    h = lib()
    h.fhe_part_write_words.restype = C.c_int
    h.fhe_part_write_words.argtypes = [C.c_char_p, C.POINTER(PartLayout), _U64P, C.c_char_p,
                                       C.POINTER(C.c_uint32), C.POINTER(C.c_uint8), _U64P]
    idx = np.ascontiguousarray(indices, dtype=np.uint32)
    sd = np.ascontiguousarray(seeds, dtype=np.uint8)
    bw = np.ascontiguousarray(b, dtype=np.uint64)
    mods = np.ascontiguousarray(moduli, dtype=np.uint64)
    lay = PartLayout(1, 1, layout["N"], layout["sizeQ"], layout["sizeP"], layout["numPartQ"], layout["numPerPartQ"],
                     len(idx))
    _check(h.fhe_part_write_words(path.encode(), C.byref(lay), mods.ctypes.data_as(_U64P), tag.encode(),
                                  idx.ctypes.data_as(C.POINTER(C.c_uint32)), sd.ctypes.data_as(C.POINTER(C.c_uint8)),
                                  bw.ctypes.data_as(_U64P)))


class CryptoContext:
    """One engine context (one GPU).  Names follow the OpenFHE calls of the reference."""

    def __init__(self, logN=16, L=20, K=4, alpha=4, q0bits=60, qbits=45, pbits=60, hw=192, sigma=3.19, device=0,
                 boot_primes=0, boot_bits=58):
        self.p = Params(logN, L, K, alpha, q0bits, qbits, pbits, hw, sigma, device, boot_primes, boot_bits)
        h = _VP()
        _check(lib().fhe_ctx_create(C.byref(self.p), C.byref(h)))
        self.h = h
        self.logN, self.N, self.L, self.K, self.alpha = logN, 1 << logN, L, K, alpha
        self.slots = self.N // 2
        self.dnum = (L + alpha - 1) // alpha
        m = np.empty(L + K, dtype=np.uint64)
        _check(lib().fhe_ctx_moduli(self.h, m.ctypes.data_as(_U64P)))
        self.moduli = m

    def close(self):
        if getattr(self, "h", None):
            lib().fhe_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except (TypeError, AttributeError):   # module globals already torn down at interpreter exit
            pass

    # ---- context info
    def GetScalingFactorReal(self, level):
        return lib().fhe_ctx_scale(self.h, level)

    def sync(self):
        _check(lib().fhe_ctx_sync(self.h))

    def launches(self):
        return lib().fhe_ctx_launches(self.h)

    def rot_index(self, k):
        return lib().fhe_rot_index(self.h, k)

    def stat(self, name):
        """A named engine statistic (fhe_ctx_stat): "launches", "keyswitches", "ks_limbs",
        "pt_encodes", "pt_cached", "host_waits"."""
        h = lib()
        h.fhe_ctx_stat.restype = C.c_int
        h.fhe_ctx_stat.argtypes = [_VP, C.c_char_p, C.POINTER(C.c_longlong)]
        v = C.c_longlong()
        _check(h.fhe_ctx_stat(self.h, name.encode(), C.byref(v)))
        return v.value

    def counters(self):
        """(key switches issued, sum of their limb counts) since the context was created."""
        h = lib()
        h.fhe_ctx_counters.restype = C.c_int
        h.fhe_ctx_counters.argtypes = [_VP, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]
        k, l = C.c_longlong(), C.c_longlong()
        _check(h.fhe_ctx_counters(self.h, C.byref(k), C.byref(l)))
        return k.value, l.value

    def memory(self):
        """Device memory in bytes: free, total, held by the stream-ordered pool, live in the
        pool, cached BSGS plaintexts."""
        h = lib()
        h.fhe_ctx_memory.restype = C.c_int
        h.fhe_ctx_memory.argtypes = [_VP, C.POINTER(C.c_longlong)]
        out = (C.c_longlong * 5)()
        _check(h.fhe_ctx_memory(self.h, out))
        return dict(zip(("free", "total", "pool_reserved", "pool_used", "pt_cache"), list(out)))

    def set_option(self, name, value):
        """Engine switches: "matvec_tensor_cores" (1 = tcgen05 BSGS products, 0 = CUDA cores),
        "merged_rescale", "profile_every", "plaintext_cache" (1 = a BSGS plan keeps its plaintext
        words for the next call at the same level and scale), "plaintext_cache_reserve_mib",
        "pdl", "ntt_cluster", "boot_delta_log2" (the bootstrap input scale, read by
        EvalBootstrapSetup: 0 = 2^(bits(q0) - 11), -1 = the canonical level-1 scale, else
        2^value)."""
        _check(lib().fhe_ctx_set_option(self.h, name.encode(), int(value)))

    def stream_ptr(self):
        """The engine's cudaStream_t (an int), e.g. for torch.cuda.ExternalStream."""
        return lib().fhe_ctx_stream(self.h)

    def profile(self, on=True):
        _check(lib().fhe_prof_enable(self.h, 1 if on else 0))

    def profile_collect(self):
        """{kernel: (launches, total_ms, algorithmic_bytes, int8_macs)} since the last collect
        (int8_macs: multiply-accumulates given to the tensor cores, 0 for the other kernels)."""
        import json
        buf = C.create_string_buffer(1 << 16)
        _check(lib().fhe_prof_collect(self.h, buf, len(buf)))
        return {k: tuple(v) for k, v in json.loads(buf.value.decode()).items()}

    # ---- keys
    def KeyGen(self, seed=1):
        _check(lib().fhe_keygen(self.h, seed32(seed)))

    def EvalRotateKeyGen(self, steps, conj=False):
        arr = (C.c_int32 * len(steps))(*steps)
        _check(lib().fhe_keygen_rotations(self.h, arr, len(steps), 1 if conj else 0))

    def keygen_auto(self, indices):
        """Keys for automorphism indices (the autoIndices of a rotation-index contract)."""
        h = lib()
        h.fhe_keygen_auto.restype = C.c_int
        h.fhe_keygen_auto.argtypes = [_VP, _U64P, C.c_int]
        w = np.ascontiguousarray(indices, dtype=np.uint64)
        _check(h.fhe_keygen_auto(self.h, w.ctypes.data_as(_U64P), len(w)))

    def key_words(self, which=0):
        out = np.empty((self.dnum, 2, self.L + self.K, self.N), dtype=np.uint64)
        _check(lib().fhe_key_export(self.h, which, out.ctypes.data_as(_U64P)))
        return out

    def import_key(self, which, words):
        w, p = _u64(words)
        _check(lib().fhe_key_import(self.h, which, p))

    def secret_coeffs(self):
        s = np.empty(self.N, dtype=np.int8)
        _check(lib().fhe_secret_export(self.h, s.ctypes.data_as(C.POINTER(C.c_int8))))
        return s

    def public_key_words(self):
        out = np.empty((2, self.L, self.N), dtype=np.uint64)
        _check(lib().fhe_pubkey_export(self.h, out.ctypes.data_as(_U64P)))
        return out

    # ---- encoding / encryption
    def MakeCKKSPackedPlaintext(self, values, level=0, scale=0.0):
        z = np.asarray(values, dtype=np.complex128).ravel()
        re = np.ascontiguousarray(z.real)
        im = np.ascontiguousarray(z.imag)
        h = _VP()
        _check(lib().fhe_encode(self.h, re.ctypes.data_as(_DP), im.ctypes.data_as(_DP), len(z), level, scale,
                                C.byref(h)))
        return Plaintext(self, h)

    def periodic_encode_comp(self, periods, level=0, scale=0.0):
        """Compressed store entries of period vectors (the reference's periodicEncodeComp,
        periodic_encode.hpp:263-276): periods (count, period) complex -> words
        [count][L - level][2 period]; word j2 of a limb equals word j2 << log2(N / (2 period)) of
        the dense encoding of the tiled vector."""
        z = np.asarray(periods, dtype=np.complex128)
        if z.ndim == 1:
            z = z[None]
        count, period = z.shape
        re = np.ascontiguousarray(z.real)
        im = np.ascontiguousarray(z.imag)
        out = np.empty((count, self.L - level, 2 * period), dtype=np.uint64)
        _check(lib().fhe_encode_periodic(self.h, re.ctypes.data_as(_DP), im.ctypes.data_as(_DP), period, count, level,
                                         scale, out.ctypes.data_as(_U64P)))
        return out

    def Decode(self, pt):
        re = np.empty(self.slots)
        im = np.empty(self.slots)
        _check(lib().fhe_decode(self.h, pt.h, re.ctypes.data_as(_DP), im.ctypes.data_as(_DP)))
        return re + 1j * im

    def Encrypt(self, pt):
        h = _VP()
        _check(lib().fhe_encrypt(self.h, pt.h, C.byref(h)))
        return Ciphertext(self, h)

    def Decrypt(self, ct):
        h = _VP()
        _check(lib().fhe_decrypt(self.h, ct.h, C.byref(h)))
        return self.Decode(Plaintext(self, h))

    def decrypt_pt(self, ct):
        h = _VP()
        _check(lib().fhe_decrypt(self.h, ct.h, C.byref(h)))
        return Plaintext(self, h)

    # ---- evaluation
    def _bin(self, fn, a, b):
        h = _VP()
        _check(fn(self.h, a.h, b.h, C.byref(h)))
        return Ciphertext(self, h)

    def EvalMult(self, a, b):
        if isinstance(b, Plaintext):
            return self._bin(lib().fhe_mul_ct_pt, a, b)
        return self._bin(lib().fhe_mul_ct_ct_relin, a, b)

    def EvalAdd(self, a, b):
        if isinstance(b, Plaintext):
            return self._bin(lib().fhe_add_pt, a, b)
        return self._bin(lib().fhe_add, a, b)

    def EvalSub(self, a, b):
        return self._bin(lib().fhe_sub, a, b)

    def EvalMultConst(self, a, v, scale=0.0):
        h = _VP()
        _check(lib().fhe_mul_const(self.h, a.h, float(v), float(scale), C.byref(h)))
        return Ciphertext(self, h)

    def EvalAddConst(self, a, v):
        h = _VP()
        _check(lib().fhe_add_const(self.h, a.h, float(v), C.byref(h)))
        return Ciphertext(self, h)

    def RescaleInPlace(self, ct):
        _check(lib().fhe_rescale(self.h, ct.h))

    def LevelReduceInPlace(self, ct, levels):
        _check(lib().fhe_level_reduce(self.h, ct.h, levels))

    def EvalRotate(self, ct, k):
        h = _VP()
        _check(lib().fhe_rotate(self.h, ct.h, k, C.byref(h)))
        return Ciphertext(self, h)

    def EvalFastRotation(self, ct, ks):
        n = len(ks)
        arr = (C.c_int32 * n)(*ks)
        outs = (_VP * n)()
        _check(lib().fhe_rotate_hoisted(self.h, ct.h, arr, n, outs))
        return [Ciphertext(self, outs[i]) for i in range(n)]

    def EvalRotateSum(self, cts, ks):
        """sum_i EvalRotate(cts[i], ks[i]) with one batched key switch and one ModDown."""
        n = len(cts)
        arr = (_VP * n)(*[c.h for c in cts])
        kk = (C.c_int32 * n)(*ks)
        h = _VP()
        _check(lib().fhe_rotate_sum(self.h, arr, kk, n, C.byref(h)))
        return Ciphertext(self, h)

    def EvalConj(self, ct):
        h = _VP()
        _check(lib().fhe_conjugate(self.h, ct.h, C.byref(h)))
        return Ciphertext(self, h)

    def Copy(self, ct):
        h = _VP()
        _check(lib().fhe_ct_copy(self.h, ct.h, C.byref(h)))
        return Ciphertext(self, h)

    # ---- circuit level
    def mul_vec_rescale(self, ct, values):
        """mulPt: ct (.) values (per slot, repeated) then RescaleInPlace, canonical scale."""
        z = np.asarray(values, dtype=np.complex128).ravel()
        re, im = np.ascontiguousarray(z.real), np.ascontiguousarray(z.imag)
        h = _VP()
        _check(lib().fhe_mul_vec_rescale(self.h, ct.h, re.ctypes.data_as(_DP), im.ctypes.data_as(_DP), len(z),
                                         C.byref(h)))
        return Ciphertext(self, h)

    def align(self, ct, level):
        _check(lib().fhe_align(self.h, ct.h, level))

    def mul_rescale(self, a, b):
        h = _VP()
        _check(lib().fhe_mul_rescale(self.h, a.h, b.h, C.byref(h)))
        return Ciphertext(self, h)

    def EvalPolyVec(self, ct, coeffs):
        """sum_i coeffs[i] (.) x^i with per-slot real coefficient vectors (power basis)."""
        c = np.ascontiguousarray(np.asarray(coeffs, dtype=np.float64))
        if c.ndim == 1:
            c = c[:, None]
        h = _VP()
        _check(lib().fhe_poly_eval(self.h, ct.h, c.ctypes.data_as(_DP), c.shape[0] - 1, c.shape[1], C.byref(h)))
        return Ciphertext(self, h)

    def EvalChebyshevSeries(self, ct, coeffs):
        c = np.ascontiguousarray(np.asarray(coeffs, dtype=np.float64))
        h = _VP()
        _check(lib().fhe_cheb_eval(self.h, ct.h, c.ctypes.data_as(_DP), len(c), C.byref(h)))
        return Ciphertext(self, h)

    def EvalChebyshevSeriesBatch(self, cts, coeffs):
        """EvalChebyshevSeries on ciphertexts of one level and scale with batched products."""
        c = np.ascontiguousarray(np.asarray(coeffs, dtype=np.float64))
        ins = (_VP * len(cts))(*[x.h for x in cts])
        outs = (_VP * len(cts))()
        _check(lib().fhe_cheb_eval_n(self.h, ins, len(cts), c.ctypes.data_as(_DP), len(c), outs))
        return [Ciphertext(self, outs[k]) for k in range(len(cts))]

    def matvec_plan(self, W, D, b1):
        """Masked block-cyclic BSGS plan of W (rows <= D); column chunk s acts on input s."""
        W = np.ascontiguousarray(np.asarray(W, dtype=np.float64))
        h = _VP()
        _check(lib().fhe_matvec_plan(self.h, W.ctypes.data_as(_DP), W.shape[0], W.shape[1], D, b1, C.byref(h)))
        return _MvPlan(h, self)

    def matvec_keygen(self, D, b1):
        _check(lib().fhe_matvec_keygen(self.h, D, b1))

    def matvec(self, plan, inputs):
        n = len(inputs)
        arr = (_VP * n)(*[c.h for c in inputs])
        h = _VP()
        _check(lib().fhe_matvec_bsgs(self.h, plan.h, arr, n, C.byref(h)))
        return Ciphertext(self, h)

    def EvalBootstrapSetup(self, bound=24.0, degree=59, double_angles=3):
        """EvalMod = Chebyshev interpolant of degree `degree` + `double_angles` double-angle
        steps (baseline config 3: 59 and 3; degree 31 with 4 takes the same levels, fewer products)."""
        _check(lib().fhe_bootstrap_setup_r(self.h, bound, degree, double_angles))

    def EvalBootstrap(self, ct):
        h = _VP()
        _check(lib().fhe_bootstrap(self.h, ct.h, C.byref(h)))
        return Ciphertext(self, h)

    def EvalBootstrapBatch(self, cts):
        """fhe_bootstrap_n: every ciphertext of the list, refreshed, in order."""
        h = lib()
        h.fhe_bootstrap_n.restype = C.c_int
        h.fhe_bootstrap_n.argtypes = [_VP, C.POINTER(_VP), C.c_int, C.POINTER(_VP)]
        ins = (_VP * len(cts))(*[c.h for c in cts])
        outs = (_VP * len(cts))()
        _check(h.fhe_bootstrap_n(self.h, ins, len(cts), outs))
        return [Ciphertext(self, outs[i]) for i in range(len(cts))]

    def bootstrap_level(self):
        return lib().fhe_bootstrap_level(self.h)

    # ---- raw words
    def ct_from_words(self, words, level, scale=1.0):
        w, p = _u64(words)
        h = _VP()
        _check(lib().fhe_ct_import(self.h, p, level, scale, C.byref(h)))
        return Ciphertext(self, h)

    def save_keys_part(self, path, which, tag="fhe-ssm"):
        """Seeded part file (FSSMSKY1) of the keys `which` (0 = relinearisation, else automorphism
        indices), as the reference's writeSeededPart writes it."""
        h = lib()
        h.fhe_keys_save_part.restype = C.c_int
        h.fhe_keys_save_part.argtypes = [_VP, C.c_char_p, _U64P, C.c_int, C.c_char_p]
        w = np.ascontiguousarray(which, dtype=np.uint64)
        _check(h.fhe_keys_save_part(self.h, path.encode(), w.ctypes.data_as(_U64P), len(w), tag.encode()))

    def load_keys_part(self, path):
        """Keys of a seeded part file (b from the file, a expanded from the seeds on the device);
        returns how many were added."""
        h = lib()
        h.fhe_keys_load_part.restype = C.c_int
        h.fhe_keys_load_part.argtypes = [_VP, C.c_char_p, C.POINTER(C.c_int)]
        n = C.c_int()
        _check(h.fhe_keys_load_part(self.h, path.encode(), C.byref(n)))
        return n.value

    def pt_from_words(self, words, level, scale=1.0):
        w, p = _u64(words)
        h = _VP()
        _check(lib().fhe_pt_import(self.h, p, level, scale, C.byref(h)))
        return Plaintext(self, h)

    def pt_words(self, pt):
        nl = self.L - pt.level
        out = np.empty((nl, self.N), dtype=np.uint64)
        _check(lib().fhe_pt_export(self.h, pt.h, out.ctypes.data_as(_U64P)))
        return out

    def ntt(self, words, mod_idx, inverse=False):
        w = np.ascontiguousarray(words, dtype=np.uint64).copy()
        n = w.size // self.N
        mi = (C.c_int * n)(*[int(x) for x in mod_idx])
        _check(lib().fhe_ntt_host(self.h, w.ctypes.data_as(_U64P), n, mi, 1 if inverse else 0))
        return w

    def keyswitch_raw(self, d, level, key):
        d, dp = _u64(d)
        k, kp = _u64(key)
        nl = self.L - level
        o0 = np.empty((nl, self.N), dtype=np.uint64)
        o1 = np.empty_like(o0)
        _check(lib().fhe_keyswitch_host(self.h, dp, level, kp, o0.ctypes.data_as(_U64P), o1.ctypes.data_as(_U64P)))
        return o0, o1


def _register_diagnostics():
    h = lib()
    h.fhe_bootstrap_stage.restype = C.c_int
    h.fhe_bootstrap_stage.argtypes = [_VP, _VP, C.c_int, C.POINTER(_VP)]


def cheb_depth(coeffs):
    """Levels EvalChebyshevSeries consumes for these coefficients (host computation, no GPU)."""
    c = np.ascontiguousarray(np.asarray(coeffs, dtype=np.float64))
    d = C.c_int()
    _check(lib().fhe_cheb_depth(c.ctypes.data_as(_DP), len(c), C.byref(d)))
    return d.value


def bootstrap_stage(ctx, ct, upto):
    """Diagnostics: the bootstrap pipeline stopped after stage `upto` (1..4)."""
    _register_diagnostics()
    h = _VP()
    _check(lib().fhe_bootstrap_stage(ctx.h, ct.h, upto, C.byref(h)))
    return Ciphertext(ctx, h)
