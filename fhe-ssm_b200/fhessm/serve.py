"""The serve loop and its client side: the request/response file protocol of the reference's
stateful server (hpc_gpu_port/gpu_real_model.cu:4363-4483) as driven by ml-eval/fhe_client.py
(:1394-1493).  The loop itself is native (fhe_serve_files / fhe_serve_model in libfhessm.so);
this module holds the ciphertext file format and the client calls."""
import ctypes as C
import json
import os
import struct
import time

import numpy as np

from . import FheError, _check, lib

MAGIC = b"FSSMCT01"


class WireCt(C.Structure):
    _fields_ = [("level", C.c_int), ("nl", C.c_int), ("logN", C.c_int), ("scale", C.c_double),
                ("words", C.POINTER(C.c_uint64))]


STEP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(WireCt), C.POINTER(C.c_int),
                      C.POINTER(WireCt))


def write_ct_file(path, level, scale, words):
    """A ciphertext file: magic, int32 level, limbs, logN, pad, double scale, [2][limbs][N] words."""
    w = np.ascontiguousarray(words, dtype=np.uint64)
    nl, n = w.shape[1], w.shape[2]
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC + struct.pack("<iiiid", level, nl, n.bit_length() - 1, 0, scale))
        f.write(w.tobytes())
    os.replace(tmp, path)


def read_ct_file(path):
    with open(path, "rb") as f:
        head = f.read(32)
        if head[:8] != MAGIC:
            raise FheError(-7, f"{path}: not a ciphertext file")
        level, nl, logn, _, scale = struct.unpack("<iiiid", head[8:32])
        words = np.frombuffer(f.read(), dtype=np.uint64).reshape(2, nl, 1 << logn).copy()
    return level, scale, words


def submit(reqdir, n, cts, reset=False, **meta):
    """Client: request n with ciphertexts [(level, scale, words), ...]; `reset` starts a new session."""
    pre = os.path.join(reqdir, f"req.{n}")
    for i, (level, scale, words) in enumerate(cts):
        write_ct_file(f"{pre}.{i}", level, scale, words)
    with open(pre + ".meta", "w") as f:
        json.dump(dict(count=len(cts), **meta), f)
    if reset:
        open(pre + ".reset", "w").close()
    open(pre + ".ready", "w").close()


def wait_response(reqdir, n, timeout=600.0, poll=0.01):
    """Client: the ciphertexts and meta of response n (raises FheError on resp.n.error)."""
    pre = os.path.join(reqdir, f"resp.{n}")
    t0 = time.time()
    while True:
        if os.path.exists(pre + ".error"):
            raise FheError(-7, open(pre + ".error").read().strip())
        if os.path.exists(pre + ".done"):
            meta = json.load(open(pre + ".meta"))
            return [read_ct_file(f"{pre}.{i}") for i in range(meta["count"])], meta
        if time.time() - t0 > timeout:
            raise TimeoutError(f"no response {n} in {timeout} s")
        time.sleep(poll)


def serve_files(reqdir, step, timeout_ms=60000, max_requests=0):
    """Run the native serve loop with a Python step(reset, [(level, scale, words)]) ->
    [(level, scale, words)] (used to test the protocol without a GPU).  Returns requests served."""
    def cb(user, reset, n_in, inp, n_out, out):
        try:
            cts = []
            for i in range(n_in):
                w = inp[i]
                a = np.ctypeslib.as_array(w.words, shape=(2 * w.nl << w.logN,)).reshape(2, w.nl, 1 << w.logN).copy()
                cts.append((w.level, w.scale, a))
            res = step(bool(reset), cts)
            # out[i].words has room for the words of input i only: check every result first
            if not 1 <= len(res) <= n_in:
                return -7
            res = [(lv, sc, np.ascontiguousarray(wd, dtype=np.uint64)) for lv, sc, wd in res]
            for i, (_, _, words) in enumerate(res):
                if (words.ndim != 3 or words.shape[0] != 2 or words.shape[2] != 1 << inp[i].logN
                        or not 1 <= words.shape[1] <= inp[i].nl):
                    return -7
            for i, (level, scale, words) in enumerate(res):
                out[i].level, out[i].nl, out[i].scale = level, words.shape[1], scale
                C.memmove(out[i].words, words.ctypes.data, words.nbytes)
            n_out[0] = len(res)
            return 0
        except Exception:
            return -7
    fn = STEP_FN(cb)
    h = lib()
    h.fhe_serve_files.restype = C.c_int
    h.fhe_serve_files.argtypes = [C.c_char_p, C.c_int, C.c_int, STEP_FN, C.c_void_p, C.POINTER(C.c_int)]
    served = C.c_int()
    _check(h.fhe_serve_files(reqdir.encode(), timeout_ms, max_requests, fn, None, C.byref(served)))
    return served.value


def serve_model(model, reqdir, timeout_ms=600000, max_requests=0):
    """Serve an EncryptedModel: one pack of conversations per request, carried state across
    requests, req.<N>.reset for a new session.  Returns the number of requests served."""
    h = lib()
    h.fhe_serve_model.restype = C.c_int
    h.fhe_serve_model.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.POINTER(C.c_int)]
    served = C.c_int()
    _check(h.fhe_serve_model(model.h, reqdir.encode(), timeout_ms, max_requests, C.byref(served)))
    return served.value
