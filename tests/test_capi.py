"""The C-ABI library loads on a machine without a GPU and exports every symbol that
include/fhessm.h declares (no compute call is made here)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fhessm.h")
LIB = os.path.join(ROOT, "fhe-ssm_b200", "fhessm", "libfhessm.so")


def declared_symbols():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(fhe_[a-z0-9_]+)\s*\(", txt)))


def test_header_declares_the_operator_surface():
    syms = declared_symbols()
    for need in ("fhe_ctx_create", "fhe_keygen", "fhe_encode", "fhe_encrypt", "fhe_decrypt", "fhe_mul_ct_pt",
                 "fhe_mul_ct_ct_relin", "fhe_rescale", "fhe_rotate", "fhe_rotate_hoisted", "fhe_conjugate"):
        assert need in syms


@pytest.mark.skipif(not os.path.exists(LIB), reason="libfhessm.so not built")
def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


@pytest.mark.skipif(not os.path.exists(LIB), reason="libfhessm.so not built")
def test_errors_are_reported_not_raised():
    """A null argument returns a negative status and a message (no device touched)."""
    lib = ctypes.CDLL(LIB)
    lib.fhe_ctx_create.restype = ctypes.c_int
    lib.fhe_last_error.restype = ctypes.c_char_p
    rc = lib.fhe_ctx_create(None, None)
    assert rc < 0
    assert b"null" in lib.fhe_last_error()
