"""Seeded key part files (FSSMSKY1) on CPU: the engine's writer and header reader against the
reference's own header reader and byte I/O (hpc_gpu_port/seeded_keys.hpp:195, :302-317,
:321-325, :352-375, compiled where they lie by oracle/ref_extract.sh when the reference tree is
present), and against a golden digest of the file bytes for machines without it.  The layout
is the reference's: magic, version, expander, N, sizeQ, sizeP, numPartQ, numPerPartQ, count,
key tag, moduli, then per key its automorphism index, 32-byte seed and b words."""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "fhe-ssm_b200", "fhessm", "libfhessm.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref_pins.so")
GOLD = os.path.join(ROOT, "tests", "golden", "part_file.json")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="libfhessm.so not built")

LAYOUT = dict(N=1024, sizeQ=5, sizeP=2, numPartQ=2, numPerPartQ=3)


def sample_file(path):
    """A small part file with seeded words: 3 keys (relinearisation slot 0 and two automorphisms)."""
    from fhessm import write_part_words
    rng = np.random.default_rng(77)
    mods = rng.integers(1 << 40, 1 << 60, LAYOUT["sizeQ"] + LAYOUT["sizeP"], dtype=np.uint64)
    idx = np.array([0, 5, 2047], dtype=np.uint32)
    seeds = rng.integers(0, 256, (3, 32), dtype=np.uint8)
    b = rng.integers(0, 1 << 60, (3, LAYOUT["numPartQ"], LAYOUT["sizeQ"] + LAYOUT["sizeP"], LAYOUT["N"]),
                     dtype=np.uint64)
    write_part_words(path, LAYOUT, mods, "fhe-ssm-test", idx, seeds, b)
    return mods, idx, seeds, b


def test_part_file_roundtrip_and_golden_bytes(tmp_path):
    from fhessm import part_header
    path = str(tmp_path / "evalrot.part000.seeded.bin")
    mods, idx, seeds, b = sample_file(path)
    lay, m2, tag = part_header(path)
    assert (lay["version"], lay["expander"], lay["count"]) == (1, 1, 3)
    assert all(lay[k] == v for k, v in LAYOUT.items())
    assert (m2 == mods).all() and tag == "fhe-ssm-test"
    raw = open(path, "rb").read()
    head = 8 + 4 * 9 + len(tag) + 8 * len(mods)
    per = 4 + 32 + b[0].size * 8
    assert len(raw) == head + 3 * per                       # bytesPerKey / headerBytes of the reference
    assert raw[:8] == b"FSSMSKY1"
    for k in range(3):
        rec = raw[head + k * per: head + (k + 1) * per]
        assert int.from_bytes(rec[:4], "little") == idx[k] and rec[4:36] == seeds[k].tobytes()
        assert (np.frombuffer(rec[36:], dtype="<u8") == b[k].ravel()).all()
    gold = json.load(open(GOLD))
    assert hashlib.sha256(raw).hexdigest() == gold["sha256"]


def test_part_header_refuses_bad_files(tmp_path):
    from fhessm import FheError, part_header
    p = str(tmp_path / "bad.bin")
    open(p, "wb").write(b"FSSMSKY2" + bytes(64))
    with pytest.raises(FheError, match="bad magic"):
        part_header(p)
    open(p, "wb").write(b"FSSMSKY1" + (2).to_bytes(4, "little") + bytes(40))
    with pytest.raises(FheError, match="version"):
        part_header(p)
    open(p, "wb").write(b"FSSMSKY1" + bytes(6))
    with pytest.raises(FheError, match="short header"):
        part_header(p)


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="the reference's reader is not compiled here (oracle/_ref)")
def test_reference_reader_parses_engine_part_file(tmp_path):
    ref = C.CDLL(REF_SO)
    U64P = C.POINTER(C.c_uint64)
    ref.ref_read_part.argtypes = [C.c_char_p, C.POINTER(C.c_uint32), U64P, C.c_char_p, C.c_int,
                                  C.POINTER(C.c_uint32), C.POINTER(C.c_uint8), U64P, C.c_int, C.c_char_p, C.c_int]
    path = str(tmp_path / "evalrot.part000.seeded.bin")
    mods, idx, seeds, b = sample_file(path)
    head = (C.c_uint32 * 8)()
    m2 = np.zeros(len(mods), dtype=np.uint64)
    tag, err = C.create_string_buffer(64), C.create_string_buffer(256)
    i2 = (C.c_uint32 * 3)()
    s2 = np.zeros((3, 32), dtype=np.uint8)
    bh = np.zeros((3, 16), dtype=np.uint64)
    rc = ref.ref_read_part(path.encode(), head, m2.ctypes.data_as(U64P), tag, 64, i2,
                           s2.ctypes.data_as(C.POINTER(C.c_uint8)), bh.ctypes.data_as(U64P), 16, err, 256)
    assert rc == 0, err.value
    assert list(head) == [1, 1, LAYOUT["N"], LAYOUT["sizeQ"], LAYOUT["sizeP"], LAYOUT["numPartQ"],
                          LAYOUT["numPerPartQ"], 3]
    assert (m2 == mods).all() and tag.value == b"fhe-ssm-test"
    assert list(i2) == list(idx) and (s2 == seeds).all()
    assert (bh == b.reshape(3, -1)[:, :16]).all()
