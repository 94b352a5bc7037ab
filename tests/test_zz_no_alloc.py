"""fhe_keyswitch_noalloc: the key switch whose working memory is a static device array.

Called through the C-ABI on device buffers and compared word for word with the allocating
entry point fhe_keyswitch_host on the same inputs and keys.  The file name sorts last so
the suite also runs it after every other GPU test in the same process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FHE_ERR_ARG = -1


@pytest.fixture(scope="module")
def env():
    import torch
    import fhessm
    cx = fhessm.CryptoContext(logN=16, L=20, K=4, alpha=4, hw=192)
    cx.KeyGen(seed=11)
    cx.EvalRotateKeyGen([1])
    h = fhessm.lib()
    h.fhe_keyswitch_noalloc.restype = C.c_int
    h.fhe_keyswitch_noalloc.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    yield cx, h, torch
    cx.sync()
    cx.close()


def rand_limbs(cx, nl, rng):
    return np.stack([rng.integers(0, int(cx.moduli[i]), cx.N, dtype=np.uint64) for i in range(nl)])


def to_dev(torch, words):
    return torch.from_numpy(np.ascontiguousarray(words).view(np.int64)).to("cuda:0")


def from_dev(t):
    return t.cpu().numpy().view(np.uint64)


def noalloc(cx, h, torch, which, d, level):
    nl = cx.L - level
    o0 = torch.empty((nl, cx.N), dtype=torch.int64, device="cuda:0")
    o1 = torch.empty_like(o0)
    rc = h.fhe_keyswitch_noalloc(cx.h, which, d.data_ptr(), level, o0.data_ptr(), o1.data_ptr())
    assert rc == 0, h.fhe_last_error().decode()
    return o0, o1


def test_noalloc_matches_allocating_keyswitch_on_consecutive_calls(env):
    cx, h, torch = env
    rng = np.random.default_rng(21)
    k = cx.rot_index(1)
    lv1, lv2 = 4, 9                       # 16 limbs (the largest that fits at N = 2^16), then 11
    w1, w2 = rand_limbs(cx, cx.L - lv1, rng), rand_limbs(cx, cx.L - lv2, rng)
    d1, d2 = to_dev(torch, w1), to_dev(torch, w2)
    torch.cuda.synchronize()
    # two calls back to back on the context's stream, no synchronisation between them
    a0, a1 = noalloc(cx, h, torch, 0, d1, lv1)
    b0, b1 = noalloc(cx, h, torch, k, d2, lv2)
    cx.sync()
    torch.cuda.synchronize()
    e0, e1 = cx.keyswitch_raw(w1, lv1, cx.key_words(0))
    f0, f1 = cx.keyswitch_raw(w2, lv2, cx.key_words(k))
    assert (from_dev(a0) == e0).all() and (from_dev(a1) == e1).all()
    assert (from_dev(b0) == f0).all() and (from_dev(b1) == f1).all()
    assert e0.any() and f1.any()
    # the first input again, after the scratch held the second call's data
    c0, c1 = noalloc(cx, h, torch, 0, d1, lv1)
    cx.sync()
    assert (from_dev(c0) == e0).all() and (from_dev(c1) == e1).all()


def _pool_high_water(reset):
    """Used-memory high-water mark of device 0's default memory pool (the pool the engine's
    stream-ordered allocations come from), through the driver API; reset=True restarts it."""
    cu = C.CDLL("libcuda.so.1")
    pool = C.c_void_p()
    assert cu.cuDeviceGetDefaultMemPool(C.byref(pool), 0) == 0
    used_high = 8   # CU_MEMPOOL_ATTR_USED_MEM_HIGH (value type cuuint64_t)
    v = C.c_uint64(0)
    if reset:
        assert cu.cuMemPoolSetAttribute(pool, used_high, C.byref(v)) == 0
    assert cu.cuMemPoolGetAttribute(pool, used_high, C.byref(v)) == 0
    return v.value


def test_noalloc_allocates_nothing(env):
    """The property the entry point exists for: across calls (after the first, which sets up the
    per-GPU scratch address), neither the pool's high-water mark nor the device's free memory
    moves."""
    cx, h, torch = env
    rng = np.random.default_rng(5)
    lv = 6
    d = to_dev(torch, rand_limbs(cx, cx.L - lv, rng))
    o0 = torch.empty((cx.L - lv, cx.N), dtype=torch.int64, device="cuda:0")
    o1 = torch.empty_like(o0)
    k = cx.rot_index(1)
    assert h.fhe_keyswitch_noalloc(cx.h, 0, d.data_ptr(), lv, o0.data_ptr(), o1.data_ptr()) == 0
    cx.sync()
    torch.cuda.synchronize()
    mem0 = cx.memory()
    free0 = torch.cuda.mem_get_info(0)[0]
    hw0 = _pool_high_water(reset=True)
    for which in (0, k, 0):
        assert h.fhe_keyswitch_noalloc(cx.h, which, d.data_ptr(), lv, o0.data_ptr(), o1.data_ptr()) == 0
    cx.sync()
    mem1 = cx.memory()
    assert _pool_high_water(reset=False) <= hw0, "the pool's high-water mark grew during no-alloc calls"
    assert (mem1["pool_used"], mem1["pool_reserved"]) == (mem0["pool_used"], mem0["pool_reserved"])
    assert torch.cuda.mem_get_info(0)[0] == free0


def test_noalloc_refuses_oversize_and_host_memory(env):
    cx, h, torch = env
    d = torch.zeros((cx.L, cx.N), dtype=torch.int64, device="cuda:0")
    o = torch.zeros_like(d)
    rc = h.fhe_keyswitch_noalloc(cx.h, 0, d.data_ptr(), 0, o.data_ptr(), o.data_ptr())
    msg = h.fhe_last_error().decode()
    assert rc == FHE_ERR_ARG and "scratch" in msg and "at most 16 limbs" in msg, msg
    host = np.zeros((cx.L - 5, cx.N), dtype=np.uint64)
    rc = h.fhe_keyswitch_noalloc(cx.h, 0, host.ctypes.data, 5, o.data_ptr(), o.data_ptr())
    assert rc == FHE_ERR_ARG and "not device memory" in h.fhe_last_error().decode()
