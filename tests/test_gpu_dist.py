"""Limb-partitioned key switching on 2 GPUs (NCCL), word for word against the single-GPU key
switch.  Two processes, one per GPU, each with a context of the same chain and the same key seed;
rank 0 makes the NCCL unique id and shares it through a queue.  For several levels each rank
key-switches its own block of d's limbs (fhe_keyswitch_dist) and its result block must equal the
same block of fhe_keyswitch_host on the whole of d.  Skipped with fewer than 2 GPUs."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import ctypes
        cu = ctypes.CDLL("libcuda.so.1")
        n = ctypes.c_int(0)
        return n.value if cu.cuInit(0) == 0 and cu.cuDeviceGetCount(ctypes.byref(n)) == 0 else 0
    except OSError:
        return 0


def _rank(rank, world, qid, qres):
    for p in (os.path.join(ROOT, "fhe-ssm_b200"), os.path.join(ROOT, "tests")):
        sys.path.insert(0, p)
    try:
        import torch
        import fhessm
        from fhessm import dist
        torch.cuda.set_device(rank)
        cx = fhessm.CryptoContext(logN=16, L=12, K=4, alpha=4, hw=192, device=rank)
        cx.KeyGen(seed=31)
        cx.EvalRotateKeyGen([3])
        if rank == 0:
            uid = dist.unique_id()
            for _ in range(world - 1):
                qid.put(uid)
        else:
            uid = qid.get(timeout=120)
        dist.init(cx, world, rank, uid)
        rng = np.random.default_rng(7)
        ok = True
        for level, which in ((0, 0), (3, cx.rot_index(3)), (9, 0)):
            nl = cx.L - level
            d = np.stack([rng.integers(0, int(cx.moduli[i]), cx.N, dtype=np.uint64) for i in range(nl)])
            lo, cnt, _ = dist.limb_block(nl, world, rank)
            dev = torch.from_numpy(np.ascontiguousarray(d[lo:lo + cnt]).view(np.int64)).to(f"cuda:{rank}")
            o0 = torch.zeros((max(cnt, 1), cx.N), dtype=torch.int64, device=f"cuda:{rank}")
            o1 = torch.zeros_like(o0)
            torch.cuda.synchronize()
            dist.keyswitch(cx, which, dev.data_ptr(), level, o0.data_ptr(), o1.data_ptr())
            cx.sync()
            e0, e1 = cx.keyswitch_raw(d, level, cx.key_words(which))
            g0, g1 = o0.cpu().numpy().view(np.uint64)[:cnt], o1.cpu().numpy().view(np.uint64)[:cnt]
            ok = ok and bool((g0 == e0[lo:lo + cnt]).all() and (g1 == e1[lo:lo + cnt]).all())
        cx.close()
        qres.put((rank, ok))
    except Exception as ex:
        qres.put((rank, repr(ex)))


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_limb_partitioned_keyswitch_two_gpus():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    qid, qres = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, qid, qres)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(qres.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(120)
    assert all(v is True for v in res.values()), res
