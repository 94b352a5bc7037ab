"""Limb-partitioned key switching on CPU: two gloo ranks split one hybrid key switch by limbs
(fhessm.dist.partitioned_keyswitch_cpu: all-gather of d's coefficient limbs before ModUp, of the
special limbs before ModDown, the C oracle doing each rank's share), and the gathered result must
equal the oracle's single-process key switch word for word.  Also checks the limb blocks."""
import os

import numpy as np
import pytest

from conftest import ROOT


def test_limb_blocks_cover_every_limb_once():
    from fhessm.dist import limb_block
    for n in (1, 2, 4, 7, 20, 30):
        for ws in (1, 2, 3, 4, 8):
            seen = []
            for r in range(ws):
                lo, cnt, per = limb_block(n, ws, r)
                assert 0 <= cnt <= per and per * ws >= n
                seen += list(range(lo, lo + cnt))
            assert seen == list(range(n)), (n, ws)


def _rank(rank, ws, port, q):
    import sys
    for p in (os.path.join(ROOT, "fhe-ssm_b200"), os.path.join(ROOT, "tests")):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from fhessm.dist import partitioned_keyswitch_cpu
    from oracle_lib import Oracle, derive_seed, gen_chain, load
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=ws)
        lib = load()
        qs, ps = gen_chain(10, 7, 60, 45, 3, 60, lib)
        o = Oracle(10, qs, ps, 2, lib)
        ms = (5).to_bytes(8, "little") + bytes(24)
        se = o.secret_eval(o.secret(derive_seed(lib, ms, 0xFFFFFFF1), 32))
        key = o.keygen_switch(se, se, derive_seed(lib, ms, 3))
        rng = np.random.default_rng(11)
        ok = True
        for nl in (7, 5, 2):
            d = np.stack([rng.integers(0, int(o.mods[i]), o.N, dtype=np.uint64) for i in range(nl)])
            g0, g1 = partitioned_keyswitch_cpu(o, d, nl, key)
            e0, e1 = o.keyswitch(d, nl, key)
            ok = ok and bool((g0 == e0).all() and (g1 == e1).all())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok))
    except Exception as ex:   # reported to the parent, which fails the test
        q.put((rank, repr(ex)))


@pytest.mark.parametrize("ws", [2, 3])
def test_partitioned_keyswitch_gloo_matches_single(ws):
    import multiprocessing as mp
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(ws))
    for p in procs:
        p.join(60)
    assert all(v is True for v in res.values()), res
