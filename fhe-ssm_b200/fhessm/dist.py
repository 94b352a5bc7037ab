"""Limb-partitioned key switching across GPUs (single-pack latency).

The reference splits one context's RNS limbs over several GPUs (gpu_real_model.cu:847-884, the
--devices flag; FIDESlib places limb i on device i mod G, :995-997, :1158-1161).  Here each rank
owns a contiguous block of the Q limbs and of the K special limbs of every polynomial
(`limb_block`); a hybrid key switch then needs two all-gathers:

  1. the rank's Q limbs of d, inverse-transformed to coefficient form -> every rank holds all
     of d in coefficient form, which each digit's base conversion reads (ModUp);
  2. the rank's special limbs of both inner-product polynomials, in coefficient form -> every
     rank holds the P part that ModDown converts (4 MiB at K = 4, N = 2^16).

Everything else (base conversion to the rank's own limbs, NTTs, the key inner product, ModDown's
final step) is local to a rank's limbs.  On GPUs the engine runs both all-gathers with NCCL on its
own stream (fhe_dist_init / fhe_keyswitch_dist); `partitioned_keyswitch_cpu` is the same exchange
over any torch.distributed group (gloo on CPU) with the C oracle doing each rank's arithmetic,
which is how the plan is tested without GPUs.
"""
import ctypes as C

import numpy as np

from . import FheError, _check, lib


def limb_block(n, world, rank):
    """Rank `rank`'s block of n limbs: (first, count, per) with per = ceil(n / world) (the padded
    block every rank contributes to an all-gather; ranks past the end own nothing)."""
    per = -(-n // world)
    lo = min(n, rank * per)
    return lo, min(n, lo + per) - lo, per


def partitioned_keyswitch_cpu(o, d, nl, key, group=None):
    """One hybrid key switch of d (all nl Q limbs, eval form; every rank passes the same words) split
    over the ranks of a torch.distributed group: returns (out0, out1), all nl limbs, gathered from
    the ranks' shares.  o: an oracle context (tests/oracle_lib.Oracle) of the same chain."""
    import torch
    import torch.distributed as dist
    ws, rank = dist.get_world_size(group), dist.get_rank(group)
    N, K = o.N, o.np_
    qlo, nqo, qper = limb_block(nl, ws, rank)
    plo, npo, pper = limb_block(K, ws, rank)

    def gather(own, per):
        # own: (count, ...) -> the ranks' blocks, each padded to `per` rows, in rank order
        pad = np.zeros((per,) + own.shape[1:], dtype=np.uint64)
        pad[: own.shape[0]] = own
        parts = [torch.zeros(pad.shape, dtype=torch.int64) for _ in range(ws)]
        dist.all_gather(parts, torch.from_numpy(pad.view(np.int64)), group=group)
        return np.concatenate([p.numpy().view(np.uint64) for p in parts])

    # exchange 1: the rank's Q limbs of d in coefficient form
    own_coef = np.stack([o.intt(d[i], i) for i in range(qlo, qlo + nqo)]) if nqo else np.zeros((0, N), np.uint64)
    dcoef = np.ascontiguousarray(gather(own_coef, qper)[:nl])
    # ModUp and the inner product on the rank's own limbs
    no = nqo + npo
    from oracle_lib import p64
    ext = np.zeros((o.dnum(nl), no, N), dtype=np.uint64)
    i0 = np.zeros((no, N), dtype=np.uint64)
    i1 = np.zeros((no, N), dtype=np.uint64)
    if no:
        o.lib.oc_ks_part_ext(o.ctx, p64(dcoef), nl, qlo, nqo, plo, npo, p64(ext))
        o.lib.oc_ks_part_inner(o.ctx, p64(ext), nl, p64(np.ascontiguousarray(key)), qlo, nqo, plo, npo, p64(i0),
                               p64(i1))
    # exchange 2: the rank's special limbs of both polynomials in coefficient form
    own_p = np.stack([np.stack([o.intt(ip[nqo + k], o.nq + plo + k) for k in range(npo)]) if npo
                      else np.zeros((0, N), np.uint64) for ip in (i0, i1)], axis=1)   # (npo, 2, N)
    pcoef = gather(own_p, pper)[:K]                                                    # (K, 2, N)
    outs = []
    for c, ip in enumerate((i0, i1)):
        out = np.zeros((nqo, N), dtype=np.uint64)
        if nqo:
            o.lib.oc_ks_part_moddown(o.ctx, p64(np.ascontiguousarray(ip[:nqo])),
                                     p64(np.ascontiguousarray(pcoef[:, c])), nl, qlo, nqo, p64(out))
        outs.append(gather(out, qper)[:nl])
    return outs[0], outs[1]


# ------------------------------------------------------------------------------ GPUs ----
def unique_id():
    """An NCCL unique id (128 bytes) made by the engine; rank 0 makes it, every rank passes it to
    init() (share it with torch.distributed.broadcast_object_list or any side channel)."""
    h = lib()
    h.fhe_dist_unique_id.restype = C.c_int
    h.fhe_dist_unique_id.argtypes = [C.c_char_p]
    buf = C.create_string_buffer(128)
    _check(h.fhe_dist_unique_id(buf))
    return buf.raw


def init(ctx, world, rank, uid):
    """Join the context to a limb-partitioned group of `world` GPUs (one context per rank)."""
    if len(uid) != 128:
        raise FheError(-1, "unique id must be 128 bytes")
    h = lib()
    h.fhe_dist_init.restype = C.c_int
    h.fhe_dist_init.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_char_p]
    _check(h.fhe_dist_init(ctx.h, world, rank, uid))


def keyswitch(ctx, which, d_own_ptr, level, out0_ptr, out1_ptr):
    """fhe_keyswitch_dist on device buffers: the rank's own Q limbs of d in, its own limbs of the
    result out (limb_block(L - level, world, rank) gives their first index and count)."""
    h = lib()
    h.fhe_keyswitch_dist.restype = C.c_int
    h.fhe_keyswitch_dist.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
    _check(h.fhe_keyswitch_dist(ctx.h, which, d_own_ptr, level, out0_ptr, out1_ptr))
