"""A plaintext slot-vector stand-in for fhessm.CryptoContext's operator surface (CPU test
infrastructure).

Circuits written against the engine's Python mirror (rotations, per-slot plaintext products,
ciphertext products, the BSGS matvec on D-slot lanes, Chebyshev series, bootstrapping) run here
on the slot vectors themselves, with the levels counted the way the engine counts them and its
level rules enforced (a ciphertext sum lands at the lower of the two levels, as the engine's
reconciling EvalAdd does; a plaintext is added at the ciphertext's level; a rescaling product
needs a level left; align only downwards).  Scales are not kept, so the level the engine spends
on equal-level operands with unrelated scales is not counted here.  What this checks is the
circuit's data movement and level bookkeeping: a layout or rotation mistake gives a wrong
vector, a level mistake an exception.  The numerics of the encrypted path are the GPU tests'
business."""
import numpy as np


class SimCt:
    def __init__(self, z, level, scale=1.0):
        self.z = np.asarray(z, dtype=np.float64)
        self.level = level
        self.scale = scale


class SimPt(SimCt):
    pass


class SimPlan:
    def __init__(self, W, D):
        self.W, self.D = W, D


class SimContext:
    """slots, L and the bootstrap's output level as the engine's; a degree-d Chebyshev series
    is counted at ceil(log2(d + 1)) + 1 levels, at least what the engine's evaluation takes."""

    def __init__(self, slots, L=34, boot_level=17):
        self.slots, self.L, self.boot_level = slots, L, boot_level
        self.rotation_keys = set()
        self.mv_keys = set()
        self.bootstraps = 0
        self.rotations = 0

    # helpers -----------------------------------------------------------------------------------
    def _tile(self, values):
        v = np.asarray(values)
        if np.iscomplexobj(v):
            assert np.abs(v.imag).max() == 0.0
            v = v.real
        v = np.asarray(v, dtype=np.float64).ravel()
        assert self.slots % len(v) == 0, "a slot vector's length must divide the slots"
        return np.tile(v, self.slots // len(v))

    def _need(self, ct, k, what):
        if self.L - ct.level - 1 < k:
            raise RuntimeError(f"{what}: no level left (level {ct.level})")

    # keys ----------------------------------------------------------------------------------------
    def EvalRotateKeyGen(self, steps):
        self.rotation_keys |= {int(s) % self.slots for s in steps}

    def matvec_keygen(self, D, b1):
        self.mv_keys.add(D)

    # encode / encrypt -----------------------------------------------------------------------------
    def MakeCKKSPackedPlaintext(self, values, level=0, scale=0.0):
        return SimPt(self._tile(values), level, scale)

    def Encrypt(self, pt):
        return SimCt(pt.z.copy(), pt.level, pt.scale)

    def Decrypt(self, ct):
        return ct.z.copy()

    def Copy(self, ct):
        return SimCt(ct.z.copy(), ct.level, ct.scale)

    # arithmetic ----------------------------------------------------------------------------------
    def EvalAdd(self, a, b):
        if isinstance(b, SimPt) and a.level != b.level:
            raise RuntimeError(f"add: ciphertext at level {a.level}, plaintext at {b.level}")
        return SimCt(a.z + b.z, max(a.level, b.level))

    def EvalSub(self, a, b):
        return SimCt(a.z - b.z, max(a.level, b.level))

    def EvalAddConst(self, a, v):
        return SimCt(a.z + v, a.level)

    def EvalRotate(self, ct, k):
        if int(k) % self.slots not in self.rotation_keys:
            raise RuntimeError(f"rotate: no key for step {k}")
        self.rotations += 1
        return SimCt(np.roll(ct.z, -int(k)), ct.level)   # slot s receives slot s + k

    def EvalFastRotation(self, ct, ks):
        return [self.EvalRotate(ct, k) for k in ks]

    def EvalRotateSum(self, cts, ks):
        if len({c.level for c in cts}) != 1:
            raise RuntimeError("rotate_sum: inputs at different levels")
        out = self.EvalRotate(cts[0], ks[0])
        for c, k in zip(cts[1:], ks[1:]):
            out = SimCt(out.z + self.EvalRotate(c, k).z, out.level)
        return out

    def align(self, ct, level):
        if level < ct.level:
            raise RuntimeError("align: only downwards")
        ct.level = level

    def mul_vec_rescale(self, ct, values):
        self._need(ct, 1, "mul_vec_rescale")
        return SimCt(ct.z * self._tile(values), ct.level + 1)

    def mul_rescale(self, a, b):
        lv = max(a.level, b.level)
        self._need(SimCt(None, lv), 1, "mul_rescale")
        return SimCt(a.z * b.z, lv + 1)

    def EvalChebyshevSeries(self, ct, coeffs):
        d = len(coeffs) - 1
        depth = int(np.ceil(np.log2(d + 1))) + 1
        self._need(ct, depth, "chebyshev")
        return SimCt(np.polynomial.chebyshev.chebval(ct.z, np.asarray(coeffs, dtype=np.float64)), ct.level + depth)

    def EvalBootstrap(self, ct):
        self.bootstraps += 1
        return SimCt(ct.z.copy(), self.boot_level)

    def EvalBootstrapBatch(self, cts):
        return [self.EvalBootstrap(c) for c in cts]

    # the BSGS matvec on D-slot lanes ------------------------------------------------------------
    def matvec_plan(self, W, D, b1):
        W = np.asarray(W, dtype=np.float64)
        assert W.shape[0] <= D and W.shape[1] % D == 0
        return SimPlan(W, D)

    def matvec(self, plan, inputs):
        D, W = plan.D, plan.W
        if D not in self.mv_keys:
            raise RuntimeError(f"matvec: no keys for D = {D}")
        if len({c.level for c in inputs}) != 1:
            raise RuntimeError("matvec: inputs at different levels")
        self._need(inputs[0], 1, "matvec")
        X = [c.z.reshape(-1, D) for c in inputs]          # (lanes, D) each
        Y = np.zeros_like(X[0])
        for s, x in enumerate(X):
            Y[:, : W.shape[0]] += x @ W[:, s * D:(s + 1) * D].T
        return SimCt(Y.ravel(), inputs[0].level + 1)
