"""fhessm.rwkv7 -- the RWKV-7 (x070) polynomial model of config 5, in recurrent form.

The reference holds this model only as a plaintext PyTorch harness
(results/vector-d-20261104/harness/rwkv7_model.py, the x070 forward with every non-polynomial
operation routed through one site hook); its encrypted port is not in the reference tree.  This
module restates that forward one token at a time for a batch of conversations, in float64:

  * ``RWKV7Shape`` and ``synthetic_weights``: the parameter set under the reference's
    state-dict names (rwkv7_model.py:234-306), seeded;
  * ``step``: one token through every block and the output norm, with the sites evaluated
    exactly or as the circuit evaluates them (``Sites``: Chebyshev polynomials on fitted
    intervals, Newton inverse square roots from a linear seed), carrying the per-layer state
    (the two time-shift inputs and the per-head wkv matrix);
  * ``fit_sites``: the polynomial of every site from a calibration run.

Per layer (rwkv7_model.py:329-392): x0 = ln1(x); time shift xx = prev - x0; six mixes
x_* = x0 + xx m_*; r, k, v linear; decay w = exp(-e^{-1/2} sigmoid(w0 + tanh(x_w W1) W2));
value residual v += (v_first - v) sigmoid(v0 + (x_v V1) V2) from layer 1 on; in-context rate
a = sigmoid(a0 + (x_a A1) A2); gate g = sigmoid(x_g G1) G2; kk = normalize(k k_k) per head;
k <- k (1 + (a - 1) k_a); the state S <- S diag(w) + (S (-kk)) (kk a)^T + v k^T, y = S r
(wkv7_recurrence, :277-298); GroupNorm per head, the bonus ((r k r_k) summed per head) v, the
output projection of y g; then the channel mix relu(x_k Wk)^2 Wv on ln2 with its own time shift.
"""
from dataclasses import dataclass

import numpy as np

EXP_M05 = float(np.exp(-0.5))


@dataclass
class RWKV7Shape:
    n_layer: int = 24
    n_embd: int = 1024
    head_size: int = 64
    d_decay: int = 64
    d_aaa: int = 64
    d_mv: int = 32
    d_gate: int = 128
    dim_ffn: int = 4096
    vocab_size: int = 65536

    @property
    def n_head(self):
        return self.n_embd // self.head_size


RWKV7_04B = RWKV7Shape()   # config 5: 24 layers, d = 1024, head size 64, V = 65,536


def synthetic_weights(sh: RWKV7Shape, seed: int = 7):
    """Seeded parameters under the reference's state-dict names: norm gains near 1, mixes in
    [0, 1), matrices N(0, 1/fan_in), decay bias around -1 (rwkv7_model.py:234-306)."""
    rng = np.random.default_rng(seed)
    C, H, N, F = sh.n_embd, sh.n_head, sh.head_size, sh.dim_ffn
    mat = lambda o, i: rng.normal(0.0, 1.0 / np.sqrt(i), (o, i))      # a Linear's (out, in) weight
    lora = lambda i, o, s=1.0: rng.normal(0.0, s / np.sqrt(i), (i, o))   # x @ W with W (in, out)
    w = {"emb.weight": rng.normal(0.0, 0.5, (sh.vocab_size, C)),
         "ln_out.weight": 1.0 + 0.1 * rng.normal(size=C), "ln_out.bias": 0.1 * rng.normal(size=C),
         "head.weight": mat(sh.vocab_size, C)}
    for i in range(sh.n_layer):
        p = f"blocks.{i}."
        if i == 0:
            w[p + "ln0.weight"] = 1.0 + 0.1 * rng.normal(size=C)
            w[p + "ln0.bias"] = 0.1 * rng.normal(size=C)
        for ln in ("ln1", "ln2"):
            w[p + ln + ".weight"] = 1.0 + 0.1 * rng.normal(size=C)
            w[p + ln + ".bias"] = 0.1 * rng.normal(size=C)
        a = p + "att."
        for m in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"):
            w[a + m] = rng.uniform(0.0, 1.0, C)
        w[a + "w0"] = -1.0 + 0.5 * rng.normal(size=C)
        w[a + "w1"], w[a + "w2"] = lora(C, sh.d_decay), lora(sh.d_decay, C, 0.5)
        w[a + "a0"] = 0.5 * rng.normal(size=C)
        w[a + "a1"], w[a + "a2"] = lora(C, sh.d_aaa), lora(sh.d_aaa, C, 0.5)
        if i > 0:
            w[a + "v0"] = 0.5 * rng.normal(size=C)
            w[a + "v1"], w[a + "v2"] = lora(C, sh.d_mv), lora(sh.d_mv, C, 0.5)
        w[a + "g1"], w[a + "g2"] = lora(C, sh.d_gate), lora(sh.d_gate, C, 0.5)
        w[a + "k_k"] = 0.8 + 0.2 * rng.uniform(size=C)
        w[a + "k_a"] = rng.uniform(size=C)
        w[a + "r_k"] = 0.5 * rng.normal(size=(H, N))
        for lin in ("receptance", "key", "value", "output"):
            w[a + lin + ".weight"] = mat(C, C)
        w[a + "ln_x.weight"] = 1.0 + 0.1 * rng.normal(size=C)
        w[a + "ln_x.bias"] = 0.1 * rng.normal(size=C)
        f = p + "ffn."
        w[f + "x_k"] = rng.uniform(0.0, 1.0, C)
        w[f + "key.weight"] = mat(F, C)
        w[f + "value.weight"] = mat(C, F) * 0.5
    return w


# -------------------------------------------------------------------------------- sites ----
SITE_FUNCS = {   # rwkv7_model.py:46-56
    "w_tanh": np.tanh,
    "decay": lambda x: np.exp(-EXP_M05 / (1.0 + np.exp(-x))),
    "v_sigmoid": lambda x: 1.0 / (1.0 + np.exp(-x)),
    "a_sigmoid": lambda x: 1.0 / (1.0 + np.exp(-x)),
    "g_sigmoid": lambda x: 1.0 / (1.0 + np.exp(-x)),
    "relu2": lambda x: np.maximum(x, 0.0) ** 2,
}
RSQRT_EPS = {"ln": 1e-5, "gn": 64e-5, "kk": 0.0}


def cheb_fit(f, lo, hi, degree):
    """Chebyshev interpolant of f on [lo, hi] (Chebyshev nodes of the first kind), coefficients
    in the variable t = (2x - lo - hi) / (hi - lo) (rwkv7_model.py:113-127 evaluates the same
    series by Clenshaw)."""
    n = degree + 1
    t = np.cos(np.pi * (np.arange(n) + 0.5) / n)
    fx = f(0.5 * (hi - lo) * t + 0.5 * (hi + lo))
    c = np.array([2.0 / n * np.sum(fx * np.cos(np.pi * j * (np.arange(n) + 0.5) / n)) for j in range(n)])
    c[0] /= 2.0
    return c


def cheb_val(x, c, lo, hi):
    t = (2.0 * x - (lo + hi)) / (hi - lo)
    return np.polynomial.chebyshev.chebval(t, c)


class Sites:
    """Exact site functions (fits None), or the circuit's: a Chebyshev series per site kind and
    block on its interval, and Newton 1/sqrt from a linear seed per norm site.  record=True keeps
    the input range of every site (calibration)."""

    def __init__(self, fits=None, record=False):
        self.fits = fits
        self.record = record
        self.ranges = {}

    def _rec(self, name, x):
        if self.record:
            x = np.asarray(x)
            x = x[np.isfinite(x)]     # a diverged site (calibration with fitted sites) adds nothing
            if x.size == 0:
                return
            lo, hi = self.ranges.get(name, (np.inf, -np.inf))
            self.ranges[name] = (min(lo, float(np.min(x))), max(hi, float(np.max(x))))

    def poly(self, name, kind, x):
        self._rec(name, x)
        if self.fits is None or name not in self.fits:
            return SITE_FUNCS[kind](x)
        lo, hi, c = self.fits[name]
        return cheb_val(x, c, lo, hi)

    def rsqrt(self, name, kind, x):
        """1/sqrt(x + eps) (kk: 1/max(sqrt(x), 1e-12))"""
        v = x + RSQRT_EPS[kind]
        self._rec(name, v)
        if self.fits is None or name not in self.fits:
            return 1.0 / np.maximum(np.sqrt(np.maximum(v, 0.0)), 1e-12) if kind == "kk" else 1.0 / np.sqrt(v)
        a, b, steps = self.fits[name]
        y = a + b * v
        for al, be in steps:
            y = y * (al - be * v * y * y)
        return y


def _ln(sites, name, x, wgt, bias):
    mu = x.mean(-1, keepdims=True)
    xc = x - mu
    var = (xc * xc).mean(-1, keepdims=True)
    return xc * sites.rsqrt(name, "ln", var) * wgt + bias


def new_state(sh: RWKV7Shape, lanes: int):
    C, H, N = sh.n_embd, sh.n_head, sh.head_size
    return [{"att": np.zeros((lanes, C)), "ffn": np.zeros((lanes, C)), "S": np.zeros((lanes, H, N, N))}
            for _ in range(sh.n_layer)]


def block_step(sh: RWKV7Shape, w, i, x, st, v_first, sites, ln0=True):
    """One block for one token: x (lanes, C) -> (x', v_first); st (the block's state) is updated.
    ln0=False: x is already through block 0's input norm (the client applies it before encrypting,
    the reference folds it into the embedding table)."""
    B, C = x.shape
    H, N = sh.n_head, sh.head_size
    p = f"blocks.{i}."
    a_ = p + "att."
    if i == 0 and ln0:
        x = _ln(sites, p + "ln0", x, w[p + "ln0.weight"], w[p + "ln0.bias"])
    x0 = _ln(sites, p + "ln1", x, w[p + "ln1.weight"], w[p + "ln1.bias"])
    xx = st["att"] - x0
    st["att"] = x0
    xr, xw, xk, xv, xa, xg = (x0 + xx * w[a_ + m] for m in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g"))
    r = xr @ w[a_ + "receptance.weight"].T
    z = w[a_ + "w0"] + sites.poly(a_ + "w_tanh", "w_tanh", xw @ w[a_ + "w1"]) @ w[a_ + "w2"]
    dec = sites.poly(a_ + "decay", "decay", z)
    k = xk @ w[a_ + "key.weight"].T
    v = xv @ w[a_ + "value.weight"].T
    if i == 0:
        v_first = v
    else:
        v = v + (v_first - v) * sites.poly(a_ + "v_sigmoid", "v_sigmoid", w[a_ + "v0"] + (xv @ w[a_ + "v1"]) @ w[a_ + "v2"])
    a = sites.poly(a_ + "a_sigmoid", "a_sigmoid", w[a_ + "a0"] + (xa @ w[a_ + "a1"]) @ w[a_ + "a2"])
    g = sites.poly(a_ + "g_sigmoid", "g_sigmoid", xg @ w[a_ + "g1"]) @ w[a_ + "g2"]
    kk = (k * w[a_ + "k_k"]).reshape(B, H, N)
    kk = (kk * sites.rsqrt(a_ + "kk_rsqrt", "kk", (kk * kk).sum(-1, keepdims=True))).reshape(B, C)
    k = k * (1.0 + (a - 1.0) * w[a_ + "k_a"])
    # wkv7 state update, one step (rwkv7_model.py:290-296): S <- S diag(w) + (S (-kk)) (kk a)^T + v k^T
    S = st["S"]
    dh, kh, vh, rh = (t.reshape(B, H, N) for t in (dec, k, v, r))
    ah, bh = -kk.reshape(B, H, N), (kk * a).reshape(B, H, N)
    Sa = np.einsum("bhij,bhj->bhi", S, ah)
    S = S * dh[:, :, None, :] + Sa[..., :, None] * bh[:, :, None, :] + vh[..., :, None] * kh[:, :, None, :]
    st["S"] = S
    y = np.einsum("bhij,bhj->bhi", S, rh)
    yc = y - y.mean(-1, keepdims=True)
    var = (yc * yc).mean(-1, keepdims=True)
    y = (yc * sites.rsqrt(a_ + "gn_rsqrt", "gn", var)).reshape(B, C) * w[a_ + "ln_x.weight"] + w[a_ + "ln_x.bias"]
    y = y + ((rh * kh * w[a_ + "r_k"]).sum(-1, keepdims=True) * vh).reshape(B, C)
    x = x + (y * g) @ w[a_ + "output.weight"].T
    f = p + "ffn."
    xf = _ln(sites, p + "ln2", x, w[p + "ln2.weight"], w[p + "ln2.bias"])
    xx = st["ffn"] - xf
    st["ffn"] = xf
    kf = (xf + xx * w[f + "x_k"]) @ w[f + "key.weight"].T
    x = x + sites.poly(f + "relu2", "relu2", kf) @ w[f + "value.weight"].T
    return x, v_first


def step(sh: RWKV7Shape, w, tokens, state, sites=None, hidden=None):
    """One token per conversation through every block: tokens (lanes,) -> logits (lanes, V).
    state is new_state(...) and is updated in place; hidden (a list) collects each block's output."""
    sites = sites or Sites()
    x = w["emb.weight"][np.asarray(tokens)].astype(np.float64)
    v_first = None
    for i in range(sh.n_layer):
        x, v_first = block_step(sh, w, i, x, state[i], v_first, sites)
        if hidden is not None:
            hidden.append(x.copy())
    x = _ln(sites, "ln_out", x, w["ln_out.weight"], w["ln_out.bias"])
    return x @ w["head.weight"].T


def _site_ranges(sh: RWKV7Shape, w, token_batches, fits):
    rec = Sites(fits, record=True)
    st = new_state(sh, len(token_batches[0]))
    for t in token_batches:
        step(sh, w, t, st, rec)
    return rec.ranges


def fit_sites(sh: RWKV7Shape, w, token_batches, degree=15, margin=0.1, tol=1e-4, seed_margin=(1.25, 2.0), rounds=1):
    """Polynomial sites from a calibration run: every Chebyshev site on its observed interval
    widened by `margin` of its width (the harness's fit.py does the same per site), every norm
    site a linear seed with the tuned Newton steps that reach `tol` on [m / lo, M * hi].  With
    rounds > 1 the model is run again with the fitted sites and every site refitted on the union
    of the ranges seen so far: the polynomial model's own trajectory leaves the exact model's
    ranges (most at low degree), and a Newton seed above its window diverges."""
    ranges = _site_ranges(sh, w, token_batches, None)
    fits = _fit_ranges(ranges, degree, margin, tol, seed_margin)
    for _ in range(rounds - 1):
        more = _site_ranges(sh, w, token_batches, fits)
        ranges = {k: (min(lo, more.get(k, (lo, hi))[0]), max(hi, more.get(k, (lo, hi))[1]))
                  for k, (lo, hi) in ranges.items()}
        fits = _fit_ranges(ranges, degree, margin, tol, seed_margin)
    return fits


def newton_steps(a, b, m0, m1, tol, cap=40, widen=0.02):
    """Coefficients (alpha_k, beta_k) of y <- y (alpha_k - beta_k v y^2), each the minimax choice
    for the range of t = y sqrt(v) left by the steps before, from the linear seed y = a + b v on
    [m0, m1], until t is within tol of 1.  With t in [l, h] the map g(t) = alpha t - beta t^3
    equioscillates at l, its maximum t* = sqrt((h^2 + h l + l^2) / 3) and h:
        beta = 2 / ((2/3) t* S + l h (h + l)),  alpha = beta S,  S = h^2 + h l + l^2,
    and the next range is [g(l), g(t*)].  Standard Newton is alpha = 3/2, beta = 1/2, the best
    choice only near t = 1; far below it grows t by 1.5 a step where this grows it by up to 2.6
    (a window spanning six decades: 10 steps against 17).  Every range is widened by `widen` on
    both sides before its step is chosen, until t is within 5 % of 1."""
    v = np.geomspace(m0, m1, 4001)
    t = (a + b * v) * np.sqrt(v)
    l, h = float(t.min()), float(t.max())
    steps = []
    while max(1.0 - l, h - 1.0) > tol and len(steps) < cap:
        l, h = l * (1.0 - widen), h * (1.0 + widen)
        S = h * h + h * l + l * l
        ts = np.sqrt(S / 3.0)
        be = 2.0 / ((2.0 / 3.0) * ts * S + l * h * (h + l))
        al = be * S
        steps.append((al, be))
        l, h = al * l - be * l ** 3, al * ts - be * ts ** 3
        widen = 0.0 if max(1.0 - l, h - 1.0) < 0.05 else widen
    return np.array(steps).reshape(-1, 2)


def _fit_ranges(ranges, degree, margin, tol, seed_margin):
    from .model import linear_rsqrt_seed
    fits = {}
    for name, (lo, hi) in ranges.items():
        kind = name.split(".")[-1]
        if name.endswith(("ln0", "ln1", "ln2", "ln_out", "gn_rsqrt", "kk_rsqrt")):
            # the wkv readout's variance reaches eps on a cold state: the window spans decades
            m0, m1 = max(lo, 1e-12) / seed_margin[0], hi * seed_margin[1]
            a, b = linear_rsqrt_seed(m0, m1)
            fits[name] = (a, b, newton_steps(a, b, m0, m1, tol))
            continue
        pad = margin * (hi - lo) + 1e-6
        fits[name] = (lo - pad, hi + pad, cheb_fit(SITE_FUNCS[kind], lo - pad, hi + pad, degree))
    return fits


# ----------------------------------------------------------------- the encrypted wkv state ----
class EncryptedWkv:
    """The x070 state update on the engine for ``blocks`` head blocks (conversation l, head h:
    block b = l H + h), every vector in the contiguous channel layout (block b's channel j at
    slot b N + j).  The state is N ciphertexts, one per row index: row ciphertext i holds row i of
    every block's N x N matrix, S_b[i][j] at slot b N + j, so that the state update needs no
    change of layout:

      * S diag(w): a slot product of every row ciphertext with w;
      * (S a) b^T: row i's per-block sum of S_i (.) a (log2 N doublings by -1 and a mask leave
        it at the block's last slot; log2 N doublings by +1 spread it over the block) times b;
      * v k^T: v[i] of every block over the block (v rotated left by i, all i from one hoisted
        rotation, the first-slot mask, log2 N doublings by -1) times k;
      * the readout y[i] = (S' r)[i], taken from the old rows (below): row i's per-block sums at
        the block's last slot, moved to slot i by a left rotation of N - 1 - i; the N moves are
        one batched rotate-and-sum.

    One step (wkv7_recurrence, rwkv7_model.py:290-296, with a = -kk and b = kk a):
        S_i <- S_i (.) w + spread(sum(S_i (.) a)) (.) b + bcast_i(v) (.) k,
        y_i  = sum_j S_i[j] w_j r_j + (S a)_i (b . r) + v_i (k . r).
    Every product is a relinearised, rescaled ciphertext product (mul_rescale), every mask a
    plaintext product; the engine's EvalAdd reconciles levels and scales.  A row spends 3 levels
    a step (S' and y both 3 below S).  Only left rotations by 1 .. N - 1 and +-2^t are used: the
    hoisted broadcasts, the readout moves and the BSGS babies share their keys."""

    def __init__(self, cx, N=64, blocks=1):
        if cx.slots % N or blocks * N > cx.slots:
            raise ValueError("the contiguous layout needs N | slots and blocks * N <= slots")
        self.cx, self.N, self.blocks = cx, N, blocks
        self.lg = int(np.log2(N))
        first, last = np.zeros(cx.slots), np.zeros(cx.slots)
        first[: blocks * N: N] = 1.0
        last[N - 1: blocks * N: N] = 1.0
        self.first, self.last = first, last   # the first and last slot of every block in use

    @staticmethod
    def rotations(N=64):
        r = set(range(1, N))
        for t in range(int(np.log2(N))):
            r |= {1 << t, -(1 << t)}
        return sorted(r)

    # layout helpers --------------------------------------------------------------------------
    def pack_state(self, S):
        """S (blocks, N, N) -> N slot vectors (row i of every block)"""
        S = np.asarray(S, dtype=np.float64)
        out = []
        for i in range(self.N):
            z = np.zeros(self.cx.slots)
            z[: self.blocks * self.N] = S[:, i, :].ravel()
            out.append(z)
        return out

    def pack_channel(self, v):
        """v (blocks, N) -> slot vector"""
        z = np.zeros(self.cx.slots)
        z[: self.blocks * self.N] = np.asarray(v, dtype=np.float64).ravel()
        return z

    def unpack_channel(self, z):
        return np.asarray(z).real[: self.blocks * self.N].reshape(self.blocks, self.N)

    def unpack_state(self, rows):
        """N decrypted row vectors -> (blocks, N, N)"""
        return np.stack([self.unpack_channel(z) for z in rows], axis=1)

    # moves -------------------------------------------------------------------------------------
    def _doubling(self, ct, step):
        cx = self.cx
        for t in range(self.lg):
            ct = cx.EvalAdd(ct, cx.EvalRotate(ct, step << t))
        return ct

    def block_sum(self, ct, scale=1.0):
        """scale * sum_j ct[b N + j] in every slot of block b (one level)"""
        s = self.cx.mul_vec_rescale(self._doubling(ct, 1), scale * self.first)
        return self._doubling(s, -1)

    def last_sum(self, ct):
        """sum_j ct[b N + j] at the block's last slot, zeros elsewhere (one level)"""
        return self.cx.mul_vec_rescale(self._doubling(ct, -1), self.last)

    def step(self, S, w, a, b, k, r, v):
        """(S', y) for the row ciphertexts S and the channel-layout inputs (y in the channel
        layout)"""
        cx, N = self.cx, self.N
        vrot = [v] + cx.EvalFastRotation(v, list(range(1, N)))
        wr = cx.mul_rescale(w, r)
        br = self.block_sum(cx.mul_rescale(b, r))   # b . r over each block
        kr = self.block_sum(cx.mul_rescale(k, r))
        S2, heads = [], []
        for i in range(N):
            sa = self.last_sum(cx.mul_rescale(S[i], a))        # (S a)_i at the block's last slot
            vi = cx.mul_vec_rescale(vrot[i], self.first)        # v_i at the block's first slot
            sw = cx.mul_rescale(S[i], w)
            sab = cx.mul_rescale(self._doubling(sa, 1), b)      # the last slot spread down the block
            vk = cx.mul_rescale(self._doubling(vi, -1), k)      # the first slot spread up the block
            S2.append(cx.EvalAdd(cx.EvalAdd(sw, sab), vk))
            heads.append(cx.EvalAdd(self.last_sum(cx.mul_rescale(S[i], wr)), cx.mul_rescale(sa, br)))
        lv = max(h.level for h in heads)   # the rotate-and-sum's inputs share one level and scale
        for h in heads:
            if h.level < lv:
                cx.align(h, lv)
        y = cx.EvalAdd(cx.EvalRotateSum(heads[:N - 1], [N - 1 - i for i in range(N - 1)]), heads[N - 1])
        return S2, cx.EvalAdd(y, cx.mul_rescale(v, kr))


# ------------------------------------------------------------------ the encrypted RWKV-7 block ----
class EncryptedRWKV7Block:
    """One RWKV-7 block (time mix with the wkv state, channel mix) on the engine for ``convs``
    conversations of C = H N channels (H heads of N), with the circuit's sites (``fits``:
    Chebyshev series, Newton 1/sqrt), against which ``block_step(..., Sites(fits))`` is the
    float64 mirror.  Every vector is in the contiguous layout: conversation l's channel c at slot
    l C + c (head block b = l H + h at slots b N .. b N + N - 1).  This is the engine's matvec
    layout with D = C, so every linear layer is one BSGS matvec (LoRA matrices padded to C x C);
    a per-head sum (kk normalisation, GroupNorm, the bonus) is log2 N doublings by +1, a mask at
    the head's first slot and log2 N doublings by -1, a per-conversation sum (LayerNorm) the same
    over C.  The wkv state is EncryptedWkv's N row ciphertexts in the same layout, so nothing
    changes layout inside the block.  A ciphertext is bootstrapped when it has fewer levels left
    than the next operation needs (the state rows together, in one batched bootstrap)."""

    # The wkv state reaches |S| ~ 10, its readout |y| ~ 50 and the attention output before the
    # gate ~ 20; at the bootstrap's default input scale (2^49 over a 60-bit q0) the sine's
    # curvature costs (2 pi |m| / 2^11)^2 / 6 of a value m, 4e-3 at 50.  Each can be carried
    # scaled down, for free (every factor folded into a plaintext the circuit multiplies anyway):
    #   * the state / S_SCALE: key weights / S_SCALE (v k^T and so the whole recurrence scale
    #     with it; kk's normalisation takes S_SCALE back in its k_k product);
    #   * the readout by 1 / (Y_SCALE S_SCALE): receptance weights / Y_SCALE; GroupNorm takes the
    #     factor back squared in the variance's block-sum mask (Newton runs on the true variance,
    #     its iterate at 1/sqrt(var + eps)) and once in ln_x's weight;
    #   * the normed output / G_SCALE: ln_x weight and bias and the bonus / G_SCALE, the gate's
    #     G2 * G_SCALE.
    # A bootstrap's error is absolute, though: scaling a value down multiplies it, in the value's
    # own units, by the factor, and GroupNorm then divides by the head's deviation.  At the 0.4B
    # shape (24 layers, 32 conversations) S_SCALE = Y_SCALE = G_SCALE = 4 ran the error up by
    # 1e-4 a layer and a lane out of a Newton window at layer 12; G_SCALE = 4 alone measured
    # logits relErrRms 1.7-2.8e-3 against 0.8-1.1e-3 with no scaling.  The factors stay at 1.
    S_SCALE, Y_SCALE, G_SCALE = 1.0, 1.0, 1.0

    def __init__(self, cx, sh: RWKV7Shape, w, layer, fits, convs=1, b1=8):
        C, N = sh.n_embd, sh.head_size
        if cx.slots % C or convs * C > cx.slots:
            raise ValueError("the contiguous layout needs C | slots and convs * C <= slots")
        self.cx, self.sh, self.w, self.layer, self.fits = cx, sh, w, layer, fits
        self.C, self.N, self.H, self.convs = C, N, sh.n_head, convs
        self.wkv = EncryptedWkv(cx, N, convs * self.H)
        self.lane_mask = np.zeros(cx.slots)
        self.lane_mask[: convs * C] = 1.0
        p = f"blocks.{layer}."
        self.p, self.a_ = p, p + "att."
        a_ = self.a_
        pad = lambda M: np.pad(M, ((0, C - M.shape[0]), (0, C - M.shape[1])))
        plan = lambda M: cx.matvec_plan(M, C, b1)
        self.plans = {
            "r": plan(w[a_ + "receptance.weight"] / self.Y_SCALE),
            "k": plan(w[a_ + "key.weight"] / self.S_SCALE),
            "v": plan(w[a_ + "value.weight"]), "o": plan(w[a_ + "output.weight"]),
            "w1": plan(pad(w[a_ + "w1"].T)), "w2": plan(pad(w[a_ + "w2"].T)),
            "a1": plan(pad(w[a_ + "a1"].T)), "a2": plan(pad(w[a_ + "a2"].T)),
            "g1": plan(pad(w[a_ + "g1"].T)), "g2": plan(pad(w[a_ + "g2"].T) * self.G_SCALE),
        }
        self.mid = {"w1": sh.d_decay, "a1": sh.d_aaa, "g1": sh.d_gate}
        if layer > 0:
            self.plans["v1"] = plan(pad(w[a_ + "v1"].T))
            self.plans["v2"] = plan(pad(w[a_ + "v2"].T))
            self.mid["v1"] = sh.d_mv
        F = sh.dim_ffn
        if F % C:
            raise ValueError("dim_ffn must be a multiple of n_embd")
        kf, vf = w[p + "ffn.key.weight"], w[p + "ffn.value.weight"]
        self.ffn_k = [plan(kf[c * C:(c + 1) * C]) for c in range(F // C)]
        self.ffn_v = plan(vf)                          # (C, F): column chunk s acts on input s
        self.state = None                              # (prev_att, prev_ffn, [state rows]) ciphertexts
        self.bootstraps = 0

    @staticmethod
    def rotations(sh: RWKV7Shape, slots=None):
        """the rotation steps the block uses"""
        r = set(EncryptedWkv.rotations(sh.head_size))
        for t in range(int(np.log2(sh.n_embd))):
            r |= {1 << t, -(1 << t)}
        return sorted(r)

    # packing -------------------------------------------------------------------------------------
    def pack(self, x):
        """x (convs, C) -> the contiguous slot vector"""
        z = np.zeros(self.cx.slots)
        z[: self.convs * self.C] = np.asarray(x, dtype=np.float64).ravel()
        return z

    def unpack(self, z):
        return np.asarray(z).real[: self.convs * self.C].reshape(self.convs, self.C)

    def tile(self, v):
        """a per-channel vector on every conversation in use, zeros elsewhere"""
        z = np.zeros(self.cx.slots)
        z[: self.convs * self.C] = np.tile(np.asarray(v, dtype=np.float64).ravel(), self.convs)
        return z

    def every(self, period, scale, first=1):
        """scale at the first ``first`` slots of every block of ``period`` slots in use"""
        z = np.zeros(self.cx.slots)
        for s in range(0, self.convs * self.C, period):
            z[s:s + first] = scale
        return z

    # level management and arithmetic --------------------------------------------------------------
    def left(self, ct):
        return self.cx.L - ct.level - 1

    def boot(self, ct):
        self.bootstraps += 1
        return self.cx.EvalBootstrap(ct)

    def ensure(self, ct, k):
        if self.left(ct) < k:
            return self.boot(ct)
        return ct

    def add(self, a, b):
        return self.cx.EvalAdd(a, b)

    def sub(self, a, b):
        return self.cx.EvalSub(a, b)

    def mulv(self, ct, v):
        return self.cx.mul_vec_rescale(self.ensure(ct, 1), self.tile(v))

    def mask(self, ct, m):
        return self.cx.mul_vec_rescale(self.ensure(ct, 1), m)

    def addv(self, ct, v):
        """ct + v (per channel) at ct's level and scale"""
        cx = self.cx
        return cx.EvalAdd(ct, cx.MakeCKKSPackedPlaintext(self.tile(v), level=ct.level, scale=ct.scale))

    def mulmul(self, a, b):
        """a * b, relinearised and rescaled; an operand without a level left is bootstrapped"""
        return self.cx.mul_rescale(self.ensure(a, 1), self.ensure(b, 1))

    def mulc(self, ct, c):
        """ct * c, rescaled onto the next level's canonical scale (a constant slot vector)"""
        return self.cx.mul_vec_rescale(self.ensure(ct, 1), np.full(8, float(c)))

    def mv(self, name, ct):
        return self.cx.matvec(self.plans[name], [self.ensure(ct, 2)])

    # circuit pieces -----------------------------------------------------------------------------
    def cheb(self, name, x, mask=None):
        """the site polynomial of `name` on x: [lo, hi] mapped to [-1, 1], the series, and a mask
        (the series' constant term lands in every slot; slots outside the conversations in use,
        or past a LoRA width, must stay zero for the sums and bootstraps that follow)"""
        cx = self.cx
        lo, hi, c = self.fits[name]
        depth = 3 + int(np.ceil(np.log2(len(c))))
        x = self.ensure(x, depth)
        t = self.mulc(x, 2.0 / (hi - lo))
        t = cx.EvalAddConst(t, -(lo + hi) / (hi - lo))
        return self.mask(cx.EvalChebyshevSeries(t, c), self.lane_mask if mask is None else mask)

    def newton(self, name, v):
        """the site's 1/sqrt(v) by its linear seed and tuned Newton steps (v: eps already added).
        Slots outside the conversations hold eps alone, where Newton would climb towards
        1/sqrt(eps) (40 for GroupNorm's) and a bootstrap of that range loses precision in every
        slot: the alpha y term carries the lane mask, which sends them to zero."""
        cx = self.cx
        a, b, steps = self.fits[name]
        v = self.ensure(v, 4)
        y = cx.EvalAddConst(self.mulc(v, b), a)
        for al, be in steps:   # y <- alpha y - beta v y^3
            if self.left(y) < 3:
                y = self.boot(y)
            if self.left(v) < 3:
                v = self.boot(v)
            y2 = self.mulmul(y, y)
            t = self.mulmul(self.mulc(v, -be), y)
            u = self.mulmul(t, y2)
            y = self.add(cx.mul_vec_rescale(y, al * self.lane_mask), u)
        return y

    def group_sum(self, x, width, scale):
        """scale * (the sum over each block of `width` slots) in every slot of the block"""
        cx = self.cx
        s = self.ensure(x, 1)
        for t in range(int(np.log2(width))):
            s = cx.EvalAdd(s, cx.EvalRotate(s, 1 << t))
        s = cx.mul_vec_rescale(s, self.every(width, scale))
        for t in range(int(np.log2(width))):
            s = cx.EvalAdd(s, cx.EvalRotate(s, -(1 << t)))
        return s

    def layer_norm(self, name, x, wgt, bias):
        cx, C = self.cx, self.C
        x = self.ensure(x, 4)
        xc = self.sub(x, self.group_sum(x, C, 1.0 / C))
        var = self.group_sum(self.mulmul(xc, xc), C, 1.0 / C)
        y = self.newton(name, cx.EvalAddConst(var, RSQRT_EPS["ln"]))
        xc = self.ensure(xc, 2)
        return self.addv(self.mulv(self.mulmul(xc, y), wgt), bias)

    def refresh(self, cts, k, batch=16):
        """the ciphertexts with fewer than k levels left bootstrapped, `batch` to a call"""
        low = [i for i, c in enumerate(cts) if self.left(c) < k]
        out = list(cts)
        self.bootstraps += len(low)
        for s in range(0, len(low), batch):
            part = low[s:s + batch]
            for i, c in zip(part, self.cx.EvalBootstrapBatch([cts[i] for i in part])):
                out[i] = c
        return out

    # the block ------------------------------------------------------------------------------------
    def step(self, x, v_first=None):
        """(x, v_first) -> (the block's output, v_first), both contiguous; v_first is None for
        block 0, which makes it.  x comes at most at the top of the chain's user region (with a
        bootstrapping chain the scales of the two regions are anchored separately, and products
        must not cross from one to the other)."""
        cx, w, a_, p, N, C, wkv = self.cx, self.w, self.a_, self.p, self.N, self.C, self.wkv
        if self.state is None:   # the cold state, at the input's level
            zero = cx.Encrypt(cx.MakeCKKSPackedPlaintext(np.zeros(cx.slots), level=x.level))
            self.state = [zero, cx.Copy(zero), [cx.Copy(zero) for _ in range(N)]]
        prev_att, prev_ffn, S = self.state
        mid = lambda name: self.every(C, 1.0, self.mid[name])
        # ---- time mix
        x0 = self.ensure(self.layer_norm(p + "ln1", x, w[p + "ln1.weight"], w[p + "ln1.bias"]), 6)
        xx = self.sub(prev_att, x0)
        mix = {m: self.ensure(self.add(x0, self.mulv(xx, w[a_ + m])), 6) for m in ("x_r", "x_w", "x_k", "x_v", "x_a", "x_g")}
        r = self.mv("r", mix["x_r"])
        k = self.mv("k", mix["x_k"])
        v = self.mv("v", mix["x_v"])
        if self.layer == 0:
            v_first = v
        else:   # v += (v_first - v) sigmoid(v0 + (x_v V1) V2)
            vm = self.cheb(a_ + "v_sigmoid", self.addv(self.mv("v2", self.mv("v1", mix["x_v"])), w[a_ + "v0"]))
            v = self.add(v, self.mulmul(self.sub(v_first, v), vm))
        wt = self.cheb(a_ + "w_tanh", self.mv("w1", mix["x_w"]), mid("w1"))
        dec = self.cheb(a_ + "decay", self.addv(self.mv("w2", wt), w[a_ + "w0"]))
        a = self.cheb(a_ + "a_sigmoid", self.addv(self.mv("a2", self.mv("a1", mix["x_a"])), w[a_ + "a0"]))
        gs = self.cheb(a_ + "g_sigmoid", self.mv("g1", mix["x_g"]), mid("g1"))
        g = self.mv("g2", gs)
        kk = self.mulv(k, w[a_ + "k_k"].ravel() * self.S_SCALE)
        kn = self.newton(a_ + "kk_rsqrt", self.group_sum(self.mulmul(kk, kk), N, 1.0))
        kk = self.mulmul(self.ensure(kk, 2), kn)
        a = self.ensure(a, 4)
        kmod = self.mulmul(k, self.addv(self.mulv(self.addv(a, -np.ones(C)), w[a_ + "k_a"].ravel()), np.ones(C)))
        b = self.mulmul(kk, a)
        na = self.mulc(kk, -1.0)
        # ---- the wkv state
        S = self.refresh(S, 3)
        # an input deeper than the rows would take the rows down with it (64 bootstraps a refresh)
        k_in = max(3, min(self.left(c) for c in S))
        ins = [self.ensure(c, k_in) for c in (dec, na, b, kmod, r, v)]
        S, y = wkv.step(S, *ins)
        # GroupNorm per head (7 levels: the variance, up to a few hundred, must reach Newton with
        # the 4 it needs and no bootstrap of its own)
        y = self.ensure(y, 7)
        yc = self.sub(y, self.group_sum(y, N, 1.0 / N))
        ys = self.Y_SCALE * self.S_SCALE
        var = self.group_sum(self.mulmul(yc, yc), N, ys ** 2 / N)   # the true variance
        gn = self.newton(a_ + "gn_rsqrt", cx.EvalAddConst(var, RSQRT_EPS["gn"]))
        yc = self.ensure(yc, 3)
        y = self.addv(self.mulv(self.mulmul(yc, gn), w[a_ + "ln_x.weight"] * (ys / self.G_SCALE)),
                      w[a_ + "ln_x.bias"] / self.G_SCALE)
        # bonus ((r k r_k) summed over the head) v, / G_SCALE (r is / Y_SCALE, k / S_SCALE)
        rk = self.mulv(self.mulmul(self.ensure(r, 3), self.ensure(kmod, 3)),
                       w[a_ + "r_k"].ravel() * (ys / self.G_SCALE))
        y = self.add(y, self.mulmul(self.ensure(self.group_sum(rk, N, 1.0), 2), self.ensure(v, 2)))
        att = self.mv("o", self.mulmul(self.ensure(y, 3), self.ensure(g, 2)))
        x1 = self.add(x, att)
        # ---- channel mix
        f = p + "ffn."
        xf = self.ensure(self.layer_norm(p + "ln2", x1, w[p + "ln2.weight"], w[p + "ln2.bias"]), 4)
        xxf = self.sub(prev_ffn, xf)
        kf_in = self.ensure(self.add(xf, self.mulv(xxf, w[f + "x_k"])), 3)
        hs = [self.ensure(self.cheb(f + "relu2", cx.matvec(pl, [kf_in])), 2) for pl in self.ffn_k]
        lv = max(h.level for h in hs)   # the matvec's inputs share one level and scale
        for h in hs:
            if h.level < lv:
                cx.align(h, lv)
        x2 = self.add(x1, cx.matvec(self.ffn_v, hs))
        self.state = [x0, xf, S]
        return x2, v_first


class EncryptedRWKV7:
    """Every block of an RWKV-7 on the engine (EncryptedRWKV7Block each) for ``convs``
    conversations in the contiguous layout, the value of block 0 carried to the others.  The
    client applies block 0's input norm before encrypting (the reference folds ln0 into the
    embedding table) and the output norm and head after decrypting (``client_logits``), as the
    reference's server does not evaluate them."""

    def __init__(self, cx, sh: RWKV7Shape, w, fits, convs=1, b1=8):
        self.cx, self.sh, self.w, self.fits = cx, sh, w, fits
        self.blocks = [EncryptedRWKV7Block(cx, sh, w, i, fits, convs, b1) for i in range(sh.n_layer)]

    @staticmethod
    def keygen(cx, sh: RWKV7Shape, b1=8):
        """the rotation and matvec keys the blocks use"""
        cx.EvalRotateKeyGen(EncryptedRWKV7Block.rotations(sh, cx.slots))
        cx.matvec_keygen(sh.n_embd, b1)

    @property
    def bootstraps(self):
        return sum(b.bootstraps for b in self.blocks)

    def pack(self, x):
        return self.blocks[0].pack(x)

    def unpack(self, z):
        return self.blocks[0].unpack(z)

    def step(self, x_ct):
        v_first = None
        for b in self.blocks:
            x_ct, v_first = b.step(x_ct, v_first)
        return x_ct

    def client_input(self, tokens, sites=None):
        """the embedding rows through block 0's input norm, (convs, C)"""
        sites = sites or Sites(self.fits)
        w = self.w
        return _ln(sites, "blocks.0.ln0", w["emb.weight"][np.asarray(tokens)], w["blocks.0.ln0.weight"],
                   w["blocks.0.ln0.bias"])

    def client_logits(self, hidden, sites=None):
        sites = sites or Sites(self.fits)
        w = self.w
        return _ln(sites, "ln_out", hidden, w["ln_out.weight"], w["ln_out.bias"]) @ w["head.weight"].T
