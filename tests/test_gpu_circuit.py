"""GPU tests of the circuit layer against float64 plaintext references.

Mirrors the CPU-twin verdicts of harness/cpu_real_model.cpp (poly_gate_deg3 < 1e-3,
lemma2_scan < 1e-3, bootstrap < 5e-3) and the server selftest of gpu_real_model.cu
:3965-4100 (encdec, rotate, matvec, rmsnorm, bootstrap): the decrypted result of each
encrypted operation is compared with numpy on the same inputs.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def ctx(logN=13, L=10, K=3, alpha=3, seed=3, boot_primes=0):
    import fhessm
    cx = fhessm.CryptoContext(logN=logN, L=L, K=K, alpha=alpha, hw=192, boot_primes=boot_primes)
    cx.KeyGen(seed=seed)
    return cx


@pytest.fixture(scope="module")
def cx():
    return ctx()


def test_mul_vec_rescale_and_align(cx):
    rng = np.random.default_rng(0)
    z = rng.uniform(-1, 1, cx.slots) + 1j * rng.uniform(-1, 1, cx.slots)
    v = rng.uniform(-1, 1, cx.slots)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(z))
    r = cx.mul_vec_rescale(ct, v)
    assert r.level == 1
    assert abs(r.scale / cx.GetScalingFactorReal(1) - 1) < 1e-12
    assert np.abs(cx.Decrypt(r) - z * v).max() < 1e-6
    cx.align(ct, 4)
    assert ct.level == 4 and abs(ct.scale / cx.GetScalingFactorReal(4) - 1) < 1e-9
    assert np.abs(cx.Decrypt(ct) - z).max() < 1e-6
    # periodic vector (n divides the slot count): repeated across the slots
    p = rng.uniform(-1, 1, 64)
    r2 = cx.mul_vec_rescale(ct, p)
    assert np.abs(cx.Decrypt(r2) - z * np.tile(p, cx.slots // 64)).max() < 1e-6


def test_poly_gate_deg3_vector_coefficients(cx):
    """g = z (p0 + p1 z + p2 z^2) with per-channel coefficients (cpu_real_model.cpp:556-578)."""
    rng = np.random.default_rng(1)
    d = 64
    z = rng.uniform(-1, 1, d)
    p0, p1, p2 = 0.5 + 0.01 * np.arange(d) / d, np.full(d, 0.25), np.full(d, 0.1)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(np.tile(z, cx.slots // d)))
    g = cx.EvalPolyVec(ct, [np.zeros(d), p0, p1, p2])
    ref = z * (p0 + p1 * z + p2 * z * z)
    got = cx.Decrypt(g).real[:d]
    assert np.abs(got - ref).max() < 1e-3
    assert np.abs(got - ref).max() < 1e-6     # much tighter than the reference's 1e-3 verdict


def test_chebyshev_series(cx):
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, cx.slots)
    c = rng.uniform(-1, 1, 16) / np.arange(1, 17)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(x))
    y = cx.EvalChebyshevSeries(ct, c)
    ref = np.polynomial.chebyshev.chebval(x, c)
    assert np.abs(cx.Decrypt(y).real - ref).max() < 1e-6


@pytest.mark.parametrize("ncoef", [12, 16, 24, 32])
def test_chebyshev_series_batched_matches_single(cx, ncoef):
    """The batched evaluator (two ciphertexts, products batched, as in the bootstrap's EvalMod)
    gives the single evaluator's words, for leaf-times-giant and product-times-giant trees."""
    rng = np.random.default_rng(40 + ncoef)
    c = rng.uniform(-1, 1, ncoef) / np.arange(1, ncoef + 1)
    xs = [rng.uniform(-1, 1, cx.slots) for _ in range(2)]
    cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(x)) for x in xs]
    got = cx.EvalChebyshevSeriesBatch(cts, c)
    for k in range(2):
        single = cx.EvalChebyshevSeries(cts[k], c)
        assert (got[k].words() == single.words()).all()
        ref = np.polynomial.chebyshev.chebval(xs[k], c)
        assert np.abs(cx.Decrypt(got[k]).real - ref).max() < 1e-6


@pytest.mark.parametrize("ncoef", [8, 16, 24, 32])
def test_chebyshev_series_consumes_the_planned_depth(cx, ncoef):
    """The evaluator uses exactly the levels fhe_cheb_depth plans (the bootstrap relies on it)."""
    import fhessm
    rng = np.random.default_rng(60 + ncoef)
    c = rng.uniform(0.5, 1.0, ncoef)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(rng.uniform(-1, 1, cx.slots)))
    y = cx.EvalChebyshevSeries(ct, c)
    assert y.level - ct.level == fhessm.cheb_depth(c)


def test_lemma2_scan(cx):
    """s_t = a (.) s_{t-1} + b (.) x_t over 8 steps (cpu_real_model.cpp:580-603)."""
    rng = np.random.default_rng(3)
    d = 64
    a = 0.90 + 0.09 * (np.arange(d) % 7) / 7.0
    b = 1.0 - a
    xs = [np.sin(0.3 * t + 0.11 * np.arange(d)) * 0.4 for t in range(3)]
    s = cx.Encrypt(cx.MakeCKKSPackedPlaintext(np.zeros(cx.slots)))
    ref = np.zeros(d)
    for t in range(3):
        x = cx.Encrypt(cx.MakeCKKSPackedPlaintext(np.tile(xs[t], cx.slots // d)))
        cx.align(x, s.level)
        s1 = cx.mul_vec_rescale(s, a)
        bx = cx.mul_vec_rescale(x, b)
        s = cx.EvalAdd(s1, bx)
        ref = a * ref + b * xs[t]
    assert np.abs(cx.Decrypt(s).real[:d] - ref).max() < 1e-3


def block_pack(lanes, D, slots):
    """lanes: (2R, D) real -> slot vector (R blocks of D, lane r real part, lane r+R imaginary)."""
    R = slots // D
    z = np.zeros(slots, dtype=np.complex128)
    for r in range(lanes.shape[0]):
        blk = r % R
        z[blk * D: blk * D + lanes.shape[1]] += lanes[r] * (1 if r < R else 1j)
    return z


def block_unpack(z, D, nlanes, width):
    R = len(z) // D
    out = np.zeros((nlanes, width))
    for r in range(nlanes):
        blk = r % R
        seg = z[blk * D: blk * D + width]
        out[r] = seg.real if r < R else seg.imag
    return out


@pytest.mark.parametrize("rows,cols", [(64, 64), (48, 100)])
def test_matvec_bsgs_lanes(cx, rows, cols):
    """Per-lane y = W u with every lane different (matvec_square, matvec_rect and the
    batched no-bleed check of cpu_real_model.cpp:270-463), complex-packed lanes."""
    D, b1 = 64, 8
    cx.matvec_keygen(D, b1)
    rng = np.random.default_rng(7 + rows)
    W = rng.normal(0, 0.3, (rows, cols))
    R = cx.slots // D
    nlanes = 2 * R
    U = rng.uniform(-1, 1, (nlanes, cols))
    nsets = (cols + D - 1) // D
    ins = []
    for s in range(nsets):
        part = U[:, s * D:(s + 1) * D]
        ins.append(cx.Encrypt(cx.MakeCKKSPackedPlaintext(block_pack(part, D, cx.slots), level=1)))
    plan = cx.matvec_plan(W, D, b1)
    y = cx.matvec(plan, ins)
    assert y.level == 2
    got = block_unpack(cx.Decrypt(y), D, nlanes, rows)
    ref = U @ W.T
    assert np.abs(got - ref).max() < 1e-3
    assert np.abs(got - ref).max() < 1e-6
    assert np.abs(ref[0] - ref[1]).max() > 1e-2        # lanes genuinely differ (no-bleed is meaningful)


@pytest.mark.parametrize("b1", [2, 4, 8, 16])
def test_matvec_tensor_core_products_bit_identical(cx, b1):
    """The tcgen05 byte-split product kernel and the CUDA-core kernel give the same words
    (D = 128: G = D / b1 = 64, 32, 16, 8 giant steps, the outputs of one product; G = 64 is the
    largest plan matvec_plan accepts)."""
    D = 128
    cx.matvec_keygen(D, b1)
    rng = np.random.default_rng(11 + b1)
    W = rng.normal(0, 0.3, (D, 2 * D))
    R = cx.slots // D
    U = rng.uniform(-1, 1, (2 * R, 2 * D))
    ins = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(block_pack(U[:, s * D:(s + 1) * D], D, cx.slots), level=1))
           for s in range(2)]
    plan = cx.matvec_plan(W, D, b1)
    out = {}
    for tc in (0, 1):
        cx.set_option("matvec_tensor_cores", tc)
        out[tc] = cx.matvec(plan, ins).words()
    cx.set_option("matvec_tensor_cores", 1)
    assert (out[0] == out[1]).all()
    got = block_unpack(cx.Decrypt(cx.matvec(plan, ins)), D, 2 * R, D)
    assert np.abs(got - U @ W.T).max() < 1e-5


def test_plaintext_cache_bit_identical(cx):
    """The plan's plaintext cache (the reference's --cache-diags): a repeated call at the same
    level and scale reuses the cached words, a call at another level regenerates them, and
    every result equals the uncached one word for word."""
    D, b1 = 128, 8
    cx.matvec_keygen(D, b1)
    rng = np.random.default_rng(31)
    W = rng.normal(0, 0.3, (D, D))
    R = cx.slots // D
    U = rng.uniform(-1, 1, (2 * R, D))
    plan = cx.matvec_plan(W, D, b1)
    res = {}
    for lvl in (1, 2):
        ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(block_pack(U, D, cx.slots), level=lvl))
        cx.set_option("plaintext_cache", 1)
        first = cx.matvec(plan, [ct]).words()
        again = cx.matvec(plan, [ct]).words()      # served from the cache
        cx.set_option("plaintext_cache", 0)
        fresh = cx.matvec(plan, [ct]).words()
        cx.set_option("plaintext_cache", 1)
        assert (first == again).all() and (first == fresh).all()
        res[lvl] = first
    assert res[1].shape != res[2].shape


def test_matvec_1024_block():
    """A 1024-wide block (the model's D) at N = 2^14: the 2048-point plaintext generation and
    the double-hoisted BSGS with b1 = 64 against numpy, every lane different."""
    import fhessm
    c = fhessm.CryptoContext(logN=14, L=8, K=4, alpha=4, hw=192)
    c.KeyGen(seed=21)
    D, b1 = 1024, 64
    c.matvec_keygen(D, b1)
    rng = np.random.default_rng(5)
    W = rng.normal(0, 0.02, (D, D))
    R = c.slots // D
    U = rng.uniform(-1, 1, (2 * R, D))
    ct = c.Encrypt(c.MakeCKKSPackedPlaintext(block_pack(U, D, c.slots), level=1))
    y = c.matvec(c.matvec_plan(W, D, b1), [ct])
    got = block_unpack(c.Decrypt(y), D, 2 * R, D)
    assert np.abs(got - U @ W.T).max() < 1e-5


@pytest.mark.parametrize("logN,L", [(13, 22)])
def test_bootstrap_small_ring(logN, L):
    boot_check(logN, L, tol=5e-3)


def boot_check(logN, L, tol):
    # q0 60 bits, 45-bit user primes, the top 14 limbs (CoeffToSlot 3 + scaling 1 + EvalMod 10)
    # 58-bit primes so that the bootstrap circuit keeps ~58 bits of plaintext precision
    cx = ctx(logN=logN, L=L, K=4, alpha=4, seed=11, boot_primes=14)
    cx.EvalBootstrapSetup(24.0, 59)
    rng = np.random.default_rng(4)
    z = rng.uniform(-1, 1, cx.slots) + 1j * rng.uniform(-1, 1, cx.slots)
    ct = cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, level=L - 3))
    out = cx.EvalBootstrap(ct)
    assert out.level == cx.bootstrap_level()
    err = np.abs(cx.Decrypt(out) - z).max()
    bits = -np.log2(err)
    print(f"bootstrap N=2^{logN} L={L}: max err {err:.3e} ({bits:.1f} bits), level after {out.level}")
    assert err < tol
    # a second bootstrap of the refreshed ciphertext (state carried across steps)
    cx.align(out, L - 2)
    out2 = cx.EvalBootstrap(out)
    assert np.abs(cx.Decrypt(out2) - z).max() < 2 * tol
    return bits


def test_bootstrap_production_ring():
    """Config 3 shape: N = 2^16, 2^15 complex slots, HW-192 secret, L = 29 + K = 4
    (logQP = 60 + 14 x 45 + 14 x 58 + 4 x 60 = 1742 <= 1747)."""
    boot_check(16, 29, tol=5e-3)
