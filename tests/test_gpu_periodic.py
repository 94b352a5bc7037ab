"""Periodic (compressed) encode == dense encode, word for word.

The reference's own check of its store-entry encoder (hpc_gpu_port/periodic_encode_test.cpp:
1-14, identity stated in periodic_encode.hpp:1-40): the ring-N encoding of a vector made of
N/(2 period) copies of one period is the ring-(2 period) encoding of that period, so word j2 of
the compressed entry equals word j2 << log2(N / (2 period)) of the dense plaintext.  Here the
compressed words come from the device generator the matvec plans use (k_ptgen2048 at period
1024, k_ptgen below) through fhe_encode_periodic, and the dense words from fhe_encode, at the
405M model's chain (45-, 58- and 60-bit limbs)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cx():
    import fhessm
    return fhessm.CryptoContext(logN=16, L=28, K=4, alpha=4, hw=192, boot_primes=14)


@pytest.mark.parametrize("period", [1024, 256, 64])
@pytest.mark.parametrize("level", [0, 9, 20])
def test_periodic_equals_dense(cx, period, level):
    rng = np.random.default_rng(period + level)
    vecs = [rng.normal(0, 0.02, period),                                             # a weight diagonal
            rng.uniform(-1, 1, period) + 1j * rng.uniform(-1, 1, period),            # complex-packed lanes
            np.where(rng.uniform(0, 1, period) < 0.5, 0.0, rng.normal(0, 1, period))]  # masked (block-cyclic)
    comp = cx.periodic_encode_comp(np.stack(vecs), level=level)
    rep = cx.slots // period
    assert comp.shape == (3, cx.L - level, 2 * period)
    for t, v in enumerate(vecs):
        dense = cx.pt_words(cx.MakeCKKSPackedPlaintext(np.tile(v, rep), level=level))
        assert dense.shape == (cx.L - level, cx.N)
        bad = np.argwhere(dense[:, ::rep] != comp[t])
        assert bad.size == 0, f"vector {t}: {len(bad)} words differ, first (limb, word) {tuple(bad[0])}"
        assert comp[t].any()
