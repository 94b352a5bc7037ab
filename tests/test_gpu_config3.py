"""Config 3 of the baseline at its own shape: full-slot bootstrapping of 32 ciphertexts in one
batch, with the precision reported in bits.

N = 2^16, 2^15 complex slots, sparse ternary secret of Hamming weight 192.  Chain: q0 60 bits,
14 x 45-bit user primes and the 14 x 58-bit primes the bootstrap consumes, K = 4 x 60-bit special
primes (logQP 1742).  Pipeline: ModRaise, CoeffToSlot in 3 merged FFT levels, EvalMod as the
degree-59 Chebyshev interpolant of the scaled cosine followed by 3 double-angle steps,
SlotToCoeff in 3 levels.  Slot values U[-1, 1] in both the real and imaginary parts, seeded.
Precision = -log2(max |decrypted - input|) over every slot of every ciphertext; the bound
asserted (1e-4, 13.3 bits) sits above the measured error with margin and well below the 5e-3 the
generic bootstrap tests allow."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_config3_batch_of_32_bootstraps():
    import fhessm
    cx = fhessm.CryptoContext(logN=16, L=29, K=4, alpha=4, hw=192, boot_primes=14)
    try:
        cx.KeyGen(seed=3)
        cx.EvalBootstrapSetup(24.0, 59, 3)
        rng = np.random.default_rng(33)
        zs = [rng.uniform(-1, 1, cx.slots) + 1j * rng.uniform(-1, 1, cx.slots) for _ in range(32)]
        cts = [cx.Encrypt(cx.MakeCKKSPackedPlaintext(z, level=cx.L - 3)) for z in zs]
        outs = cx.EvalBootstrapBatch(cts)
        errs = []
        for z, o in zip(zs, outs):
            assert o.level == cx.bootstrap_level()
            errs.append(float(np.abs(cx.Decrypt(o) - z).max()))
        worst, mean = max(errs), float(np.mean(errs))
        print(f"config 3: 32 bootstraps, precision {-np.log2(worst):.2f} bits (worst ciphertext), "
              f"{-np.log2(mean):.2f} bits (mean of the per-ciphertext maxima), level after {outs[0].level}")
        assert worst < 1e-4
    finally:
        cx.close()
