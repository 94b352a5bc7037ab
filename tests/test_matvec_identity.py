"""The slot-level identity behind the BSGS matvec plan (matvec.cu), checked on plain vectors with
numpy (no encryption, no GPU).  A ciphertext holds R blocks of D slots; y = W u applies the same
D x D matrix to every block.  With k = g b1 + j the block-cyclic rotation is split by masks into
the families AA, AB, BA of D-periodic vectors, and, because a D-periodic vector is unchanged by a
rotation of D slots, the BA terms ride the giant rotation of AA and AB on the baby rot(u, j - D):
    y = sum_g rot(I_g, g b1),  I_g = sum_j AA_gj . rot(u, j) + (AB_gj + BA_gj) . rot(u, j - D)."""
import numpy as np
import pytest


def rot(v, k):
    """Slot rotation to the left by k (the encrypted EvalRotate(ct, k))."""
    return np.roll(v, -k)


def families(W, D, b1):
    """Per (g, j): the merged family vectors of one period, by the masks of matvec_plan."""
    G = D // b1
    A0 = np.zeros((G, b1, D))
    A1 = np.zeros((G, b1, D))
    for g in range(G):
        for j in range(b1):
            k = g * b1 + j
            for p in range(D):
                ga = p >= g * b1            # giant A keeps inner slots p >= g b1
                mj = p + j < D              # baby rot(u, j) is valid where p + j < D
                c = (p - g * b1) % D        # output channel of this inner slot
                w = W[c, (c + k) % D]
                if ga and mj:
                    A0[g, j, p] = w          # AA
                elif ga != mj:
                    A1[g, j, p] = w          # AB (ga, not mj) and BA (not ga, mj) merged
    return A0, A1


@pytest.mark.parametrize("D,b1,R", [(16, 4, 4), (16, 16, 2), (32, 8, 3), (8, 1, 5)])
def test_merged_giant_family_equals_block_matvec(D, b1, R):
    rng = np.random.default_rng(D * 100 + b1)
    W = rng.normal(size=(D, D))
    U = rng.normal(size=(R, D))
    u = U.ravel()
    G = D // b1
    A0, A1 = families(W, D, b1)
    y = np.zeros(R * D)
    for g in range(G):
        I = np.zeros(R * D)
        for j in range(b1):
            I += np.tile(A0[g, j], R) * rot(u, j) + np.tile(A1[g, j], R) * rot(u, j - D)
        y += rot(I, g * b1)
    assert np.allclose(y.reshape(R, D), U @ W.T)


def test_two_giant_families_agree_with_the_merged_one():
    """The unmerged form sum_g rot(IA_g, g b1) + rot(IB_g, g b1 - D) gives the same vector."""
    D, b1, R = 16, 4, 3
    rng = np.random.default_rng(7)
    W = rng.normal(size=(D, D))
    u = rng.normal(size=R * D)
    G = D // b1
    y2 = np.zeros(R * D)
    for g in range(G):
        IA = np.zeros(R * D)
        IB = np.zeros(R * D)
        for j in range(b1):
            k = g * b1 + j
            aa, ab, ba = np.zeros(D), np.zeros(D), np.zeros(D)
            for p in range(D):
                ga, mj = p >= g * b1, p + j < D
                c = (p - g * b1) % D
                w = W[c, (c + k) % D]
                if ga and mj:
                    aa[p] = w
                elif ga:
                    ab[p] = w
                elif mj:
                    ba[p] = w
            IA += np.tile(aa, R) * rot(u, j) + np.tile(ab, R) * rot(u, j - D)
            IB += np.tile(ba, R) * rot(u, j)
        y2 += rot(IA, g * b1) + rot(IB, g * b1 - D)
    assert np.allclose(y2.reshape(R, D), u.reshape(R, D) @ W.T)
