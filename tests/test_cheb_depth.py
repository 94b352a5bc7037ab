"""The level plan of the Chebyshev evaluator (fhe_cheb_depth, host code: no GPU).  The
bootstrap places SlotToCoeff at the level its EvalMod polynomial leaves, so the plan must follow
the evaluator's baby-step / giant-step tree exactly.  Expected depths, baby step bs with
bs^2 >= degree + 1: babies T_2..T_{bs-1} are aligned to the deepest baby (depth log2(bs)), a
leaf is one level below them, and each giant product adds one level."""
import os

import numpy as np
import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "fhe-ssm_b200", "fhessm", "libfhessm.so")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="libfhessm.so not built")


@pytest.mark.parametrize("degree,depth", [
    (3, 2),     # bs 2: leaves at depth 1 (c0 + c1 T1), one product with the giant T2 (depth 1)
    (7, 4),     # bs 4: babies to depth 2, leaves 3, one giant product (T4, depth 2) -> 4
    (15, 5),    # bs 4: giants T4, T8; two product levels over the leaves
    (23, 5),    # bs 8: the top quotient is a leaf, so T16 x leaf is the last product
    (31, 6),    # bs 8: the top quotient is itself a product (T8 x leaf)
    (59, 7),    # bs 8: giants T8, T16, T32
])
def test_depth_of_dense_series(degree, depth):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "fhe-ssm_b200"))
    import fhessm
    c = np.random.default_rng(degree).uniform(0.5, 1.0, degree + 1)
    assert fhessm.cheb_depth(c) == depth


def test_trailing_zeros_lower_the_depth():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "fhe-ssm_b200"))
    import fhessm
    c = np.zeros(32)
    c[:8] = 1.0                        # degree 31 nominally, degree 7 in fact: babies of bs 8 and one leaf
    assert fhessm.cheb_depth(c) == 4
