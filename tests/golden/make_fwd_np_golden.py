#!/usr/bin/env python3
"""Writes tests/golden/fwd_np_small.npz: logits of the reference's float64 model forward.

Imports _fwd_np from the reference's ml-eval/train_fhe_native_ssm.py (:829-890, the float64
reference the reference checks its FHE circuit against), sets its CFG to a small shape, feeds it
the seeded synthetic weights of fhessm.model renamed to the reference's parameter names (decays
through its a_raw parametrisation, :841, and non-unit norm gains), and records the logits of a
token sequence.  tests/test_model_reference.py holds fhessm.model.plain_step to these numbers.

    python tests/golden/make_fwd_np_golden.py <reference root>
"""
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "fhe-ssm_b200"))

SHAPE = dict(d=64, dff=128, n_layer=2, vocab=97, D=64)
WEIGHT_SEED, GAIN_SEED, TOKEN_SEED, T = 77, 78, 79, 12


def small_weights():
    """The synthetic weights of the test shape with seeded norm gains in [0.5, 1.5]."""
    from fhessm.model import ModelConfig, synthetic_weights
    cfg = ModelConfig(**SHAPE)
    w = synthetic_weights(cfg, seed=WEIGHT_SEED)
    rng = np.random.default_rng(GAIN_SEED)
    for L in w["layers"]:
        L["g1"] = rng.uniform(0.5, 1.5, cfg.d)
        L["g2"] = rng.uniform(0.5, 1.5, cfg.d)
    w["g_out"] = rng.uniform(0.5, 1.5, cfg.d)
    ids = np.random.default_rng(TOKEN_SEED).integers(0, cfg.vocab, T)
    return cfg, w, ids


def reference_names(cfg, w):
    """fhessm.model weights under the reference's parameter names (train_fhe_native_ssm.py:836-888)."""
    lo, hi = cfg.a_min, cfg.a_max
    r = {"emb.weight": w["emb"], "g_out": w["g_out"]}
    for i, L in enumerate(w["layers"]):
        p = f"blocks.{i}."
        f = (L["decay"] - lo) / (hi - lo)
        r[p + "tm.a_raw"] = np.log(f / (1.0 - f))          # a = lo + (hi - lo) sigmoid(a_raw)
        r[p + "tm.g1"], r[p + "tm.mix"] = L["g1"], L["mix"]
        r[p + "tm.win.weight"], r[p + "tm.wout.weight"] = L["win"], L["wout"]
        r[p + "tm.c"], r[p + "tm.dd"] = L["c"], L["dd"]
        for k in range(3):
            r[p + f"tm.p{k}"] = L[f"p{k}"]
        r[p + "cm.g2"] = L["g2"]
        r[p + "cm.wk.weight"], r[p + "cm.wr.weight"], r[p + "cm.wv.weight"] = L["wk"], L["wr"], L["wv"]
        for k in range(4):
            r[p + f"cm.q{k}"] = L[f"q{k}"]
        for k in range(3):
            r[p + f"cm.r{k}"] = L[f"r{k}"]
    return r


def reference_logits(ref_root):
    spec = importlib.util.spec_from_file_location("ref_train_fhe_native_ssm",
                                                  os.path.join(ref_root, "ml-eval", "train_fhe_native_ssm.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    cfg, w, ids = small_weights()
    mod.CFG.update({"d_model": cfg.d, "n_layer": cfg.n_layer, "d_ffn": cfg.dff, "vocab": cfg.vocab,
                    "shift_mix": cfg.shift_mix, "a_min": cfg.a_min, "a_max": cfg.a_max, "alpha_res": cfg.alpha,
                    "nonlin": "poly", "block": "sequential"})
    return ids, mod._fwd_np(reference_names(cfg, w), ids)


if __name__ == "__main__":
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FHESSM_REFERENCE", "")
    ids, logits = reference_logits(ref_root)
    np.savez(os.path.join(HERE, "fwd_np_small.npz"), ids=ids, logits=logits)
    print("wrote", os.path.join(HERE, "fwd_np_small.npz"), logits.shape)
