#!/usr/bin/env python3
"""Writes tests/golden/rwkv7_small.npz: logits and block outputs of the reference's RWKV-7 harness.

Imports RWKV7 from the reference's results/vector-d-20261104/harness/rwkv7_model.py (the x070
forward the reference evaluates its polynomial sites against), loads the seeded synthetic weights
of fhessm.rwkv7 under its state-dict names, and runs a token sequence through it in exact mode.
tests/test_rwkv7_reference.py holds fhessm.rwkv7.step, one token at a time, to these numbers.

    python tests/golden/make_rwkv7_golden.py <reference root>
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "fhe-ssm_b200"))

SHAPE = dict(n_layer=2, n_embd=128, head_size=64, d_decay=16, d_aaa=16, d_mv=8, d_gate=32, dim_ffn=256,
             vocab_size=512)
WEIGHT_SEED, TOKEN_SEED, B, T = 3, 5, 2, 10


def small_model():
    from fhessm.rwkv7 import RWKV7Shape, synthetic_weights
    sh = RWKV7Shape(**SHAPE)
    w = synthetic_weights(sh, seed=WEIGHT_SEED)
    ids = np.random.default_rng(TOKEN_SEED).integers(0, sh.vocab_size, (B, T))
    return sh, w, ids


def reference_logits(ref_root):
    """(logits (B, T, V), last block's output (B, T, C)) of the reference harness, float32 inside."""
    import torch
    sys.path.insert(0, os.path.join(ref_root, "results", "vector-d-20261104", "harness"))
    from rwkv7_model import RWKV7, RWKV7Config
    sh, w, ids = small_model()
    cfg = RWKV7Config(**SHAPE)
    model = RWKV7(cfg)
    own = model.state_dict()
    sd = {}
    for k, v in own.items():
        if k not in w:
            # block 0 has value-residual parameters it never uses (rwkv7_model.py:315, demo.py:383)
            if not k.startswith("blocks.0.att.v"):
                raise KeyError(f"no synthetic weight for {k}")
            sd[k] = torch.zeros(tuple(v.shape))
            continue
        sd[k] = torch.tensor(np.asarray(w[k]).reshape(tuple(v.shape)), dtype=torch.float32)
    model.load_state_dict(sd, strict=True)
    model.eval()
    with torch.no_grad():
        logits, hidden = model(torch.tensor(ids), return_hidden=True)
    return logits.double().numpy(), hidden[-1].double().numpy()


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FHESSM_REFERENCE", "/root/reference")
    lg, hid = reference_logits(ref)
    _, _, ids = small_model()
    np.savez_compressed(os.path.join(HERE, "rwkv7_small.npz"), ids=ids, logits=lg, hidden=hid)
    print("wrote rwkv7_small.npz", lg.shape, hid.shape)
