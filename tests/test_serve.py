"""The serve loop's file protocol (req.<N>.* in, resp.<N>.* out, reset, errors, stop,
serve.status) on CPU: the native loop runs with a Python step function, no GPU involved."""
import json
import os
import threading

import numpy as np
import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "fhe-ssm_b200", "fhessm", "libfhessm.so")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="libfhessm.so not built")


def test_serve_protocol(tmp_path):
    from fhessm import FheError
    from fhessm import serve as sv
    d = str(tmp_path)
    seen = []

    def step(reset, cts):
        seen.append(reset)
        level, scale, w = cts[0]
        if scale < 0:
            raise RuntimeError("refused")
        out = (w[:, :-1, :] ^ np.uint64(0x5A5A)).copy()         # one limb fewer, words changed
        return [(level + 1, scale * 2, out)]

    served = {}
    th = threading.Thread(target=lambda: served.setdefault("n", sv.serve_files(d, step, timeout_ms=20000)))
    th.start()
    rng = np.random.default_rng(0)
    w0 = rng.integers(0, 2**60, (2, 3, 1024), dtype=np.uint64)
    sv.submit(d, 0, [(2, 1.5, w0)], reset=True, lanes=64, tokensReal=1)
    (resp, meta) = sv.wait_response(d, 0, timeout=20)
    level, scale, w = resp[0]
    assert (level, scale) == (3, 3.0) and (w == (w0[:, :-1, :] ^ np.uint64(0x5A5A))).all()
    assert meta["lanes"] == 64 and meta["tokensReal"] == 1 and meta["reset"] is True
    assert not os.path.exists(os.path.join(d, "req.0.ready"))           # request files consumed
    # next step of the same session, then a malformed request, then a step that fails
    sv.submit(d, 1, [(2, 1.5, w0)], lanes=64)
    sv.wait_response(d, 1, timeout=20)
    with open(os.path.join(d, "req.2.meta"), "w") as f:
        f.write("{}")
    open(os.path.join(d, "req.2.ready"), "w").close()
    with pytest.raises(FheError, match="meta"):
        sv.wait_response(d, 2, timeout=20)
    sv.submit(d, 3, [(2, -1.0, w0)])
    with pytest.raises(FheError, match="step failed"):
        sv.wait_response(d, 3, timeout=20)
    st = json.load(open(os.path.join(d, "serve.status")))
    assert st["stateful"] is True and st["served"] == 2
    open(os.path.join(d, "stop"), "w").close()
    th.join(30)
    assert not th.is_alive() and served["n"] == 2
    assert seen == [True, False, False]


def test_serve_refuses_oversized_outputs_and_foreign_meta(tmp_path):
    """An output must fit its input's buffer (same ring, no more limbs, no more outputs than
    inputs); the reference's meta fields are checked (ringDim, level, interleave, packTokens)
    and echoed in its order."""
    from fhessm import FheError
    from fhessm import serve as sv
    d = str(tmp_path)
    mode = {}

    def step(reset, cts):
        level, scale, w = cts[0]
        if mode.get("grow"):
            return [(level, scale, np.concatenate([w, w[:, :1]], axis=1))]   # one limb more than the input
        if mode.get("two"):
            return [(level, scale, w), (level, scale, w)]                     # two outputs for one input
        return [(level, scale, w)]

    th = threading.Thread(target=lambda: sv.serve_files(d, step, timeout_ms=20000))
    th.start()
    w0 = np.random.default_rng(1).integers(0, 2**60, (2, 2, 1024), dtype=np.uint64)
    mode["grow"] = True
    sv.submit(d, 0, [(3, 1.0, w0)])
    with pytest.raises(FheError, match="step failed"):
        sv.wait_response(d, 0, timeout=20)
    mode.clear()
    mode["two"] = True
    sv.submit(d, 1, [(3, 1.0, w0)])
    with pytest.raises(FheError, match="step failed"):
        sv.wait_response(d, 1, timeout=20)
    mode.clear()
    sv.submit(d, 2, [(3, 1.0, w0)], ringDim=2048)
    with pytest.raises(FheError, match="ringDim"):
        sv.wait_response(d, 2, timeout=20)
    sv.submit(d, 3, [(3, 1.0, w0)], interleave=1)
    with pytest.raises(FheError, match="interleaved"):
        sv.wait_response(d, 3, timeout=20)
    sv.submit(d, 4, [(3, 1.0, w0)], packTokens=1, tokensReal=1, dpad=1024, interleave=0, lanes=64,
              ringDim=1024, level=3)
    (resp, meta) = sv.wait_response(d, 4, timeout=20)
    assert (resp[0][2] == w0).all()
    assert list(meta)[:8] == ["count", "packTokens", "tokensReal", "dpad", "interleave", "lanes", "ringDim", "level"]
    assert (meta["dpad"], meta["lanes"], meta["ringDim"], meta["level"]) == (1024, 64, 1024, 3)
    open(os.path.join(d, "stop"), "w").close()
    th.join(30)
    assert not th.is_alive()
