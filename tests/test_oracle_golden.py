"""The CPU oracle against golden fixtures produced by the reference itself
(tests/golden/make_golden.py): every stage and the logits must be bit-identical."""
import hashlib
import json
import os

import numpy as np
import pytest

import cases
from oracle import lib, model as om

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def stages():
    return np.load(os.path.join(GOLD, "stages.npz"))


def test_quant_matches_reference(stages):
    q, s = lib.quant_rows(cases.quant_inputs())
    np.testing.assert_array_equal(q, stages["quant.xq"])
    np.testing.assert_array_equal(s, stages["quant.scale"])


def test_elementwise_match_reference(stages):
    e = cases.edge_values()
    np.testing.assert_array_equal(lib.squareplus_clamp(e, -50.0, 50.0), stages["sqp.y"])
    np.testing.assert_array_equal(lib.ste_clamp(e, -20.0, 20.0), stages["ste20.y"])
    np.testing.assert_array_equal(lib.ste_clamp(e, 0.0, 32000.0), stages["ste_dec.y"])
    y, z = cases.gate_inputs()
    np.testing.assert_array_equal(lib.sigmoid_gate(y, z), stages["gate.y"])


def test_dt_value_matches_reference(stages):
    e = cases.edge_values()
    mod = lib.ste_clamp(e, -20.0, 20.0)
    sp = lib.squareplus_clamp(mod, -3.0e38, 3.0e38)  # clamp bounds that never bind: plain squareplus
    dtv = lib.ste_clamp((sp * np.float32(0.01)).astype(np.float32), 0.001, 0.1)
    np.testing.assert_array_equal(dtv, stages["dtv.y"])


def test_norm_matches_reference(stages):
    x, g, st = cases.norm_inputs()
    y, inv = lib.bitshift_norm(x, g, st[0])
    np.testing.assert_array_equal(inv, stages["norm.inv_rms"])
    np.testing.assert_array_equal(y, stages["norm.y"])
    assert len(np.unique(inv)) >= 8  # the inputs reach many threshold bands


def test_scan_matches_reference(stages):
    u, nums = cases.scan_inputs()
    np.testing.assert_array_equal(lib.scan_convex(u, nums), stages["scan.h"])


def test_weight_quant_matches_reference(stages):
    q, s = om.weight_quant(cases.weight_input())
    np.testing.assert_array_equal(q, stages["wq.q"])
    assert np.float32(s) == stages["wq.scale"][0]


@pytest.mark.parametrize("name", sorted(cases.MODEL_CASES))
def test_model_forward_matches_reference(name):
    with open(os.path.join(GOLD, f"model_{name}.json")) as f:
        fx = json.load(f)
    cfg, sd, ids = cases.model_inputs(name)
    cap = {}
    logits = om.forward(om.prepare(sd), cfg, ids.numpy(), cap=cap)
    L = ids.shape[1]
    for key, h in fx["stages_sha256"].items():
        okey = key if key.endswith(".out") else key + ".out"
        a = cap[okey]
        assert sha(a.reshape(-1, a.shape[-1])) == h, f"stage {key} differs from the reference"
    assert list(logits.shape) == fx["logits_shape"]
    assert sha(logits) == fx["logits_sha256"]
    del L


def test_backward_restatements_match_reference_golden():
    # tests/golden/backward.npz: the reference's own DyadicScanFunction.backward
    # (src/mamba_integer_model.py:319-344) and QuantizeActivationsFunction.backward
    # (src/triton_kernels/bitnet_kernels.py:77-95), run by make_backward_golden.py
    import os

    import numpy as np

    from oracle import lib

    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "backward.npz"))
    for c in ("scan_a", "scan_b"):
        assert np.array_equal(lib.scan_convex(z[c + ".u"], z[c + ".nums"]).view(np.uint32), z[c + ".h"].view(np.uint32))
        gu, gn = lib.scan_convex_backward(z[c + ".grad_h"], z[c + ".h"], z[c + ".u"], z[c + ".nums"])
        assert np.array_equal(gu.view(np.uint32), z[c + ".grad_u"].view(np.uint32)), c
        assert np.array_equal(gn.view(np.uint32), z[c + ".grad_nums"].view(np.uint32)), c
    for c in ("ste_a", "ste_b"):
        gx = lib.quant_ste_backward(z[c + ".grad_xq"], z[c + ".amax"])
        assert np.array_equal(gx.view(np.uint32), z[c + ".grad_x"].view(np.uint32)), c
