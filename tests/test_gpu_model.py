"""Full MambaIntegerModel forward on the GPU against the reference's own
golden hashes (stage outputs and logits) and against the CPU oracle."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("name", sorted(cases.MODEL_CASES))
def test_model_logits_bit_exact_vs_reference(cuda_dev, name):
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    with open(os.path.join(GOLD, f"model_{name}.json")) as f:
        fx = json.load(f)
    cfg, sd, ids = cases.model_inputs(name)
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    m = m.to(cuda_dev).eval()
    with torch.no_grad():
        logits = m(ids.to(cuda_dev)).cpu().numpy()
    assert list(logits.shape) == fx["logits_shape"]
    if sha(logits) != fx["logits_sha256"]:
        from oracle import model as om
        ref = om.forward(om.prepare(sd), cfg, ids.numpy())
        ne = logits != ref
        raise AssertionError(f"{int(ne.sum())} of {ne.size} logits differ from the reference "
                             f"(max abs {np.abs(logits - ref).max()})")


def test_block_forward_matches_oracle(cuda_dev):
    from mamba_integer_b200.mamba_integer_model import MambaIntegerBlock
    from oracle import model as om
    cfg, sd, ids = cases.model_inputs("c4s")
    blk = MambaIntegerBlock(cfg, 0)
    blk.load_state_dict({k[len("layers.0."):]: v for k, v in sd.items() if k.startswith("layers.0.")})
    blk = blk.to(cuda_dev)
    x = sd["embedding.weight"][ids.reshape(-1)].reshape(ids.shape[0], ids.shape[1], -1)
    with torch.no_grad():
        y = blk(x.to(cuda_dev)).cpu().numpy()
    p = om.prepare(sd)
    ref = om.block_forward(p, "layers.0.", cfg, x.reshape(-1, x.shape[-1]).numpy(), ids.shape[0], ids.shape[1])
    assert (y.reshape(ref.shape) == ref).all()


def test_bitlinear_module_matches_reference_math(cuda_dev):
    from mamba_integer_b200.rational_bitnet import BitLinear
    from oracle import lib, model as om
    torch.manual_seed(0)
    lin = BitLinear(48, 1536)
    x = torch.randn(5, 7, 48)
    y = lin.to(cuda_dev)(x.to(cuda_dev)).cpu().numpy()
    wq, ws = om.weight_quant(lin.weight.detach().cpu().numpy())
    xq, xs = lib.quant_rows(x.reshape(-1, 48).numpy())
    ref = lib.bitlinear(xq, xs, wq, ws)
    assert (y.reshape(-1, 1536) == ref).all()
