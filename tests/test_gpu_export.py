"""A model loaded from the reference's int8 export (written by the reference
exporter, tests/golden/make_export_fixture.py) runs on the sm_100a kernels and
reproduces the reference model's logits bit for bit."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_loaded_export_gives_reference_logits(cuda_dev):
    from mamba_integer_b200.export_format import load_export
    with open(os.path.join(GOLD, "export_tiny.json")) as f:
        fx = json.load(f)
    m = load_export(os.path.join(GOLD, "export_tiny.bin"), cuda_dev).eval()
    with torch.no_grad():
        logits = m(torch.tensor(fx["ids"], dtype=torch.int64, device=cuda_dev)).cpu().numpy()
    assert list(logits.shape) == fx["logits_shape"]
    assert hashlib.sha256(np.ascontiguousarray(logits).tobytes()).hexdigest() == fx["logits_sha256"]
