"""Seeded inputs shared by make_golden.py (which runs the reference on them) and
the parity tests (which run the oracle / the GPU kernels on them)."""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from mamba_integer_b200 import synth  # noqa: E402

# name -> (base config, batch, seq_len, n_layer override)
MODEL_CASES = {
    "c1": {"base": "c1", "batch": 2, "seq_len": 256, "n_layer": None},
    "c4s": {"base": "c4", "batch": 2, "seq_len": 128, "n_layer": 2},
    "c5s": {"base": "c5", "batch": 2, "seq_len": 64, "n_layer": 1},
}


def model_inputs(name: str):
    spec = MODEL_CASES[name]
    over = {} if spec["n_layer"] is None else {"n_layer": spec["n_layer"]}
    cfg = synth.model_config(spec["base"], **over)
    sd = synth.model_state_dict(cfg, synth.CONFIGS[spec["base"]]["seed"])
    ids = synth.input_ids(spec["base"], spec["batch"], spec["seq_len"])
    return cfg, sd, ids


def hook_key(mod_name: str):
    """Reference module name -> stage key (None for modules not hooked)."""
    if mod_name in ("embedding", "norm_f", "lm_head"):
        return mod_name + ".out"
    parts = mod_name.split(".")
    if len(parts) == 2 and parts[0] == "layers":
        return mod_name + ".block.out"
    if len(parts) == 3 and parts[0] == "layers":
        leaf = parts[2]
        if leaf in ("norm", "in_proj", "x_proj", "dt_proj", "out_proj"):
            return mod_name + ".out"
        if leaf == "conv1d":
            return f"layers.{parts[1]}.conv"
    return None


def edge_values() -> np.ndarray:
    """Values that exercise clamps, the squareplus guess table and rounding."""
    special = [0.0, -0.0, 1e-30, -1e-30, 1e-7, 0.001, 0.0999, 0.1, 0.25, 0.5, 0.999, 1.0, 1.5, 2.0, 3.9, 4.0, 4.1,
               15.9, 16.0, 16.1, 19.99, 20.0, 20.01, 49.99, 50.0, 50.01, 60.0, 63.9, 64.0, 64.1, 255.9, 256.0, 256.1,
               999.0, 1e3, 31999.5, 32000.0, 32000.5, 64000.0, 1e6, 1e8, 1e10, 3.0e38]
    vals = np.array(special + [-v for v in special], dtype=np.float32)
    g = torch.Generator().manual_seed(11)
    rnd = [torch.randn(2048, generator=g) * s for s in (0.05, 1.0, 10.0, 40.0, 1000.0)]
    return np.concatenate([vals] + [r.numpy().astype(np.float32) for r in rnd])


def quant_inputs() -> np.ndarray:
    """Rows for activation_quant_dynamic: random scales, exact .5 ties, an
    all-zero row, huge and tiny rows, and a row of identical values."""
    g = torch.Generator().manual_seed(12)
    rows = [torch.randn(48, 256, generator=g) * torch.logspace(-3, 3, 48).unsqueeze(1)]
    tie = torch.zeros(1, 256)
    tie[0, 0] = 127.0
    tie[0, 1:] = torch.arange(1, 256, dtype=torch.float32) % 254 - 126.5  # x*127/amax = k + .5
    rows += [tie, torch.zeros(1, 256), torch.full((1, 256), 3.0e38), torch.full((1, 256), 1e-12),
             torch.full((1, 256), -2.5)]
    return torch.cat(rows).numpy().astype(np.float32)


def gate_inputs():
    g = torch.Generator().manual_seed(13)
    z = np.concatenate([edge_values(), (torch.randn(4096, generator=g) * 5).numpy()]).astype(np.float32)
    y = (torch.randn(z.shape[0], generator=g) * 3).numpy().astype(np.float32)
    return y, z


def norm_inputs():
    """Rows of width 256 whose variances fall into every power-of-2 band
    (1/64 .. 65536 and beyond), with random gamma and step."""
    g = torch.Generator().manual_seed(14)
    scales = torch.logspace(-4, 3, 96)
    x = torch.randn(96, 256, generator=g) * scales.unsqueeze(1) + torch.randn(96, 1, generator=g)
    gamma = (1.0 + 0.1 * torch.randn(256, generator=g)).numpy().astype(np.float32)
    step = np.array([0.875], np.float32)
    return x.numpy().astype(np.float32), gamma, step


def scan_inputs():
    g = torch.Generator().manual_seed(15)
    B, L, DN = 2, 64, 48
    u = (torch.randn(B, L, DN, generator=g) * 2).numpy().astype(np.float32)
    nums = (torch.rand(B, L, DN, generator=g) * 32000).numpy().astype(np.float32)
    nums[:, :, 0] = 0.0
    nums[:, :, 1] = 32000.0
    nums[:, :, 2] = 16384.0
    nums[:, :, 3] = np.float32(31999.37)
    return u, nums


def weight_input() -> np.ndarray:
    g = torch.Generator().manual_seed(16)
    return (torch.randn(96, 160, generator=g) * 0.05).numpy().astype(np.float32)
