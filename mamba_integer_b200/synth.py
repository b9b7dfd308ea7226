"""Seeded synthetic inputs and weights for the five benchmark configurations.

Everything is drawn on the CPU from ``torch.Generator().manual_seed(seed)`` so
the same seed gives the same tensors on any host running this torch build.
No dataset or checkpoint is involved.

Weights follow the ternary construction W = t * 2^-e with exactly half of the
entries of t non-zero (random positions) and random signs: that realises
p(-1, 0, 1) = (0.25, 0.5, 0.25) and makes ``mean|W|`` (the BitLinear absmean
scale, src/rational_bitnet.py:79) exactly 2^-(e+1), so the per-tensor weight
scale is a power of two and independent of summation order.
"""
from __future__ import annotations

import math
from typing import Dict

import torch

# BASELINE configurations (dt_rank = ceil(d_model / 16), d_inner = 2 * d_model).
CONFIGS: Dict[str, dict] = {
    "c1": dict(d_model=256, n_layer=4, vocab_size=4096, ssm_cfg=dict(d_state=16, dt_rank=16),
               batch=2, seq_len=256, seed=0),
    "c4": dict(d_model=768, n_layer=24, vocab_size=32768, ssm_cfg=dict(d_state=16, dt_rank=48),
               batch=64, seq_len=2048, seed=3),
    "c5": dict(d_model=1024, n_layer=24, vocab_size=32768, ssm_cfg=dict(d_state=16, dt_rank=64),
               batch=256, seq_len=512, seed=4),
}


def model_config(name: str, **over) -> dict:
    """Reference-style config dict (keys read by MambaIntegerModel; no ``use_ssd``)."""
    c = dict(CONFIGS[name])
    c.update(over)
    return {"d_model": c["d_model"], "n_layer": c["n_layer"], "vocab_size": c["vocab_size"],
            "ssm_cfg": dict(c["ssm_cfg"])}


def ternary_weight(out_f: int, in_f: int, g: torch.Generator, e: int = 5) -> torch.Tensor:
    """fp32 [out_f, in_f] with entries in {-2^-e, 0, 2^-e}, exactly half non-zero."""
    n = out_f * in_f
    assert n % 2 == 0
    perm = torch.randperm(n, generator=g)
    sign = torch.randint(0, 2, (n // 2,), generator=g, dtype=torch.int64) * 2 - 1
    t = torch.zeros(n, dtype=torch.float32)
    t[perm[: n // 2]] = sign.to(torch.float32)
    return (t * (2.0 ** -e)).view(out_f, in_f)


def decay_nums(d_inner: int, d_state: int, g: torch.Generator) -> torch.Tensor:
    """Integer-valued decay multipliers uniform in [ceil(0.90*2^15), floor(0.999*2^15)]."""
    lo = math.ceil(0.90 * 32768)
    hi = math.floor(0.999 * 32768)
    return torch.randint(lo, hi + 1, (d_inner, d_state), generator=g, dtype=torch.int64).to(torch.float32)


def model_state_dict(config: dict, seed: int) -> Dict[str, torch.Tensor]:
    """A full state_dict with the reference's parameter names
    (src/mamba_integer_model.py:368-394, 449-484)."""
    g = torch.Generator().manual_seed(seed)
    d = config["d_model"]
    di = 2 * d
    N = config["ssm_cfg"]["d_state"]
    R = config["ssm_cfg"]["dt_rank"]
    nl = config["n_layer"]
    V = config["vocab_size"]
    sd: Dict[str, torch.Tensor] = {}
    sd["embedding.weight"] = torch.randn(V, d, generator=g)
    for i in range(nl):
        p = f"layers.{i}."
        sd[p + "norm.gamma"] = torch.ones(d)
        sd[p + "norm.step_size"] = torch.ones(1)
        sd[p + "in_proj.weight"] = ternary_weight(2 * di, d, g)
        sd[p + "conv1d.weight"] = (torch.rand(di, 1, 4, generator=g) - 0.5)
        sd[p + "conv1d.bias"] = (torch.rand(di, generator=g) - 0.5)
        sd[p + "x_proj.weight"] = ternary_weight(R + 2 * N, di, g)
        sd[p + "dt_proj.weight"] = ternary_weight(di, R, g)
        sd[p + "out_proj.weight"] = ternary_weight(d, di, g)
        sd[p + "base_decay_nums"] = decay_nums(di, N, g)
        sd[p + "decay_shifts"] = torch.full((di, N), 15.0)
        sd[p + "res_gate"] = torch.ones(1) / math.sqrt(2 * nl)
    sd["norm_f.gamma"] = torch.ones(d)
    sd["norm_f.step_size"] = torch.ones(1)
    sd["lm_head.weight"] = ternary_weight(V, d, g)
    return sd


def zipf_ids(batch: int, seq_len: int, vocab: int, g: torch.Generator, s: float = 1.1) -> torch.Tensor:
    """Token ids from Zipf(s) over [0, vocab) by inverse-CDF sampling."""
    ranks = torch.arange(1, vocab + 1, dtype=torch.float64)
    pmf = ranks.pow(-s)
    cdf = torch.cumsum(pmf, 0)
    cdf = cdf / cdf[-1]
    u = torch.rand(batch * seq_len, generator=g, dtype=torch.float64)
    ids = torch.searchsorted(cdf, u).clamp_(max=vocab - 1)
    return ids.view(batch, seq_len).to(torch.int64)


def input_ids(name: str, batch: int | None = None, seq_len: int | None = None) -> torch.Tensor:
    c = CONFIGS[name]
    B = batch or c["batch"]
    L = seq_len or c["seq_len"]
    g = torch.Generator().manual_seed(c["seed"] + 1000)
    if name == "c1":
        return torch.randint(0, c["vocab_size"], (B, L), generator=g, dtype=torch.int64)
    return zipf_ids(B, L, c["vocab_size"], g)


def scan_i32_inputs(batch=8, L=4096, D=2048, N=16, seed=1):
    """Config 2: x, B, C = clip(round_half_even(N(0, 32)), +-127) int32; n uniform
    integers in [0.90*2^15, 0.999*2^15]; k = 15; h0 = 0."""
    g = torch.Generator().manual_seed(seed)

    def q(*shape):
        return torch.round(torch.randn(*shape, generator=g) * 32.0).clamp_(-127, 127).to(torch.int32)

    x = q(batch, L, D)
    Bm = q(batch, L, N)
    Cm = q(batch, L, N)
    n = decay_nums(D, N, g).to(torch.int32)
    return x, Bm, Cm, n


def bitlinear_inputs(M=16384, K=2048, N=8192, seed=2):
    """Config 3: A = per-token absmax int8 quantisation of N(0,1); W ternary
    (p = .25/.5/.25) with per-tensor scale 2^-6."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g)
    s = a.abs().amax(-1, keepdim=True).clamp(min=1e-8)
    v = a * (127.0 / s)
    A = (v + (torch.round(v) - v)).clamp(-127, 127).to(torch.int8)
    a_scale = (s / 127.0).view(M)
    Wf = ternary_weight(N, K, g, e=5)  # mean|W| = 2^-6
    Wq = (Wf * 32.0).to(torch.int8)
    return A, a_scale, Wq, 2.0 ** -6


def bitlinear_norm_params(N=8192, seed=2):
    """Config 3's epilogue parameters: BitShiftNorm gain gamma [N] = 1 + 0.1 N(0, 1)
    and step size 0.875 (the reference initialises both to 1; non-trivial values
    exercise the multiplications)."""
    g = torch.Generator().manual_seed(seed + 100)
    gamma = 1.0 + 0.1 * torch.randn(N, generator=g)
    return gamma.to(torch.float32), torch.tensor([0.875], dtype=torch.float32)
