"""Oracle forward of MambaIntegerModel built from the C stage restatements.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__``).

``forward`` follows MambaIntegerModel.forward (src/mamba_integer_model.py:486-495)
and MambaIntegerBlock.forward (:396-447) stage by stage on numpy arrays.  With
``capture`` it records every stage output under the names used by the parity
tests.
"""
from __future__ import annotations

from typing import Dict, Optional

import numpy as np

from . import lib


def weight_quant(w) -> tuple:
    """weight_quant_ternary (src/rational_bitnet.py:63-85): the absmean scale is
    computed with the same torch CPU call as the reference; the ternary values
    by the C restatement."""
    import torch

    wt = torch.as_tensor(np.ascontiguousarray(w, dtype=np.float32))
    scale = torch.max(wt.abs().mean(), torch.tensor(1e-6, dtype=wt.dtype))
    s = np.float32(scale.item())
    return lib.ternarize(wt.numpy(), s), s


def _np(t):
    if hasattr(t, "detach"):
        return t.detach().cpu().numpy()
    return np.asarray(t)


def prepare(sd) -> Dict[str, object]:
    """Quantise every BitLinear weight once (the reference re-quantises per call;
    the values are identical)."""
    out: Dict[str, object] = {}
    for k, v in sd.items():
        a = _np(v)
        if k.endswith("proj.weight") or k == "lm_head.weight":
            out[k] = weight_quant(a)
        else:
            out[k] = a.astype(np.float32) if a.dtype != np.float32 else a
    return out


def _bitlinear(xf, wq_ws, nthreads, cap, name):
    xq, xs = lib.quant_rows(xf, nthreads)
    wq, ws = wq_ws
    out = lib.bitlinear(xq.reshape(-1, xq.shape[-1]), xs, wq, ws, nthreads=nthreads)
    if cap is not None:
        cap[name + ".xq"] = xq.reshape(-1, xq.shape[-1])
        cap[name + ".xscale"] = xs
        cap[name + ".out"] = out.copy()
    return out


def block_forward(p: Dict[str, object], prefix: str, config: dict, x: np.ndarray, Bsz: int, L: int,
                  nthreads: int = 0, cap: Optional[dict] = None) -> np.ndarray:
    d = config["d_model"]
    di = 2 * d
    N = config["ssm_cfg"]["d_state"]
    R = config["ssm_cfg"]["dt_rank"]
    c = None if cap is None else {}
    hn, inv = lib.bitshift_norm(x, p[prefix + "norm.gamma"], p[prefix + "norm.step_size"].reshape(-1)[0],
                                nthreads)
    if c is not None:
        c["norm.out"] = hn
        c["norm.inv_rms"] = inv
    xz = _bitlinear(hn, p[prefix + "in_proj.weight"], nthreads, c, "in_proj")
    xin = np.ascontiguousarray(xz[:, :di])
    z = np.ascontiguousarray(xz[:, di:])
    conv, act = lib.conv_sqp(xin.reshape(Bsz, L, di), p[prefix + "conv1d.weight"], p[prefix + "conv1d.bias"],
                             nthreads)
    act = act.reshape(Bsz * L, di)
    if c is not None:
        c["conv.out"] = conv.reshape(Bsz * L, di)
        c["act.out"] = act
    xp = _bitlinear(act, p[prefix + "x_proj.weight"], nthreads, c, "x_proj")
    dt = np.ascontiguousarray(xp[:, :R])
    bc = np.ascontiguousarray(xp[:, R:])
    modraw = _bitlinear(dt, p[prefix + "dt_proj.weight"], nthreads, c, "dt_proj")
    yg = lib.ssm(act, bc, modraw, z, p[prefix + "base_decay_nums"], Bsz, L, nthreads=nthreads)
    if c is not None:
        c["ssm.out"] = yg
    out = _bitlinear(yg, p[prefix + "out_proj.weight"], nthreads, c, "out_proj")
    g = p[prefix + "res_gate"].reshape(-1)[0]
    y = lib.residual(x, out, g)
    if cap is not None:
        c["block.out"] = y
        cap.update({prefix + k: v for k, v in c.items()})
    return y


def forward(p: Dict[str, object], config: dict, ids: np.ndarray, nthreads: int = 0,
            cap: Optional[dict] = None, n_layer: Optional[int] = None) -> np.ndarray:
    """Logits [B, L, V] fp32 for int64 ids [B, L]; ``p`` from :func:`prepare`."""
    ids = np.asarray(ids)
    Bsz, L = ids.shape
    d = config["d_model"]
    for k in ("decay_shifts",):
        for name, v in p.items():
            if name.endswith(k) and not np.all(v == 15.0):
                raise ValueError("decay_shifts must all be 15")
    x = np.ascontiguousarray(p["embedding.weight"][ids.reshape(-1)])
    if cap is not None:
        cap["embedding.out"] = x
    nl = config["n_layer"] if n_layer is None else n_layer
    for i in range(nl):
        x = block_forward(p, f"layers.{i}.", config, x, Bsz, L, nthreads, cap)
    xn, _ = lib.bitshift_norm(x, p["norm_f.gamma"], p["norm_f.step_size"].reshape(-1)[0], nthreads)
    if cap is not None:
        cap["norm_f.out"] = xn
    logits = _bitlinear(xn, p["lm_head.weight"], nthreads, cap, "lm_head")
    lib.scale_(logits, np.float32(1.0 / np.sqrt(d)))
    return logits.reshape(Bsz, L, -1)
