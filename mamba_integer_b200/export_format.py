"""The reference's int8 model export ("0xDAD1C" files) read into this build.

The layout is the write order of the reference exporter,
scripts/export_int8.py:52-135 (little-endian; the reference's C++ reader
src/cpp_engine/mamba_infer.cpp:46-118 is an unfinished stub that reads the
conv bias twice, so the exporter defines the format):

  header   uint32 x 6: 0xDAD1C, d_model, n_layer, vocab_size, d_state, dt_rank
  embedding          fp32 [vocab, d_model]
  per layer:
    norm.gamma       fp32 [d_model]
    in_proj          fp32 scale, int8 [2*d_inner, d_model]    (ternary, [out, in])
    conv1d           fp32 weight [d_inner, 1, 4], fp32 bias [d_inner]
    x_proj           fp32 scale, int8 [dt_rank + 2*d_state, d_inner]
    dt_proj          fp32 scale, int8 [d_inner, dt_rank], fp32 bias [d_inner]
    out_proj         fp32 scale, int8 [d_model, d_inner]
    base_decay_nums  int32 [d_inner, d_state]   (the parameter rounded)
    decay_shifts     int32 [d_inner, d_state]
    res_gate         fp32 [1]
  norm_f.gamma       fp32 [d_model]
  lm_head            fp32 scale, int8 [vocab, d_model]

(d_inner = 2 * d_model.)  The format carries no BitShiftNorm step_size: a
loaded model keeps the reference's initial value 1.0.  The ternary weights
enter the model as they are (BitLinear.set_ternary) and are packed 2 bits
each on the GPU like quantised fp32 weights.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np
import torch

MAGIC = 0xDAD1C


@dataclass
class ExportedLayer:
    gamma: np.ndarray
    in_proj: tuple
    conv_w: np.ndarray
    conv_b: np.ndarray
    x_proj: tuple
    dt_proj: tuple
    dt_bias: np.ndarray
    out_proj: tuple
    nums: np.ndarray
    shifts: np.ndarray
    res_gate: np.ndarray


@dataclass
class ExportedModel:
    d_model: int
    n_layer: int
    vocab_size: int
    d_state: int
    dt_rank: int
    embedding: np.ndarray = None
    layers: List[ExportedLayer] = field(default_factory=list)
    norm_f_gamma: np.ndarray = None
    lm_head: tuple = None

    def config(self) -> dict:
        return {"d_model": self.d_model, "n_layer": self.n_layer, "vocab_size": self.vocab_size,
                "ssm_cfg": {"d_state": self.d_state, "dt_rank": self.dt_rank}}


class _Reader:
    def __init__(self, data: bytes):
        self.data = data
        self.pos = 0

    def take(self, dtype, count: int, shape=None) -> np.ndarray:
        n = np.dtype(dtype).itemsize * count
        if self.pos + n > len(self.data):
            raise ValueError(f"export file truncated at byte {self.pos} (needs {n} more)")
        a = np.frombuffer(self.data, dtype=dtype, count=count, offset=self.pos).copy()
        self.pos += n
        return a.reshape(shape) if shape is not None else a

    def scale_and_int8(self, rows: int, cols: int) -> tuple:
        s = self.take("<f4", 1)[0]
        w = self.take(np.int8, rows * cols, (rows, cols))
        return np.float32(s), w


def read_export(path: str) -> ExportedModel:
    with open(path, "rb") as f:
        data = f.read()
    r = _Reader(data)
    magic, d, nl, V, N, R = (int(v) for v in r.take("<u4", 6))
    if magic != MAGIC:
        raise ValueError(f"not a 0xDAD1C export (magic {magic:#x})")
    di = 2 * d
    m = ExportedModel(d, nl, V, N, R)
    m.embedding = r.take("<f4", V * d, (V, d))
    for _ in range(nl):
        gamma = r.take("<f4", d)
        in_proj = r.scale_and_int8(2 * di, d)
        conv_w = r.take("<f4", di * 4, (di, 1, 4))
        conv_b = r.take("<f4", di)
        x_proj = r.scale_and_int8(R + 2 * N, di)
        dt_proj = r.scale_and_int8(di, R)
        dt_bias = r.take("<f4", di)
        out_proj = r.scale_and_int8(d, di)
        nums = r.take("<i4", di * N, (di, N))
        shifts = r.take("<i4", di * N, (di, N))
        res_gate = r.take("<f4", 1)
        m.layers.append(ExportedLayer(gamma, in_proj, conv_w, conv_b, x_proj, dt_proj, dt_bias, out_proj, nums,
                                      shifts, res_gate))
    m.norm_f_gamma = r.take("<f4", d)
    m.lm_head = r.scale_and_int8(V, d)
    if r.pos != len(data):
        raise ValueError(f"{len(data) - r.pos} trailing bytes after the lm_head")
    return m


def write_export(model, path: str) -> None:
    """Write a MambaIntegerModel in the same layout (the quantised weights of
    each BitLinear as get_ternary_weights() gives them)."""
    cfg = model.config
    d, nl, V = cfg["d_model"], cfg["n_layer"], cfg["vocab_size"]
    N, R = cfg["ssm_cfg"]["d_state"], cfg["ssm_cfg"]["dt_rank"]

    def f32(t) -> bytes:
        return t.detach().cpu().to(torch.float32).contiguous().numpy().tobytes()

    def lin(m) -> bytes:
        wq, s = m.get_ternary_weights()
        return struct.pack("<f", float(s)) + wq.cpu().to(torch.int8).contiguous().numpy().tobytes()

    with open(path, "wb") as f:
        f.write(struct.pack("<6I", MAGIC, d, nl, V, N, R))
        f.write(f32(model.embedding.weight))
        for blk in model.layers:
            f.write(f32(blk.norm.gamma))
            f.write(lin(blk.in_proj))
            f.write(f32(blk.conv1d.weight))
            f.write(f32(blk.conv1d.bias))
            f.write(lin(blk.x_proj))
            f.write(lin(blk.dt_proj))
            bias = blk.dt_proj.bias
            f.write(f32(bias) if bias is not None else np.zeros(blk.dt_proj.out_features, np.float32).tobytes())
            f.write(lin(blk.out_proj))
            f.write(blk.base_decay_nums.detach().round().to(torch.int32).cpu().numpy().tobytes())
            f.write(blk.decay_shifts.detach().to(torch.int32).cpu().numpy().tobytes())
            f.write(f32(blk.res_gate))
        f.write(f32(model.norm_f.gamma))
        f.write(lin(model.lm_head))


@torch.no_grad()
def load_export(path: str, device=None):
    """A MambaIntegerModel built from a 0xDAD1C export (on `device` if given)."""
    from .mamba_integer_model import MambaIntegerModel
    e = read_export(path)
    model = MambaIntegerModel(e.config())
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    model.embedding.weight.copy_(t(e.embedding))
    for blk, L in zip(model.layers, e.layers):
        if np.any(L.dt_bias != 0):
            raise ValueError("dt_proj carries a bias in this export; the model's dt_proj has none")
        blk.norm.gamma.copy_(t(L.gamma))
        blk.in_proj.set_ternary(t(L.in_proj[1]), L.in_proj[0])
        blk.conv1d.weight.copy_(t(L.conv_w))
        blk.conv1d.bias.copy_(t(L.conv_b))
        blk.x_proj.set_ternary(t(L.x_proj[1]), L.x_proj[0])
        blk.dt_proj.set_ternary(t(L.dt_proj[1]), L.dt_proj[0])
        blk.out_proj.set_ternary(t(L.out_proj[1]), L.out_proj[0])
        blk.base_decay_nums.copy_(t(L.nums).to(torch.float32))
        blk.decay_shifts.copy_(t(L.shifts).to(torch.float32))
        blk.res_gate.copy_(t(L.res_gate))
    model.norm_f.gamma.copy_(t(e.norm_f_gamma))
    model.lm_head.set_ternary(t(e.lm_head[1]), e.lm_head[0])
    return model.to(device) if device is not None else model
