"""Drop-in ``BitLinear`` and its quantisers, running on the sm_100a kernels.

Same constructor, parameter names and forward signature as the reference
(src/rational_bitnet.py:114-219).  Differences by design:
  * the ternary weights are quantised once and cached as int8 on the device
    (re-quantised only when ``weight._version`` changes); the reference
    re-quantises on every eval forward with identical results;
  * forward runs only on CUDA tensors: per-token int8 quantisation
    (mi_quantize_rows) then the tcgen05 int8 GEMM with the BitLinear rescale
    in its epilogue (mi_bitlinear_i8).  There is no CPU path.
"""
from __future__ import annotations

import math
from typing import Tuple

import torch
import torch.nn as nn

from . import kernels


def ste_round(x: torch.Tensor) -> torch.Tensor:
    """x + (round(x) - x).detach()  (src/rational_bitnet.py:54-60)."""
    return x + (torch.round(x) - x).detach()


def weight_quant_ternary(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """AbsMean ternary quantisation (src/rational_bitnet.py:63-85).

    Evaluated with torch on the CPU exactly as the reference's CPU path does, so
    the per-tensor scale is the reference's own value (this runs once per
    weight update, not per forward)."""
    wc = w.detach().to("cpu", torch.float32)
    scale = torch.max(wc.abs().mean(), torch.tensor(1e-6, dtype=wc.dtype))
    wq = torch.clamp(ste_round(wc / scale), min=-1, max=1)
    return wq, scale


def activation_quant_dynamic(x: torch.Tensor, bits: int = 8) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-token absmax quantisation (src/rational_bitnet.py:88-111) on the GPU."""
    if bits != 8:
        raise NotImplementedError("only 8-bit activations are implemented")
    return kernels.quantize_activations(x)


def _pad16(k: int) -> int:
    return (k + 15) // 16 * 16


class BitLinear(nn.Module):
    """Linear layer with {-1, 0, 1} weights and int8 activations."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, activation_bits: int = 8,
                 is_output_layer: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.activation_bits = activation_bits
        self.is_output_layer = is_output_layer
        init_std = 1.0 / math.sqrt(in_features)
        if is_output_layer:
            init_std = init_std / math.sqrt(in_features)
        self.weight = nn.Parameter(torch.randn(out_features, in_features) * init_std)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self._packed = None  # (wq int8 [N, K16] on device, w_scale fp32 [1] on device, version, device)

    # -- weight cache -------------------------------------------------------
    def packed(self, device=None):
        """(int8 ternary weights [out, in padded to 16], w_scale [1]) on ``device``."""
        device = torch.device(device) if device is not None else self.weight.device
        ver = self.weight._version
        p = self._packed
        if p is None or p[2] != ver or p[3] != device:
            wq, scale = weight_quant_ternary(self.weight)
            K16 = _pad16(self.in_features)
            w8 = torch.zeros(self.out_features, K16, dtype=torch.int8)
            w8[:, : self.in_features] = wq.to(torch.int8)
            self._packed = (w8.to(device), scale.reshape(1).to(device), ver, device)
        return self._packed[0], self._packed[1]

    @torch.no_grad()
    def get_ternary_weights(self) -> Tuple[torch.Tensor, torch.Tensor]:
        wq, scale = weight_quant_ternary(self.weight)
        return wq.to(torch.int8), scale

    # -- forward ------------------------------------------------------------
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("BitLinear runs on the sm_100a kernels only; move the input to CUDA")
        K = self.in_features
        if x.shape[-1] != K:
            raise ValueError(f"expected last dim {K}, got {x.shape[-1]}")
        lead = x.shape[:-1]
        x2 = x.detach().to(torch.float32).reshape(-1, K).contiguous()
        T = x2.shape[0]
        K16 = _pad16(K)
        xq = torch.zeros(T, K16, dtype=torch.int8, device=x.device) if K16 != K else None
        xq, xs = kernels.quantize_rows(x2, K, out=xq)
        w8, ws = self.packed(x.device)
        y = kernels.bitlinear_i8(xq, w8, xs, ws, K=K16)
        if self.bias is not None:
            y = y + self.bias
        return y.view(*lead, self.out_features)
