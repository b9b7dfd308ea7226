"""Drop-in ``BitLinear`` and its quantisers, running on the sm_100a kernels.

Same constructor, parameter names and forward signature as the reference
(src/rational_bitnet.py:114-219).  Differences by design:
  * the ternary weights are quantised once and cached on the device, as int8
    and packed 2 bits per weight (re-quantised only when ``weight._version``
    changes); the reference re-quantises on every eval forward with identical
    results;
  * forward runs only on CUDA tensors: per-token int8 quantisation
    (mi_quantize_rows) then the tcgen05 int8 GEMM with the BitLinear rescale
    in its epilogue, fed from the 2-bit packed weights (mi_bitlinear_packed;
    mi_bitlinear_i8 when the padded input width is not a multiple of 64).
    There is no CPU path.
"""
from __future__ import annotations

import math
from typing import NamedTuple, Optional, Tuple

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


class TernaryWeights(NamedTuple):
    """Device copies of one BitLinear's quantised weights."""
    w8: torch.Tensor            # int8 {-1,0,1} [out, in padded to 16]
    w2: Optional[torch.Tensor]  # 2-bit packed uint8 [out, K/4] (None when the padded K is not a multiple of 64)
    scale: torch.Tensor         # fp32 [1]: the AbsMean scale


_SM_PAIRS: dict = {}


def _pair_kernel_wins(M: int, N: int, K: int, dev: torch.device) -> bool:
    """A GEMM heavy enough in K for the tensor cores to set its pace (K >= 1536),
    with N % 256 == 0 and a 256 x 256 tile for every SM pair: there the int8
    weights on the 2-SM kernel beat the packed weights on the one-CTA kernel
    (config-4 out_proj, K 1536: 3.83 -> 3.34 ms per step), while the store-bound
    K = 768 GEMMs (in_proj, lm_head) are faster packed."""
    if K < 1536 or N % 256 != 0:
        return False
    pairs = _SM_PAIRS.get(dev.index)
    if pairs is None:
        pairs = _SM_PAIRS[dev.index] = torch.cuda.get_device_properties(dev).multi_processor_count // 2
    return (M + 255) // 256 * (N // 256) >= pairs


def ternary_matmul(xq: torch.Tensor, tw: TernaryWeights, xs: Optional[torch.Tensor], out=None, out_scale=None,
                   K: Optional[int] = None) -> torch.Tensor:
    """xq int8 [M, K] against the ternary weights, with the BitLinear rescale
    acc * (w_scale * xs[m]) [* out_scale] (int32 accumulators if xs is None).
    The packed weights, except where the int8 copy on the 2-SM kernel is faster
    (_pair_kernel_wins); both give the same bits."""
    scale = tw.scale if xs is not None else None
    Kd = xq.shape[1] if K is None else K
    if tw.w2 is not None and not _pair_kernel_wins(xq.shape[0], tw.w8.shape[0], Kd, xq.device):
        return kernels.bitlinear_packed(xq, tw.w2, xs, scale, out_scale=out_scale, out=out, K=K)
    return kernels.bitlinear_i8(xq, tw.w8, xs, scale, out_scale=out_scale, out=out, K=K)


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
        self._cache = None  # (TernaryWeights, weight version, device)
        self._fixed = None  # (int8 {-1,0,1} [out, in], scale): quantised weights given directly

    # -- weight cache -------------------------------------------------------
    def device_weights(self, device=None) -> TernaryWeights:
        """The quantised weights on ``device``: int8 [out, in padded to 16],
        their 2-bit packed copy (packed on the GPU) and the scale."""
        device = torch.device(device) if device is not None else self.weight.device
        ver = self.weight._version
        c = self._cache
        if c is None or c[1] != ver or c[2] != device:
            if self._fixed is not None:
                wq, scale = self._fixed[0].to(torch.float32), self._fixed[1]
            else:
                wq, scale = weight_quant_ternary(self.weight)
            K16 = _pad16(self.in_features)
            w8 = torch.zeros(self.out_features, K16, dtype=torch.int8)
            w8[:, : self.in_features] = wq.to(torch.int8)
            w8 = w8.to(device)
            w2 = kernels.pack_ternary(w8) if K16 % 64 == 0 else None
            self._cache = (TernaryWeights(w8, w2, scale.reshape(1).to(device)), ver, device)
        return self._cache[0]

    @torch.no_grad()
    def get_ternary_weights(self) -> Tuple[torch.Tensor, torch.Tensor]:
        if self._fixed is not None:
            return self._fixed[0].clone(), self._fixed[1].clone()
        wq, scale = weight_quant_ternary(self.weight)
        return wq.to(torch.int8), scale

    @torch.no_grad()
    def set_ternary(self, wq: torch.Tensor, scale) -> None:
        """Use already-quantised weights (int8 {-1,0,1} [out, in] and the
        absmean scale), e.g. from the reference's int8 export, instead of
        quantising ``weight``; ``weight`` is set to wq * scale."""
        wq = torch.as_tensor(wq).to(torch.int8).reshape(self.out_features, self.in_features).cpu()
        if bool(((wq < -1) | (wq > 1)).any()):
            raise ValueError("ternary weights must be in {-1, 0, 1}")
        scale = torch.as_tensor(scale, dtype=torch.float32).reshape(()).cpu()
        self._fixed = (wq, scale)
        self.weight.copy_((wq.to(torch.float32) * scale).to(self.weight.device))
        self._cache = None

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
        y = ternary_matmul(xq, self.device_weights(x.device), xs, K=K16)
        if self.bias is not None:
            y = y + self.bias
        return y.view(*lead, self.out_features)
