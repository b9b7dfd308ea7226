"""Generate backward.npz: golden input/output pairs of the reference's two
training-side passes, computed by the UNMODIFIED reference code on the CPU.

* Convex dyadic scan backward: DyadicScanFunction.backward's sequential branch
  (src/mamba_integer_model.py:319-344), which computes the same quantities as
  the Triton fast backward the model uses on GPUs
  (src/triton_kernels/dyadic_scan.py:376-459): the reversed accumulation
  g[t] = grad_h[t] + decay[t] * g[t+1], grad_u = (1 - decay) * g and
  grad_nums = g * (h[t-1] - u) / 32768.  The branch is reached with a stand-in
  autograd context (use_ssd set, saved tensors given).
* Activation quantisation STE backward: QuantizeActivationsFunction.backward
  (src/triton_kernels/bitnet_kernels.py:77-95), plain torch arithmetic, also
  called with a stand-in context.

The reference checkout is named by $MI_REFERENCE_SRC (its src/ directory):

    MI_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_backward_golden.py
"""
from __future__ import annotations

import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def scan_case(seed: int, B: int, L: int, DN: int):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(B, L, DN, generator=g) * 2.0
    nums = torch.randint(0, 32001, (B, L, DN), generator=g).to(torch.float32)
    nums[:, :, 0] = 0.0
    nums[:, :, 1] = 32000.0
    grad_h = torch.randn(B, L, DN, generator=g)
    return u, nums, grad_h


def ste_case(seed: int, T: int, K: int):
    g = torch.Generator().manual_seed(seed)
    grad = torch.randn(T, K, generator=g) * torch.logspace(-3, 2, T).unsqueeze(1)
    amax = torch.logspace(-4, 2, T)  # rows below 0.01 take the clamped scale
    amax[3] = 0.0
    return grad, amax


def main() -> None:
    src = os.environ.get("MI_REFERENCE_SRC")
    if not src:
        raise SystemExit("set MI_REFERENCE_SRC to the reference checkout's src/ directory")
    sys.path.insert(0, src)
    import mamba_integer_model as ref_model  # noqa: E402
    from triton_kernels import bitnet_kernels as ref_bk  # noqa: E402

    out = {}
    for name, (seed, B, L, DN) in {"scan_a": (21, 2, 64, 48), "scan_b": (22, 1, 300, 40)}.items():
        u, nums, grad_h = scan_case(seed, B, L, DN)
        # the forward's values as the reference computes them (CPU branch, :301-315)
        h = ref_model.DyadicScanFunction.apply(u, nums, torch.full_like(nums, 15.0))
        ctx = SimpleNamespace(use_ssd=True, saved_tensors=(u, h, nums))
        grad_u, grad_nums, _ = ref_model.DyadicScanFunction.backward(ctx, grad_h)
        for k, v in dict(u=u, nums=nums, grad_h=grad_h, h=h, grad_u=grad_u, grad_nums=grad_nums).items():
            out[f"{name}.{k}"] = v.detach().numpy().astype(np.float32)
    for name, (seed, T, K) in {"ste_a": (23, 24, 64), "ste_b": (24, 7, 1536)}.items():
        grad, amax = ste_case(seed, T, K)
        ctx = SimpleNamespace(saved_tensors=(amax,), original_shape=(T, K))
        gx = ref_bk.QuantizeActivationsFunction.backward(ctx, grad, None)
        out[f"{name}.grad_xq"] = grad.numpy().astype(np.float32)
        out[f"{name}.amax"] = amax.numpy().astype(np.float32)
        out[f"{name}.grad_x"] = gx.numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "backward.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
