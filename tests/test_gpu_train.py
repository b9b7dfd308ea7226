"""Training-side kernels on the GPU: the convex scan backward and the
activation quantisation's straight-through backward, bit for bit against the
reference's own outputs (tests/golden/backward.npz) and the oracle, directly
and through the drop-in autograd functions."""
import os

import numpy as np
import pytest
import torch

from oracle import lib as orc

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits_eq(a, b):
    a = a.detach().cpu().numpy() if torch.is_tensor(a) else a
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))


def test_backward_kernels_match_reference_golden(cuda_dev):
    from mamba_integer_b200 import kernels as k
    z = np.load(os.path.join(GOLD, "backward.npz"))
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_dev)  # noqa: E731
    for c in ("scan_a", "scan_b"):
        gu, gn = k.scan_convex_backward(d(z[c + ".grad_h"]), d(z[c + ".h"]), d(z[c + ".u"]), d(z[c + ".nums"]))
        assert _bits_eq(gu, z[c + ".grad_u"]) and _bits_eq(gn, z[c + ".grad_nums"]), c
    for c in ("ste_a", "ste_b"):
        gx = k.quant_ste_backward(d(z[c + ".grad_xq"]), d(z[c + ".amax"]))
        assert _bits_eq(gx, z[c + ".grad_x"]), c


@pytest.mark.parametrize("B,L,DN", [(3, 517, 4096), (1, 3, 40), (2, 2048, 1536)])
def test_scan_convex_backward_matches_oracle(cuda_dev, B, L, DN):
    from mamba_integer_b200 import kernels as k
    g = torch.Generator().manual_seed(B * L + DN)
    u = torch.randn(B, L, DN, generator=g) * 3
    nums = torch.randint(0, 32001, (B, L, DN), generator=g).float()
    grad_h = torch.randn(B, L, DN, generator=g)
    h = orc.scan_convex(u.numpy(), nums.numpy())
    gu_ref, gn_ref = orc.scan_convex_backward(grad_h.numpy(), h, u.numpy(), nums.numpy())
    gu, gn = k.scan_convex_backward(grad_h.to(cuda_dev), torch.from_numpy(h).to(cuda_dev), u.to(cuda_dev),
                                    nums.to(cuda_dev))
    assert _bits_eq(gu, gu_ref) and _bits_eq(gn, gn_ref)


def test_dyadic_scan_function_autograd(cuda_dev):
    from mamba_integer_b200.mamba_integer_model import DyadicScanFunction
    g = torch.Generator().manual_seed(5)
    u = (torch.randn(2, 96, 80, generator=g) * 2).to(cuda_dev).requires_grad_(True)
    nums = torch.randint(20000, 32001, (2, 96, 80), generator=g).float().to(cuda_dev).requires_grad_(True)
    shifts = torch.full((2, 96, 80), 15.0, device=cuda_dev)
    h = DyadicScanFunction.apply(u, nums, shifts)
    grad_h = torch.randn(2, 96, 80, generator=g).to(cuda_dev)
    h.backward(grad_h)
    h_ref = orc.scan_convex(u.detach().cpu().numpy(), nums.detach().cpu().numpy())
    assert _bits_eq(h, h_ref)
    gu_ref, gn_ref = orc.scan_convex_backward(grad_h.cpu().numpy(), h_ref, u.detach().cpu().numpy(),
                                              nums.detach().cpu().numpy())
    assert _bits_eq(u.grad, gu_ref) and _bits_eq(nums.grad, gn_ref)


@pytest.mark.parametrize("K", [1536, 48, 7])
def test_quantize_activations_ste_autograd(cuda_dev, K):
    from mamba_integer_b200 import kernels as k
    g = torch.Generator().manual_seed(K)
    x = (torch.randn(37, K, generator=g) * torch.logspace(-4, 2, 37).unsqueeze(1)).to(cuda_dev).requires_grad_(True)
    xq, s = k.fast_quantize_activations(x)
    q_ref, s_ref = orc.quant_rows(x.detach().cpu().numpy())
    assert np.array_equal(xq.detach().cpu().numpy(), q_ref.astype(np.float32))
    assert _bits_eq(s.view(-1), s_ref)
    gq = (torch.randn(37, K, generator=g) * 50).to(cuda_dev)
    xq.backward(gq)
    amax = np.maximum(np.abs(x.detach().cpu().numpy()).max(-1), np.float32(1e-8)).astype(np.float32)
    assert _bits_eq(x.grad, orc.quant_ste_backward(gq.cpu().numpy(), amax))


def test_quant_ste_backward_nan_scale_propagates(cuda_dev):
    from mamba_integer_b200 import kernels as k
    gq = torch.ones(2, 64, device=cuda_dev)
    amax = torch.tensor([float("nan"), 0.5], device=cuda_dev)
    gx = k.quant_ste_backward(gq, amax).cpu()
    assert torch.isnan(gx[0]).all()
    assert torch.equal(gx[1], torch.full((64,), 100.0))  # 127 / 0.5 = 254, clamped
