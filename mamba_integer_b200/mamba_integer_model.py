"""Drop-in ``MambaIntegerModel`` / ``MambaIntegerBlock`` / ``BitShiftNorm`` on
the sm_100a kernels.

Same class names, constructor arguments (reference config dict), parameter and
buffer names (so reference checkpoints load with ``load_state_dict``) and
forward signatures as src/mamba_integer_model.py:368-495.  Forward runs only
on CUDA; results are bit-identical to the reference's CPU path (the parity
tests compare against the C restatement in oracle/, itself pinned to the
reference by golden fixtures).

The block forward is the fused pipeline
    rowprep (norm + int8 quant) -> in_proj GEMM -> conv/act/quant ->
    x_proj GEMM -> dt quant -> dt_proj GEMM -> fused selective scan + gate ->
    quant -> out_proj GEMM -> residual (folded into the next rowprep)
and ``MambaIntegerModel.forward`` strings the blocks together through
:class:`mamba_integer_b200.engine.PrefillEngine`.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import kernels
from .rational_bitnet import BitLinear


class BitShiftNormFunction(torch.autograd.Function):
    """Forward of src/mamba_integer_model.py:199-222 (input already centred once
    by the caller, as BitShiftNorm.forward does)."""

    @staticmethod
    def forward(ctx, x, gamma, step_size):
        y, _ = kernels.bitshift_norm(x.contiguous(), gamma, step_size, center_once=True)
        return y

    @staticmethod
    def backward(ctx, grad_output):  # pragma: no cover - inference build
        raise NotImplementedError("training-side kernels are not part of this build")


class DyadicScanFunction(torch.autograd.Function):
    """src/mamba_integer_model.py:260-366 (convex combination scan, decay = nums / 2^15):
    forward on mi_scan_convex, backward on mi_scan_convex_backward (the quantities of
    the reference's fast backward, src/triton_kernels/dyadic_scan.py:376-459)."""

    @staticmethod
    def forward(ctx, u, decay_nums, decay_shifts):
        if not bool((decay_shifts == 15).all()):
            raise ValueError("this build supports decay_shifts == 15 only (the reference fast path)")
        u32 = u.detach().contiguous().float()
        n32 = decay_nums.detach().contiguous().float()
        h = kernels.scan_convex(u32, n32)
        ctx.save_for_backward(u32, h, n32)
        return h

    @staticmethod
    def backward(ctx, grad_h):
        u, h, nums = ctx.saved_tensors
        grad_u, grad_nums = kernels.scan_convex_backward(grad_h.contiguous().float(), h, u, nums)
        return grad_u, grad_nums, None


class BitShiftNorm(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.gamma = nn.Parameter(torch.ones(dim))
        self.step_size = nn.Parameter(torch.ones(1))

    def forward(self, x):
        if not x.is_cuda:
            raise RuntimeError("BitShiftNorm runs on the sm_100a kernels only")
        y, _ = kernels.bitshift_norm(x.detach().float().contiguous(), self.gamma, self.step_size)
        return y


class MambaIntegerBlock(nn.Module):
    def __init__(self, config, layer_idx):
        super().__init__()
        self.config = config
        d_model, d_state = config["d_model"], config["ssm_cfg"]["d_state"]
        d_inner = d_model * 2
        dt_rank = config["ssm_cfg"]["dt_rank"]
        self.layer_idx = layer_idx
        self.norm = BitShiftNorm(d_model)
        self.in_proj = BitLinear(d_model, d_inner * 2)
        self.conv1d = nn.Conv1d(d_inner, d_inner, 4, groups=d_inner, padding=3)
        self.x_proj = BitLinear(d_inner, dt_rank + 2 * d_state)
        self.dt_proj = BitLinear(dt_rank, d_inner)
        self.out_proj = BitLinear(d_inner, d_model)
        self.base_decay_nums = nn.Parameter(torch.ones(d_inner, d_state) * 16384.0)
        self.register_buffer("decay_shifts", torch.ones(d_inner, d_state) * 15.0)
        n_layer = config.get("n_layer", 24)
        self.res_gate = nn.Parameter(torch.ones(1) / math.sqrt(2 * n_layer))

    def forward(self, hidden_states):
        from .engine import run_block

        return run_block(self, hidden_states)


class MambaIntegerModel(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        if config.get("ssm_cfg", {}).get("use_ssd", False):
            raise NotImplementedError("the multi-head SSD block (use_ssd) is not part of this build")
        self.embedding = nn.Embedding(config["vocab_size"], config["d_model"])
        self.layers = nn.ModuleList([MambaIntegerBlock(config, i) for i in range(config["n_layer"])])
        self.norm_f = BitShiftNorm(config["d_model"])
        self.lm_head = BitLinear(config["d_model"], config["vocab_size"])
        self.output_scale = 1.0 / math.sqrt(config["d_model"])
        self.gradient_checkpointing = False
        self._engine = None

    def engine(self):
        from .engine import PrefillEngine

        if self._engine is None or not self._engine.matches(self):
            self._engine = PrefillEngine(self)
        return self._engine

    def forward(self, input_ids):
        if not input_ids.is_cuda:
            raise RuntimeError("MambaIntegerModel runs on the sm_100a kernels only; move input_ids to CUDA")
        return self.engine().forward(input_ids)
