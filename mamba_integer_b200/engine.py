"""Prefill executor: runs MambaIntegerModel.forward as a fixed sequence of
sm_100a kernel launches over workspace buffers that are allocated once per
(batch, seq_len) and reused.

Per layer (T = batch*seq_len tokens, d = d_model, di = 2*d_model):
    rowprep      residual += out*res_gate; BitShiftNorm; int8 quant   [T, d]
    in_proj      tcgen05 GEMM  [T, d]  x [2di, d]^T  -> xz fp32        [T, 2di]
    conv_act     conv + ste_clamp + squareplus + int8 quant (one kernel) [T, di]
    x_proj       tcgen05 GEMM  [T, di] x [R+2N, di]^T -> dt | B | C    [T, R+2N]
    dt quant     int8 quant of the dt columns                          [T, R]
    ssm_scan     dt_proj (int8 dot products by dp4a) / decay / dt / u /
                 convex scan / h.C / gate                              [T, di]
    y quant      int8 quant                                            [T, di]
    out_proj     tcgen05 GEMM  [T, di] x [d, di]^T  -> out              [T, d]
then norm_f + lm_head (GEMM with the output_scale in its epilogue).
The GEMMs read the weights packed 2 bits each (mi_bitlinear_packed).
The residual add of each block is folded into the next row pre-pass.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import kernels
from .rational_bitnet import ternary_matmul


def _pad16(k: int) -> int:
    return (k + 15) // 16 * 16


class _Workspace:
    def __init__(self, T: int, d: int, di: int, R: int, N: int, dev):
        f32, i8 = torch.float32, torch.int8
        self.x = torch.empty(T, d, dtype=f32, device=dev)
        self.xq_d = torch.empty(T, d, dtype=i8, device=dev)
        self.xs_d = torch.empty(T, dtype=f32, device=dev)
        self.xz = torch.empty(T, 2 * di, dtype=f32, device=dev)
        self.act = torch.empty(T, di, dtype=f32, device=dev)
        self.xq_i = torch.empty(T, di, dtype=i8, device=dev)
        self.xs_i = torch.empty(T, dtype=f32, device=dev)
        self.xp = torch.empty(T, R + 2 * N, dtype=f32, device=dev)
        self.dtq = torch.zeros(T, _pad16(R), dtype=i8, device=dev)
        self.dts = torch.empty(T, dtype=f32, device=dev)
        self.y = torch.empty(T, di, dtype=f32, device=dev)
        self.out = torch.empty(T, d, dtype=f32, device=dev)
        # row maxima of the scan output (zero-filled by the dt quantisation before each scan)
        self.amax = torch.empty(T, dtype=f32, device=dev)


def _layer_params(blk, dev):
    d = blk.config["d_model"]
    di = 2 * d
    f = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
    return dict(
        gamma=f(blk.norm.gamma), step=f(blk.norm.step_size).reshape(1),
        w_in=blk.in_proj.device_weights(dev), w_x=blk.x_proj.device_weights(dev),
        w_dt=blk.dt_proj.device_weights(dev), w_out=blk.out_proj.device_weights(dev),
        conv_w=f(blk.conv1d.weight).reshape(di, 4).contiguous(), conv_b=f(blk.conv1d.bias),
        base=f(blk.base_decay_nums), res_gate=f(blk.res_gate).reshape(1),
    )


def _check_shifts(blk):
    """decay_shifts must be 15 everywhere (the reference's only shift).  Checked on a
    host copy (a device-to-host copy, no kernel) once per version of the buffer."""
    t = blk.decay_shifts
    key = (t.device, t.data_ptr(), t._version)
    if getattr(blk, "_shifts_checked", None) == key:
        return
    if not bool((t.detach().cpu() == 15).all()):
        raise ValueError("decay_shifts must be 15 everywhere (the reference's only shift)")
    blk._shifts_checked = key


class _NoTimer:
    def __call__(self, name):
        return self

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


NO_TIMER = _NoTimer()

# kernel launches of one forward: 1 embedding row pre-pass, 8 per layer, 1 lm_head
def launches_per_forward(n_layer: int) -> int:
    return 2 + 8 * n_layer


def _ssm_half(p, ws: _Workspace, batch: int, L: int, d: int, di: int, R: int, N: int, timer=NO_TIMER,
              scan_split: int = 0, h_out=None):
    """Everything between the in_proj output (ws.xz) and the out_proj output (ws.out)."""
    with timer("conv_act_quant"):
        kernels.conv_act_quant_rows(ws.xz, p["conv_w"], p["conv_b"], batch, L, di, act=ws.act, xq=ws.xq_i,
                                    xscale=ws.xs_i)
    with timer("gemm_x_proj"):
        ternary_matmul(ws.xq_i, p["w_x"], ws.xs_i, out=ws.xp)
    with timer("quant_dt"):
        kernels.quantize_rows(ws.xp, K=R, out=ws.dtq, xscale=ws.dts, clear=ws.amax)
    with timer("ssm_scan"):
        # dt_proj is fused into the scan (each channel's dot product by dp4a); ws.amax was
        # zero-filled by the dt quantisation just before
        kernels.ssm_scan_dt(ws.act, ws.xp[:, R:], ws.dtq, ws.dts, p["w_dt"].w8, p["w_dt"].scale, R, ws.xz[:, di:],
                            p["base"], batch, L, y=ws.y, amax=ws.amax, split=scan_split, h_out=h_out)
    with timer("quant_y"):
        kernels.quantize_rows(ws.y, out=ws.xq_i, xscale=ws.xs_i, amax=ws.amax)
    with timer("gemm_out_proj"):
        ternary_matmul(ws.xq_i, p["w_out"], ws.xs_i, out=ws.out)


class PrefillEngine:
    """Holds device copies of the quantised weights (2-bit packed) and the per-shape workspaces."""

    def __init__(self, model):
        cfg = model.config
        self.d = cfg["d_model"]
        self.di = 2 * self.d
        self.N = cfg["ssm_cfg"]["d_state"]
        self.R = cfg["ssm_cfg"]["dt_rank"]
        self.V = cfg["vocab_size"]
        dev = model.embedding.weight.device
        if dev.type != "cuda":
            raise RuntimeError("move the model to CUDA before running it (there is no CPU path)")
        self.dev = dev
        for blk in model.layers:
            _check_shifts(blk)
        self.layers = [_layer_params(blk, dev) for blk in model.layers]
        f = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()  # noqa: E731
        self.emb = f(model.embedding.weight)
        self.gamma_f = f(model.norm_f.gamma)
        self.step_f = f(model.norm_f.step_size).reshape(1)
        self.w_lm = model.lm_head.device_weights(dev)
        self.out_scale = torch.tensor([model.output_scale], dtype=torch.float32, device=dev)
        self._versions = self._version_key(model)
        self._ws: Dict[Tuple[int, int], _Workspace] = {}
        # lanes per channel of the fused scan (0: chosen per launch from batch x channels)
        self.scan_split = 0

    @staticmethod
    def _version_key(model):
        return (model.embedding.weight.device, tuple(p._version for p in model.parameters()))

    def matches(self, model) -> bool:
        return self._versions == self._version_key(model)

    def workspace(self, batch: int, L: int) -> _Workspace:
        key = (batch, L)
        if key not in self._ws:
            self._ws.clear()  # keep at most one shape resident
            self._ws[key] = _Workspace(batch * L, self.d, self.di, self.R, self.N, self.dev)
        return self._ws[key]

    def forward(self, input_ids: torch.Tensor, logits: torch.Tensor | None = None, timer=NO_TIMER, states=None,
                last_only: bool = False) -> torch.Tensor:
        """Logits [batch, L, vocab] for int64 ids [batch, L] on this engine's device
        ([batch, vocab] of the last position with ``last_only``).
        ``timer(name)`` (a context manager factory) brackets each kernel launch.
        ``states`` (a decode.StreamStates for this batch) receives each layer's
        conv window and final scan states, for decoding after the prompt."""
        batch, L = input_ids.shape
        T = batch * L
        d, di, R, N, V = self.d, self.di, self.R, self.N, self.V
        ws = self.workspace(batch, L)
        ids = input_ids.reshape(-1).contiguous()
        if ids.dtype != torch.int64:
            ids = ids.to(torch.int64)
        p0 = self.layers[0] if self.layers else None
        g0, s0 = (p0["gamma"], p0["step"]) if p0 else (self.gamma_f, self.step_f)
        with timer("rowprep"):
            kernels.rowprep(g0, s0, T, d, ids=ids, emb=self.emb, x_out=ws.x, xq=ws.xq_d, xscale=ws.xs_d)
        for i, p in enumerate(self.layers):
            with timer("gemm_in_proj"):
                ternary_matmul(ws.xq_d, p["w_in"], ws.xs_d, out=ws.xz)
            if states is not None:
                states.capture_window(i, ws.xz, batch, L)
            _ssm_half(p, ws, batch, L, d, di, R, N, timer, self.scan_split,
                      h_out=states.h[i] if states is not None else None)
            nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
            g, s = (nxt["gamma"], nxt["step"]) if nxt else (self.gamma_f, self.step_f)
            with timer("rowprep"):
                kernels.rowprep(g, s, T, d, x=ws.x, delta=ws.out, res_gate=p["res_gate"], x_out=ws.x,
                                xq=ws.xq_d, xscale=ws.xs_d)
        if last_only:
            # norm_f rows of the last positions only: A rows of stride L*d, their scales gathered
            xq_last = ws.xq_d.view(batch, L, d)[:, L - 1, :]
            xs_last = ws.xs_d.view(batch, L)[:, L - 1].contiguous()
            if logits is None:
                logits = torch.empty(batch, V, dtype=torch.float32, device=self.dev)
            with timer("gemm_lm_head"):
                ternary_matmul(xq_last, self.w_lm, xs_last, out_scale=self.out_scale, out=logits.view(batch, V))
            return logits.view(batch, V)
        if logits is None:
            logits = torch.empty(T, V, dtype=torch.float32, device=self.dev)
        with timer("gemm_lm_head"):
            ternary_matmul(ws.xq_d, self.w_lm, ws.xs_d, out_scale=self.out_scale, out=logits.view(T, V))
        return logits.view(batch, L, V)


def run_block(blk, hidden_states: torch.Tensor) -> torch.Tensor:
    """MambaIntegerBlock.forward (src/mamba_integer_model.py:396-447) on the GPU."""
    if not hidden_states.is_cuda:
        raise RuntimeError("MambaIntegerBlock runs on the sm_100a kernels only")
    _check_shifts(blk)
    batch, L, d = hidden_states.shape
    di = 2 * d
    R = blk.config["ssm_cfg"]["dt_rank"]
    N = blk.config["ssm_cfg"]["d_state"]
    dev = hidden_states.device
    p = _layer_params(blk, dev)
    ws = _Workspace(batch * L, d, di, R, N, dev)
    x = hidden_states.detach().float().contiguous().view(batch * L, d)
    kernels.rowprep(p["gamma"], p["step"], batch * L, d, x=x, xq=ws.xq_d, xscale=ws.xs_d)
    ternary_matmul(ws.xq_d, p["w_in"], ws.xs_d, out=ws.xz)
    _ssm_half(p, ws, batch, L, d, di, R, N)
    out = torch.empty_like(x)
    kernels.rowprep(p["gamma"], p["step"], batch * L, d, x=x, delta=ws.out, res_gate=p["res_gate"], x_out=out)
    return out.view(batch, L, d)
