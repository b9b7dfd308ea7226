"""Decode executor: greedy generation for a batch of independent streams.

The prompt runs through the prefill kernels, which leave behind, per layer,
the last three conv inputs of every stream (the conv window) and the final
scan states h [batch, d_inner, 16].  Each new token is then one pass of step
kernels over that cached state:

    rowprep      embedding gather (+ residual later) + BitShiftNorm + int8 quant  [B, d]
    per layer:
      in_proj    tcgen05 GEMM from int8 weights          -> xz        [B, 2di]
      mid        one kernel, a 4-CTA cluster per stream: conv window +
                 ste_clamp + squareplus + int8 quant; x_proj as int8 dot
                 products on 2-bit packed weights; dt quant + dt_proj +
                 decay/dt/u + one state update + h.C + gate + int8 quant [B, di]
      out_proj   tcgen05 GEMM from int8 weights          -> out       [B, d]
      rowprep    residual += out*res_gate, next norm + quant
    lm_head GEMM, argmax -> next token ids

The reference has no step API: its generation loop recomputes
MambaIntegerModel.forward over the whole sequence for every token
(scripts/inference.py:148-160, temperature sampling).  Each step here gives
the logits that forward gives the last position, bit for bit; generation is
greedy (argmax, first index of the maximum).

Streams are independent, so multi-GPU decoding shards them across ranks
(``mamba_integer_b200.distributed.shard_range``) with no collective until the
generated ids are gathered.
"""
from __future__ import annotations

import torch

from . import kernels
from .engine import PrefillEngine
from .rational_bitnet import ternary_matmul


class StreamStates:
    """Per-layer recurrent state of `batch` streams: conv windows
    [n_layer, batch, 3, di] (the inputs at t-3, t-2, t-1) and scan states
    [n_layer, batch, di, 16]."""

    def __init__(self, n_layer: int, batch: int, di: int, N: int, dev, zero: bool = True):
        # zero=False for states a prompt prefill is about to write in full (the scan writes
        # every channel's final states, capture_window all three window rows)
        self.batch = batch
        self.di = di
        alloc = torch.zeros if zero else torch.empty
        self.win = alloc(n_layer, batch, 3, di, dtype=torch.float32, device=dev)
        self.h = alloc(n_layer, batch, di, N, dtype=torch.float32, device=dev)

    def capture_window(self, layer: int, xz: torch.Tensor, batch: int, L: int) -> None:
        """Keep the conv inputs (first di columns of xz) of the last 3 positions."""
        di = self.di
        k = min(L, 3)
        w = self.win[layer]
        if k < 3:
            w[:, : 3 - k].zero_()
        w[:, 3 - k:].copy_(xz.view(batch, L, -1)[:, L - k:, :di])


class _StepWorkspace:
    def __init__(self, B: int, d: int, di: int, R: int, N: int, V: int, dev):
        f32, i8 = torch.float32, torch.int8
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)       # input of the step
        self.next_ids = torch.zeros(B, dtype=torch.int64, device=dev)  # its argmax
        self.x = torch.empty(B, d, dtype=f32, device=dev)
        self.xq_d = torch.empty(B, d, dtype=i8, device=dev)
        self.xs_d = torch.empty(B, dtype=f32, device=dev)
        self.xz = torch.empty(B, 2 * di, dtype=f32, device=dev)
        self.act = torch.empty(B, di, dtype=f32, device=dev)
        self.xq_i = torch.empty(B, di, dtype=i8, device=dev)
        self.xs_i = torch.empty(B, dtype=f32, device=dev)
        self.xp = torch.empty(B, R + 2 * N, dtype=f32, device=dev)
        self.out = torch.empty(B, d, dtype=f32, device=dev)
        self.logits = torch.empty(B, V, dtype=f32, device=dev)


class DecodeEngine:
    """Greedy decoding over the sm_100a kernels (prompt prefill, then one step
    per token).  ``use_graph`` replays each step from a CUDA graph captured on
    the first step (the step launches no allocation and no host sync)."""

    def __init__(self, model, prefill: PrefillEngine | None = None, use_graph: bool = True, fused: bool = True,
                 packed_x: bool = True):
        self.pre = prefill if prefill is not None else PrefillEngine(model)
        self.n_layer = len(self.pre.layers)
        self.use_graph = use_graph
        # fused: one mid kernel per layer (mi_decode_mid); otherwise conv step,
        # x_proj GEMM and scan step as three launches
        self.fused = fused and self.pre.di % 16 == 0
        # packed_x: the mid kernel reads x_proj's 2-bit packed weights (mi_decode_mid_packed)
        self.packed_x = (packed_x and self.fused and self.pre.di % 64 == 0
                         and all(p["w_x"].w2 is not None for p in self.pre.layers))
        # The step's GEMMs (one row per stream) read the int8 copies of the weights:
        # at a few hundred rows they are latency-bound, and the packed form's unpack
        # hand-off lengthens every K-slice, while the 4x weight bytes cost ~20 us of
        # HBM per step (256 streams, config 5: 1.48 -> 1.41 ms per step).  The
        # prompt prefill keeps the packed weights.
        i8 = lambda tw: tw._replace(w2=None)  # noqa: E731
        self._step_w = [(i8(p["w_in"]), i8(p["w_x"]), i8(p["w_out"])) for p in self.pre.layers]
        self._step_lm = i8(self.pre.w_lm)
        self.states: StreamStates | None = None
        self.ws: _StepWorkspace | None = None
        self._graph = None

    # -- launches of one step ----------------------------------------------
    def _launch_step(self) -> None:
        pre, ws, st = self.pre, self.ws, self.states
        B = ws.ids.shape[0]
        d, di, R = pre.d, pre.di, pre.R
        layers = pre.layers
        g0, s0 = (layers[0]["gamma"], layers[0]["step"]) if layers else (pre.gamma_f, pre.step_f)
        kernels.rowprep(g0, s0, B, d, ids=ws.ids, emb=pre.emb, x_out=ws.x, xq=ws.xq_d, xscale=ws.xs_d)
        for i, p in enumerate(layers):
            w_in, w_x, w_out = self._step_w[i]
            ternary_matmul(ws.xq_d, w_in, ws.xs_d, out=ws.xz)
            if self.fused and self.packed_x:
                kernels.decode_mid_packed(ws.xz, p["conv_w"], p["conv_b"], st.win[i], p["w_x"].w2, p["w_x"].scale,
                                          R, p["w_dt"].w8, p["w_dt"].scale, p["base"], st.h[i], ws.xq_i, ws.xs_i)
            elif self.fused:
                kernels.decode_mid(ws.xz, p["conv_w"], p["conv_b"], st.win[i], p["w_x"].w8, p["w_x"].scale, R,
                                   p["w_dt"].w8, p["w_dt"].scale, p["base"], st.h[i], ws.xq_i, ws.xs_i)
            else:
                kernels.conv_step(ws.xz, p["conv_w"], p["conv_b"], st.win[i], di, ws.xq_i, ws.xs_i, act=ws.act)
                ternary_matmul(ws.xq_i, w_x, ws.xs_i, out=ws.xp)
                kernels.ssm_step(ws.act, ws.xp, R, p["w_dt"].w8, p["w_dt"].scale, ws.xz[:, di:], p["base"],
                                 st.h[i], ws.xq_i, ws.xs_i)
            ternary_matmul(ws.xq_i, w_out, ws.xs_i, out=ws.out)
            nxt = layers[i + 1] if i + 1 < len(layers) else None
            g, s = (nxt["gamma"], nxt["step"]) if nxt else (pre.gamma_f, pre.step_f)
            kernels.rowprep(g, s, B, d, x=ws.x, delta=ws.out, res_gate=p["res_gate"], x_out=ws.x, xq=ws.xq_d,
                            xscale=ws.xs_d)
        ternary_matmul(ws.xq_d, self._step_lm, ws.xs_d, out_scale=pre.out_scale, out=ws.logits)
        kernels.argmax_rows(ws.logits, out=ws.next_ids)

    def launches_per_step(self) -> int:
        return 3 + (4 if self.fused else 6) * self.n_layer

    # -- public API -----------------------------------------------------------
    def start(self, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Run the prompt [batch, L]; returns the last-position logits [batch, V]
        and leaves the streams ready for step()."""
        batch, L = prompt_ids.shape
        pre = self.pre
        if self.states is None or self.states.batch != batch:
            self.states = StreamStates(self.n_layer, batch, pre.di, pre.N, pre.dev)
            self.ws = _StepWorkspace(batch, pre.d, pre.di, pre.R, pre.N, pre.V, pre.dev)
            self._graph = None
        return pre.forward(prompt_ids.to(pre.dev), states=self.states, last_only=True)

    def reserve(self, batch: int) -> None:
        """Allocate (zeroed) state and step buffers for `batch` stream slots
        without running a prompt; prompts then enter slots with prefill_slots."""
        pre = self.pre
        if self.states is None or self.states.batch != batch:
            self.states = StreamStates(self.n_layer, batch, pre.di, pre.N, pre.dev)
            self.ws = _StepWorkspace(batch, pre.d, pre.di, pre.R, pre.N, pre.V, pre.dev)
            self._graph = None

    def prefill_slots(self, slots, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Run k prompts of one length [k, L] through the prefill kernels and put
        their streams' state into the given slots (the other slots are left as
        they are); returns their last-position logits [k, V]."""
        pre = self.pre
        k = prompt_ids.shape[0]
        tmp = StreamStates(self.n_layer, k, pre.di, pre.N, pre.dev, zero=False)
        logits = pre.forward(prompt_ids.to(pre.dev), states=tmp, last_only=True)
        idx = torch.as_tensor(list(slots), dtype=torch.int64, device=pre.dev)
        self.states.win.index_copy_(1, idx, tmp.win)
        self.states.h.index_copy_(1, idx, tmp.h)
        return logits

    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """Feed one token per stream (int64 [batch]); returns the logits of the
        new position [batch, V] (a buffer reused by the next step)."""
        ws = self.ws
        ws.ids.copy_(ids.reshape(-1))
        if not self.use_graph:
            self._launch_step()
        elif self._graph is None:
            # first step eagerly (and as the capture's warm-up), then capture one
            # step that re-runs it from the same state
            self._launch_step()
            self._capture()
        else:
            self._graph.replay()
        return ws.logits

    def _capture(self) -> None:
        # the capture records the launches without running them: the states the
        # eager step left stay as they are
        stream = torch.cuda.Stream(device=self.pre.dev)
        stream.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            self._launch_step()
        torch.cuda.current_stream().wait_stream(stream)
        self._graph = g

    @staticmethod
    def argmax(logits: torch.Tensor) -> torch.Tensor:
        """Greedy choice over logits [k, V] (int64 [k])."""
        return kernels.argmax_rows(logits)

    def next_ids(self) -> torch.Tensor:
        """argmax of the logits of the last step (int64 [batch])."""
        return self.ws.next_ids

    def generate(self, prompt_ids: torch.Tensor, n_new: int) -> torch.Tensor:
        """Greedy continuation: int64 [batch, n_new]."""
        logits = self.start(prompt_ids)
        batch = prompt_ids.shape[0]
        out = torch.empty(batch, n_new, dtype=torch.int64, device=self.pre.dev)
        if n_new == 0:
            return out
        kernels.argmax_rows(logits, out=self.ws.next_ids)
        for t in range(n_new):
            out[:, t].copy_(self.ws.next_ids)
            if t + 1 < n_new:
                self.step(self.ws.next_ids)
        return out
