"""Decoding on the GPU against the CPU oracle.

The reference decodes by recomputing MambaIntegerModel.forward over the whole
sequence for every token (scripts/inference.py:148-160).  So the check for
each step is: its logits equal, bit for bit, the oracle's full forward over
prompt + tokens so far at the last position, and the greedy token is that
row's first maximum.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import lib as orc

pytestmark = pytest.mark.gpu


def _model(cfg, sd, dev):
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    return m.to(dev).eval()


def _first_argmax(a):
    return np.argmax(a, axis=-1)  # first index of the maximum (no NaN in these logits)


@pytest.mark.parametrize("use_graph,fused", [(False, False), (True, False), (False, True), (True, True)])
@pytest.mark.parametrize("name,batch,prompt,n_new", [("c1", 3, 20, 5), ("c5s", 2, 2, 4)])
def test_greedy_decode_equals_full_recompute(cuda_dev, use_graph, fused, name, batch, prompt, n_new):
    from mamba_integer_b200 import synth
    from mamba_integer_b200.decode import DecodeEngine
    from oracle import model as om
    cfg, sd, _ = cases.model_inputs(name)
    ids = synth.input_ids(cases.MODEL_CASES[name]["base"], batch, prompt)
    m = _model(cfg, sd, cuda_dev)
    eng = DecodeEngine(m, use_graph=use_graph, fused=fused)
    assert eng.fused == fused
    p = om.prepare(sd)
    seq = ids.numpy()
    logits = eng.start(ids.to(cuda_dev)).cpu().numpy()
    for t in range(n_new):
        ref = om.forward(p, cfg, seq)[:, -1, :]
        bad = logits.view(np.uint32) != ref.view(np.uint32)
        assert not bad.any(), f"step {t}: {int(bad.sum())} logits differ from the full recompute"
        nxt = _first_argmax(ref)
        if t == 0:
            from mamba_integer_b200 import kernels
            got = kernels.argmax_rows(torch.from_numpy(logits).to(cuda_dev)).cpu().numpy()
        else:
            got = eng.next_ids().cpu().numpy()
        assert (got == nxt).all(), f"step {t}: greedy ids {got} vs {nxt}"
        seq = np.concatenate([seq, nxt[:, None]], axis=1)
        logits = eng.step(torch.from_numpy(nxt).to(cuda_dev)).cpu().numpy()


def test_generate_matches_stepwise_oracle(cuda_dev):
    from mamba_integer_b200 import synth
    from mamba_integer_b200.decode import DecodeEngine
    from oracle import model as om
    cfg, sd, _ = cases.model_inputs("c1")
    ids = synth.input_ids("c1", 2, 9)
    m = _model(cfg, sd, cuda_dev)
    out = DecodeEngine(m).generate(ids.to(cuda_dev), 4).cpu().numpy()
    p = om.prepare(sd)
    seq = ids.numpy()
    for t in range(4):
        nxt = _first_argmax(om.forward(p, cfg, seq)[:, -1, :])
        assert (out[:, t] == nxt).all(), t
        seq = np.concatenate([seq, nxt[:, None]], axis=1)


def test_prefill_final_states_match_oracle(cuda_dev):
    """h_out of the fused scan = the oracle's state after the last position."""
    from mamba_integer_b200 import kernels
    bsz, L, D, R = 2, 37, 160, 16
    g = torch.Generator().manual_seed(5)
    act = (torch.rand(bsz * L, D, generator=g) * 3).float()
    bc = (torch.randn(bsz * L, 2 * 16, generator=g)).float()
    dt = (torch.randn(bsz * L, R, generator=g)).float()
    z = (torch.randn(bsz * L, D, generator=g) * 2).float()
    base = torch.randint(29492, 32736, (D, 16), generator=g).float()
    wdt = torch.randint(-1, 2, (D, R), generator=g, dtype=torch.int8)
    ws = 2.0 ** -6
    dtq, dts = orc.quant_rows(dt.numpy())
    modraw = orc.bitlinear(dtq, dts, wdt.numpy(), ws)
    y_ref, h_ref = orc.ssm(act.numpy(), bc.numpy(), modraw, z.numpy(), base.numpy(), bsz, L, want_h=True)
    dv = lambda t: t.to(cuda_dev)  # noqa: E731
    dtq_d = torch.zeros(bsz * L, 16, dtype=torch.int8)
    dtq_d[:, :R] = torch.from_numpy(dtq)
    h = torch.full((bsz, D, 16), float("nan"), device=cuda_dev)
    for split in (1, 2, 3, 4, 8):
        y = kernels.ssm_scan_dt(dv(act), dv(bc), dv(dtq_d), dv(torch.from_numpy(dts)), dv(wdt),
                                torch.tensor([ws], device=cuda_dev), R, dv(z), dv(base), bsz, L, split=split,
                                h_out=h)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), y_ref.view(np.uint32)), split
        assert np.array_equal(h.cpu().numpy().view(np.uint32), h_ref.view(np.uint32)), split


@pytest.mark.parametrize("V,ld", [(32768, 32768), (1001, 1001), (4096, 4100), (6, 6)])
def test_argmax_rows_matches_torch(cuda_dev, V, ld):
    """Full-vocabulary rows (16-byte loads), widths that are not a multiple of 4
    and strided rows (element by element); ties and NaNs placed on different
    float4 components and threads."""
    from mamba_integer_b200 import kernels
    g = torch.Generator().manual_seed(V + ld)
    full = torch.randn(9, ld, generator=g)
    x = full[:, :V]
    x[0, V - 1] = x[0, 1] = 9.0         # tie: the lower index, other component
    x[1, min(V - 1, V // 2 + 2)] = x[1, min(V - 1, V // 2 + 2) - 1] = 9.0
    x[2, V - 2] = float("nan")
    x[2, V // 3] = float("nan")         # first NaN wins
    x[3, :] = -float("inf")
    x[4, :] = 1.0                       # all equal: index 0
    x[5, V - 1] = float("inf")
    x[6, min(5, V - 1)] = 7.0
    x[6, V - 1] = 7.0
    got = kernels.argmax_rows(x.to(cuda_dev)).cpu()
    assert got.tolist() == torch.argmax(x, dim=-1).tolist()


def test_argmax_rows_ties_nan_and_inf(cuda_dev):
    from mamba_integer_b200 import kernels
    x = torch.randn(6, 1000)
    x[0, 17] = x[0, 900] = 50.0            # tie: first index
    x[1, :] = -float("inf")                 # all -inf: index 0
    x[2, 5] = float("nan")                  # NaN counts as the maximum
    x[2, 7] = float("nan")
    x[3, 999] = float("inf")
    x[4, :] = 0.0
    x[4, 3] = -0.0                          # -0 == +0: still index 0
    got = kernels.argmax_rows(x.to(cuda_dev)).cpu()
    assert got.tolist() == torch.argmax(x, dim=-1).tolist() == [17, 0, 5, 999, 0, got[5].item()]
    assert got[5].item() == int(torch.argmax(x[5]))


@pytest.mark.parametrize("D,R,B", [(80, 16, 37), (256, 16, 37), (576, 48, 37), (2048, 64, 37), (4096, 48, 37),
                                   (2048, 64, 100), (2048, 64, 256)])
def test_decode_mid_equals_unfused_step_kernels(cuda_dev, D, R, B):
    # mi_decode_mid (one CTA per stream for D % 64 != 0, a 4-CTA cluster per stream otherwise)
    # and mi_decode_mid_packed (the cluster kernel on 2-bit packed x_proj weights; D % 64 == 0)
    # against conv step -> x_proj GEMM -> scan step, each of which is checked against the oracle.
    # The cluster kernel's CTA width follows the stream count: 37 streams at D = 2048 / 4096 run
    # 512-thread CTAs (1 / 2 channels a thread), 100 streams 256 threads, 256 streams 128
    # threads (4 channels a thread); D = 576 and 256 run 128 threads with some of them idle
    from mamba_integer_b200 import kernels as k
    g = torch.Generator().manual_seed(D + R + B)
    N, P = 16, R + 32
    R16 = (R + 15) // 16 * 16
    dv = lambda t: t.to(cuda_dev)  # noqa: E731
    xz = dv(torch.randn(B, 2 * D, generator=g) * 2)
    cw = dv((torch.rand(D, 4, generator=g) - 0.5).contiguous())
    cb = dv(torch.rand(D, generator=g) - 0.5)
    win0 = torch.randn(B, 3, D, generator=g)
    w_x = dv(torch.randint(-1, 2, (P, D), generator=g, dtype=torch.int8))
    w_x_scale = dv(torch.tensor([2.0 ** -6]))
    w_dt = torch.zeros(D, R16, dtype=torch.int8)
    w_dt[:, :R] = torch.randint(-1, 2, (D, R), generator=g, dtype=torch.int8)
    w_dt, w_dt_scale = dv(w_dt), dv(torch.tensor([2.0 ** -5]))
    base = dv(torch.randint(29492, 32736, (D, N), generator=g).float())
    h0 = torch.randn(B, D, N, generator=g)
    # unfused
    win1, h1 = dv(win0.clone()), dv(h0.clone())
    act = torch.empty(B, D, device=cuda_dev)
    xq1, xs1 = torch.empty(B, D, dtype=torch.int8, device=cuda_dev), torch.empty(B, device=cuda_dev)
    k.conv_step(xz, cw, cb, win1, D, xq1, xs1, act=act)
    xp = k.bitlinear_i8(xq1, w_x, xs1, w_x_scale)
    yq1, ys1 = torch.empty(B, D, dtype=torch.int8, device=cuda_dev), torch.empty(B, device=cuda_dev)
    k.ssm_step(act, xp, R, w_dt, w_dt_scale, xz[:, D:], base, h1, yq1, ys1)
    # fused
    win2, h2 = dv(win0.clone()), dv(h0.clone())
    yq2, ys2 = torch.empty(B, D, dtype=torch.int8, device=cuda_dev), torch.empty(B, device=cuda_dev)
    xp2 = torch.empty(B, P, device=cuda_dev)
    k.decode_mid(xz, cw, cb, win2, w_x, w_x_scale, R, w_dt, w_dt_scale, base, h2, yq2, ys2, xp_out=xp2)
    assert torch.equal(win1, win2)
    assert torch.equal(xp.view(torch.int32), xp2.view(torch.int32))
    assert torch.equal(h1.view(torch.int32), h2.view(torch.int32))
    assert torch.equal(yq1, yq2)
    assert torch.equal(ys1.view(torch.int32), ys2.view(torch.int32))
    if D % 64 == 0:
        win3, h3 = dv(win0.clone()), dv(h0.clone())
        yq3, ys3 = torch.empty(B, D, dtype=torch.int8, device=cuda_dev), torch.empty(B, device=cuda_dev)
        xp3 = torch.empty(B, P, device=cuda_dev)
        k.decode_mid_packed(xz, cw, cb, win3, k.pack_ternary(w_x), w_x_scale, R, w_dt, w_dt_scale, base, h3, yq3, ys3,
                            xp_out=xp3)
        assert torch.equal(win1, win3)
        assert torch.equal(xp.view(torch.int32), xp3.view(torch.int32))
        assert torch.equal(h1.view(torch.int32), h3.view(torch.int32))
        assert torch.equal(yq1, yq3)
        assert torch.equal(ys1.view(torch.int32), ys3.view(torch.int32))
    else:
        from mamba_integer_b200._lib import MIError
        with pytest.raises(MIError):
            k.decode_mid_packed(xz, cw, cb, win2, torch.zeros(P, D // 4, dtype=torch.uint8, device=cuda_dev),
                                w_x_scale, R, w_dt, w_dt_scale, base, h2, yq2, ys2)
