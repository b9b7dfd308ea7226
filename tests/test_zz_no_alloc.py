"""The allocation-free conv/activation/quantisation entry point.

mi_conv_act_quant_noalloc exists for hosts that cannot call cudaMalloc to
provide the row-absmax workspace mi_conv_act_quant takes; it keeps that
scratch in a fixed device array inside the library.  This file is collected
last on purpose, so a run that stops at the first failure has already run
every other test.  The check: two calls in a row (the second on smaller
inputs, so stale scratch from the first call would show) must give the same
bits as the workspace entry point, through the C ABI.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(seed, scale, bsz, L, D, dev):
    g = torch.Generator().manual_seed(seed)
    xz = (torch.randn(bsz * L, 2 * D, generator=g) * scale).to(dev)
    w = (torch.rand(D, 4, generator=g) - 0.5).to(dev).contiguous()
    b = (torch.rand(D, generator=g) - 0.5).to(dev)
    return xz, w, b


def _outputs(T, D, dev):
    return (torch.empty(T, D, device=dev), torch.empty(T, D, dtype=torch.int8, device=dev),
            torch.empty(T, device=dev))


def test_noalloc_matches_workspace_entry_point_twice(cuda_dev):
    from mamba_integer_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    bsz, L, D = 3, 129, 512
    T = bsz * L
    for call, scale in enumerate((40.0, 0.5)):
        xz, w, b = _inputs(100 + call, scale, bsz, L, D, cuda_dev)
        act_r, xq_r, xs_r = _outputs(T, D, cuda_dev)
        ws = torch.empty(T, device=cuda_dev)
        _lib.check(lib.mi_conv_act_quant(xz.data_ptr(), xz.stride(0), w.data_ptr(), b.data_ptr(), act_r.data_ptr(),
                                         xq_r.data_ptr(), xs_r.data_ptr(), ws.data_ptr(), bsz, L, D, stream),
                   "mi_conv_act_quant")
        act, xq, xs = _outputs(T, D, cuda_dev)
        _lib.check(lib.mi_conv_act_quant_noalloc(xz.data_ptr(), xz.stride(0), w.data_ptr(), b.data_ptr(),
                                                 act.data_ptr(), xq.data_ptr(), xs.data_ptr(), bsz, L, D, stream),
                   "mi_conv_act_quant_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(act.view(torch.int32), act_r.view(torch.int32)), f"call {call}: activations differ"
        assert torch.equal(xq, xq_r), f"call {call}: int8 activations differ"
        assert torch.equal(xs.view(torch.int32), xs_r.view(torch.int32)), f"call {call}: scales differ"


def test_noalloc_accepts_exactly_its_row_limit(cuda_dev):
    # batch * L == 262144, the size of the fixed scratch: accepted, same bits as the workspace entry point
    from mamba_integer_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    bsz, L, D = 2, 1 << 17, 4
    T = bsz * L
    xz, w, b = _inputs(7, 3.0, bsz, L, D, cuda_dev)
    act_r, xq_r, xs_r = _outputs(T, D, cuda_dev)
    ws = torch.empty(T, device=cuda_dev)
    _lib.check(lib.mi_conv_act_quant(xz.data_ptr(), xz.stride(0), w.data_ptr(), b.data_ptr(), act_r.data_ptr(),
                                     xq_r.data_ptr(), xs_r.data_ptr(), ws.data_ptr(), bsz, L, D, stream),
               "mi_conv_act_quant")
    act, xq, xs = _outputs(T, D, cuda_dev)
    _lib.check(lib.mi_conv_act_quant_noalloc(xz.data_ptr(), xz.stride(0), w.data_ptr(), b.data_ptr(), act.data_ptr(),
                                             xq.data_ptr(), xs.data_ptr(), bsz, L, D, stream),
               "mi_conv_act_quant_noalloc")
    torch.cuda.synchronize()
    assert torch.equal(act.view(torch.int32), act_r.view(torch.int32))
    assert torch.equal(xq, xq_r)
    assert torch.equal(xs.view(torch.int32), xs_r.view(torch.int32))


def test_noalloc_rejects_more_rows_than_its_scratch(cuda_dev):
    from mamba_integer_b200 import _lib

    lib = _lib.load()
    dummy = torch.zeros(16, device=cuda_dev)
    p = dummy.data_ptr()
    rc = lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, p, p, 1 << 10, 1 << 10, 8, ctypes.c_void_p(0))
    assert rc == -2  # MI_ERR_UNSUPPORTED: batch * L above the fixed maximum, nothing launched
    rc = lib.mi_conv_act_quant_noalloc(p, 8, p, p, p, p, p, 1, (1 << 18) + 1, 4, ctypes.c_void_p(0))
    assert rc == -2  # one row above the limit
