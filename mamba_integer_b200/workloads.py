"""Single-kernel workloads of the benchmark configurations, for profiling.

    python -m mamba_integer_b200.workloads config2            # integer scan, config 2
    python -m mamba_integer_b200.workloads config3            # BitLinear, int8 weights
    python -m mamba_integer_b200.workloads config3-packed     # BitLinear, 2-bit packed weights
    python -m mamba_integer_b200.workloads config4-in_proj    # one in_proj of the config-4 prefill
    python -m mamba_integer_b200.workloads config5-step       # one decode step, config 5 shapes

Each runs its kernel(s) ``--launches`` times (default 2: a warm-up launch, then
the one a profiler would capture) on cuda:0 with the seeded synthetic inputs
of ``synth`` and prints the device error word.  Nothing is timed here;
bench.py does the timing.
"""
from __future__ import annotations

import argparse

import torch

from . import _lib, kernels, synth


def _config2(dev, launches: int) -> None:
    x, B, C, n = (t.to(dev) for t in synth.scan_i32_inputs())
    bsz, L, D = x.shape
    h = torch.zeros(bsz, D, 16, dtype=torch.int32, device=dev)
    y = torch.empty(bsz, L, D, dtype=torch.int32, device=dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(launches):
        h.zero_()
        _lib.check(lib.mi_scan_i32(x.data_ptr(), B.data_ptr(), C.data_ptr(), n.data_ptr(), 15, y.data_ptr(), None,
                                   h.data_ptr(), bsz, L, D, 16, stream), "mi_scan_i32")


def _config3(dev, launches: int, packed: bool) -> None:
    A, _, Wq, _ = synth.bitlinear_inputs()
    A, Wq = A.to(dev), Wq.to(dev)
    C = torch.empty(A.shape[0], Wq.shape[0], dtype=torch.int32, device=dev)
    Wp = kernels.pack_ternary(Wq) if packed else None
    for _ in range(launches):
        if packed:
            kernels.bitlinear_packed(A, Wp, out=C)
        else:
            kernels.bitlinear_i8(A, Wq, out=C)


def _config4_in_proj(dev, launches: int) -> None:
    """One layer's in_proj of the config-4 prefill at full size: int8 A
    [131072, 768] x packed ternary W [3072, 768] -> fp32 [131072, 3072] with
    the BitLinear rescale (the model's A-resident GEMM)."""
    g = torch.Generator().manual_seed(3)
    M, N, K = 64 * 2048, 3072, 768
    A = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8).to(dev)
    W = synth.ternary_weight(N, K, g)
    Wp = kernels.pack_ternary((W * 32).to(torch.int8).to(dev))
    xs = (torch.rand(M, generator=g) * 0.05 + 1e-3).to(dev)
    ws = torch.tensor([2.0 ** -6], device=dev)
    out = torch.empty(M, N, device=dev)
    for _ in range(launches):
        kernels.bitlinear_packed(A, Wp, xs, ws, out=out)


def _config5_step(dev, launches: int) -> None:
    """Decode steps of 256 streams after a short prompt (the per-step work does
    not depend on the prompt length), launched eagerly, without a CUDA graph."""
    from .decode import DecodeEngine
    from .mamba_integer_model import MambaIntegerModel
    c = synth.CONFIGS["c5"]
    cfg = synth.model_config("c5")
    model = MambaIntegerModel(cfg)
    model.load_state_dict(synth.model_state_dict(cfg, c["seed"]))
    model = model.to(dev).eval()
    eng = DecodeEngine(model, use_graph=False)
    logits = eng.start(synth.input_ids("c5", c["batch"], 8).to(dev))
    kernels.argmax_rows(logits, out=eng.ws.next_ids)
    for _ in range(launches):
        eng.step(eng.ws.next_ids)


CASES = {
    "config2": lambda dev, k: _config2(dev, k),
    "config3": lambda dev, k: _config3(dev, k, packed=False),
    "config3-packed": lambda dev, k: _config3(dev, k, packed=True),
    "config4-in_proj": lambda dev, k: _config4_in_proj(dev, k),
    "config5-step": lambda dev, k: _config5_step(dev, k),
}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=2)
    args = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    CASES[args.case](dev, args.launches)
    torch.cuda.synchronize()
    print(f"{args.case}: {args.launches} launches, device error word {_lib.device_error()}")


if __name__ == "__main__":
    main()
