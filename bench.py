"""Prefill throughput of the 24-layer d_model=768 Mamba-Integer model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --profile-workload CASE [--launches K]

One step = MambaIntegerModel.forward over the batch (config 4: 64 sequences x
2048 tokens, token ids Zipf(1.1) over the 32768 vocabulary, synthetic ternary
weights, seed 3), i.e. 24 blocks + norm_f + lm_head with full fp32 logits
written to HBM.  With N ranks each rank runs its shard of the 64 sequences
(distributed.shard_range: the global batch is fixed) and the step ends with an
NCCL all-gather of every sequence's last-position logits
(distributed.LastLogitsGather).  Rank 0 prints one JSON line.  After the timed
steps rank 0 hashes sequence 0's last-position logits and compares them with
the oracle's (tests/golden/bench_c4_seq0.json).

Secondary workloads (rank 0 at N = 1): config 2 integer scan, config 3
BitLinear beside torch._int_mm (cuBLASLt) at the same shape, config 5 decode
and the decode server.  At N > 1 the config-5 decode runs sharded: each rank
decodes its shard of the 256 streams, the step time is the max over ranks and
the generated ids are all-gathered at the end.

--impl reference times the CPU restatement of the reference path (oracle/, a
port of the reference's own CPU math, bit-identical to it) on the host cores:
rank 0 only, a bounded sample of the same workload per step.

--profile-workload runs one kernel class of a benchmark configuration a few
times on cuda:0 with the seeded inputs (for ncu captures; nothing is timed):
config2, config3, config3-packed, config3-norm-sqp, config4-in_proj, config5-step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "prefill tok/s (24L d768, 1/2/4/8 B200); scan GB/s & BitLinear i8 %peak"
UNIT = "tok/s"
WORKLOAD = "config4_prefill_24L_d768_b64x2048"
GLOBAL_BATCH = 64
SEQ_LEN = 2048


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# algorithmic work per launch of each kernel kind (T tokens)
def algorithmic_work(name: str, T: int, d=768, di=1536, R=48, N=16, V=32768):
    if name == "gemm_in_proj":
        return "tensor", 2.0 * T * 2 * di * d
    if name == "gemm_x_proj":
        return "tensor", 2.0 * T * (R + 2 * N) * di
    if name == "gemm_dt_proj":
        return "tensor", 2.0 * T * di * R
    if name == "gemm_out_proj":
        return "tensor", 2.0 * T * d * di
    if name == "gemm_lm_head":
        return "tensor", 2.0 * T * V * d
    if name == "ssm_scan":  # reads act, z, int8 dt row + scale, B|C; writes y (dt_proj fused)
        return "hbm", T * di * 4 * 3 + T * (R + 4) + T * 2 * N * 4 + di * N * 4 + di * R
    if name == "conv_act_quant":  # reads x half of xz; writes act, xq, scale
        return "hbm", T * di * 4 + T * di * 4 + T * di + T * 4
    if name == "rowprep":  # reads residual + delta; writes residual, xq, scale
        return "hbm", T * d * 4 * 3 + T * d + T * 4
    if name == "quant_y":
        return "hbm", T * di * 4 + T * di + T * 4
    if name == "quant_dt":
        return "hbm", T * R * 4 + T * R + T * 4
    return "hbm", 0.0


def measured_traffic(kernel: str, T: int):
    """DRAM bytes (read + write) per launch from the committed ncu summary
    profiles/roofline_traffic.json (captured at a smaller token count and
    scaled by tokens; the kernels' traffic is linear in tokens), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "roofline_traffic.json")) as f:
            t = json.load(f)[kernel]
        return t["dram_bytes_per_launch"] * T / t["tokens"]
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        rows = [r.split(",") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


class EventTimer:
    """Brackets kernel launches with CUDA events on the current stream."""

    def __init__(self):
        self.ev = {}

    def __call__(self, name):
        timer = self

        class _Ctx:
            def __enter__(self_inner):
                self_inner.a = torch.cuda.Event(enable_timing=True)
                self_inner.a.record()

            def __exit__(self_inner, *exc):
                b = torch.cuda.Event(enable_timing=True)
                b.record()
                timer.ev.setdefault(name, []).append((self_inner.a, b))
                return False

        return _Ctx()

    def per_kernel(self):
        torch.cuda.synchronize()
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in self.ev.items()}


def _time_launches(fn, iters: int, flush: torch.Tensor | None):
    """Average device time of fn() over iters launches (CUDA events on the
    current stream); the L2 flush between launches is outside the events."""
    tot = 0.0
    for _ in range(iters):
        if flush is not None:
            flush.add_(1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        tot += a.elapsed_time(b)
    return tot / iters


def secondary_metrics(dev, warmup: int = 3, iters: int = 5):
    """The other two BASELINE metrics on their own configs: the integer scan
    (config 2, GB/s) and the BitLinear GEMM (config 3, int8 TOP/s)."""
    from mamba_integer_b200 import _lib, kernels, synth

    hbm, bf16, src = peaks()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > L2
    out = {}
    # config 2: x [8,4096,2048], B/C [8,4096,16], n [2048,16] int32, y int32, h int32
    x, B, C, n = (t.to(dev) for t in synth.scan_i32_inputs())
    bsz, L, D = x.shape
    h = torch.zeros(bsz, D, 16, dtype=torch.int32, device=dev)
    y = torch.empty(bsz, L, D, dtype=torch.int32, device=dev)
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream

    def run_scan():
        h.zero_()
        _lib.check(lib.mi_scan_i32(x.data_ptr(), B.data_ptr(), C.data_ptr(), n.data_ptr(), 15, y.data_ptr(), None,
                                   h.data_ptr(), bsz, L, D, 16, st), "mi_scan_i32")

    for _ in range(warmup):
        run_scan()
    ms = _time_launches(run_scan, iters, None)  # inputs (268 MB) larger than L2
    err = _lib.device_error(st)
    nbytes = 542244864
    out["scan_i32"] = {"config": "config2: batch 8, L 4096, d_inner 2048, d_state 16, int32 y and h",
                       "ms": ms, "GB_per_s": nbytes / ms / 1e6, "hbm_frac": nbytes / ms / 1e6 / hbm,
                       "G_state_updates_per_s": bsz * L * D * 16 / ms / 1e6, "device_error_word": err,
                       "bytes_per_call": nbytes, "peak_source": src}
    del x, B, C, n, h, y
    # config 3: A int8 [16384, 2048] x W ternary int8 [8192, 2048] -> int32 C
    A, a_scale, Wq, ws = synth.bitlinear_inputs()
    A, Wq = A.to(dev), Wq.to(dev)
    Cm = torch.empty(A.shape[0], Wq.shape[0], dtype=torch.int32, device=dev)

    def run_gemm():
        kernels.bitlinear_i8(A, Wq, out=Cm)

    for _ in range(warmup):
        run_gemm()
    ms = _time_launches(run_gemm, iters, flush)  # A and W fit in L2: flush between launches
    ops = 2.0 * A.shape[0] * Wq.shape[0] * A.shape[1]
    tops = ops / ms / 1e9
    # the library bar for the same contraction: torch._int_mm (cuBLASLt int8 GEMM, int32 out), the
    # reference's own fast path for BitLinear (src/triton_kernels/bitnet_kernels.py:198-218)
    Bt = Wq.t()  # [K, N] column-major view of the [N, K] weights

    def run_int_mm():
        torch._int_mm(A, Bt, out=Cm)

    for _ in range(warmup):
        run_int_mm()
    ms_lib = _time_launches(run_int_mm, iters, flush)
    tops_lib = ops / ms_lib / 1e9
    int8_peak = max(2.0 * bf16, tops_lib)
    peak_note = ("max(2 x measured dense bf16, measured torch._int_mm at this shape)"
                 f" = {'torch._int_mm' if tops_lib > 2.0 * bf16 else '2 x bf16'}")
    out["int8_library_bar"] = {"config": "config3: M 16384, K 2048, N 8192, int32 out", "impl": "torch._int_mm (cuBLASLt)",
                               "ms": ms_lib, "TOP_per_s": tops_lib}
    out["bitlinear_i8"] = {"config": "config3: M 16384, K 2048, N 8192, int32 out, int8 weights", "ms": ms,
                           "TOP_per_s": tops, "int8_peak_frac": tops / int8_peak, "int8_peak": int8_peak,
                           "peak_note": peak_note, "vs_int_mm": ms_lib / ms,
                           "output_GB_per_s": Cm.numel() * 4 / ms / 1e6}
    # the same contraction with the weights packed 2 bits each (config 3 as specified)
    Wp = kernels.pack_ternary(Wq)

    def run_gemm_packed():
        kernels.bitlinear_packed(A, Wp, out=Cm)

    for _ in range(warmup):
        run_gemm_packed()
    ms = _time_launches(run_gemm_packed, iters, flush)
    tops = ops / ms / 1e9
    out["bitlinear_packed"] = {"config": "config3: M 16384, K 2048, N 8192, int32 out, 2-bit packed weights",
                               "ms": ms, "TOP_per_s": tops, "int8_peak_frac": tops / int8_peak,
                               "int8_peak": int8_peak, "vs_int_mm": ms_lib / ms,
                               "output_GB_per_s": Cm.numel() * 4 / ms / 1e6,
                               "device_error_word": _lib.device_error(st)}
    # config 3 as specified: int32 accumulate, then the fused BitShift-norm/squareplus epilogue
    # (exact row sums in the GEMM epilogue, one streaming pass over the rows)
    gamma, step = (t.to(dev) for t in synth.bitlinear_norm_params(Wq.shape[0]))
    a_sc = a_scale.to(dev)
    w_sc = torch.tensor([ws], dtype=torch.float32, device=dev)
    out_f = torch.empty(A.shape[0], Wq.shape[0], dtype=torch.float32, device=dev)
    stats = torch.empty(A.shape[0], 2, dtype=torch.int64, device=dev)

    def run_norm_sqp():
        kernels.bitlinear_packed_norm_sqp(A, Wp, a_sc, w_sc, gamma, step, acc=Cm, out=out_f, stats_ws=stats)

    for _ in range(warmup):
        run_norm_sqp()
    ms_e = _time_launches(run_norm_sqp, iters, flush)
    out["bitlinear_packed_norm_sqp"] = {
        "config": "config3: M 16384, K 2048, N 8192, packed weights, int32 out + BitShift norm + squareplus fp32 out",
        "ms": ms_e, "TOP_per_s": ops / ms_e / 1e9, "int8_peak_frac": ops / ms_e / 1e9 / int8_peak,
        "epilogue_ms_over_int32_gemm": ms_e - ms,
        "note": "GEMM epilogue adds exact int64 row sums; a second pass reads int32 acc and writes fp32 out",
        "device_error_word": _lib.device_error(st)}
    return out


def decode_metrics(dev, steps: int = 64, warmup: int = 3, world: int = 1, rank: int = 0):
    """Config 5: greedy decoding of 256 streams after a 512-token Zipf prompt
    (24 layers, d_model 1024).  The prompt runs through the prefill kernels
    (untimed); then `steps` decode steps, each replayed from one CUDA graph,
    are timed with CUDA events.  The state a step reads and writes does not
    depend on the position, so tok/s over these steps holds for all 512.

    Under torchrun the streams are sharded (distributed.shard_range): each rank
    decodes its shard with no collective, the timed region is bracketed by
    barriers and its time is the max over ranks, and the generated ids are
    all-gathered (distributed.gather_ids) after it."""
    import torch.distributed as dist

    from mamba_integer_b200 import distributed as mdist
    from mamba_integer_b200 import kernels, synth
    from mamba_integer_b200.decode import DecodeEngine
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel

    hbm, _, src = peaks()
    c = synth.CONFIGS["c5"]
    cfg = synth.model_config("c5")
    B_all = c["batch"]
    lo, hi = mdist.shard_range(B_all, world, rank)
    B = hi - lo
    model = MambaIntegerModel(cfg)
    model.load_state_dict(synth.model_state_dict(cfg, c["seed"]))
    model = model.to(dev).eval()
    prompt = synth.input_ids("c5", B_all, c["seq_len"])[lo:hi].to(dev)
    eng = DecodeEngine(model)
    logits = eng.start(prompt)
    kernels.argmax_rows(logits, out=eng.ws.next_ids)
    gen = torch.empty(B, steps, dtype=torch.int64, device=dev)
    for _ in range(warmup):
        eng.step(eng.ws.next_ids)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        eng.step(eng.ws.next_ids)
        gen[:, i].copy_(eng.ws.next_ids)
    b.record()
    barrier()
    ms_t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        all_ids = mdist.gather_ids(gen, B_all)
    else:
        all_ids = gen
    ms = float(ms_t.item()) / steps
    d, di, L, V, N = cfg["d_model"], 2 * cfg["d_model"], cfg["n_layer"], cfg["vocab_size"], 16
    R = cfg["ssm_cfg"]["dt_rank"]
    # algorithmic HBM bytes of one step on one rank: scan states and conv windows read and
    # written, packed weights and the step's logits
    state = 2 * L * B * di * N * 4 + 2 * L * B * 3 * di * 4
    weights = L * (2 * di * d + (R + 2 * N) * di + d * di) // 4 + L * di * 64 + V * d // 4
    nbytes = state + weights + B * V * 4
    return {"config": f"config5: 24L d1024, {B_all} streams ({B} per rank), 512-token prompt, greedy steps",
            "n_gpus": world, "steps_timed": steps, "ms_per_step": ms, "tok_per_s": B_all / ms * 1e3,
            "hbm_bytes_per_step_per_rank": nbytes, "achieved_GB_per_s_per_rank": nbytes / ms / 1e6,
            "hbm_frac": nbytes / ms / 1e6 / hbm, "peak_source": src,
            "launches_per_step": eng.launches_per_step(), "cuda_graph": True,
            "generated_ids_gathered": list(all_ids.shape)}


def server_metrics(dev, n_requests: int = 384, slots: int = 256, max_new: int = 32, seed: int = 5):
    """Config-5 model behind the continuous-batching server: n_requests Zipf
    prompts of lengths drawn from {32, 64, 128, 256}, max_new tokens each,
    `slots` streams resident.  Wall time of the whole run (prefills,
    graph-replayed steps, the per-step host loop) between two device syncs."""
    import time
    from mamba_integer_b200 import synth
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    from mamba_integer_b200.serve import DecodeServer

    c = synth.CONFIGS["c5"]
    cfg = synth.model_config("c5")
    model = MambaIntegerModel(cfg)
    model.load_state_dict(synth.model_state_dict(cfg, c["seed"]))
    model = model.to(dev).eval()
    g = torch.Generator().manual_seed(seed)
    lens = [32, 64, 128, 256]
    prompts = [synth.zipf_ids(1, lens[int(torch.randint(0, 4, (1,), generator=g))], cfg["vocab_size"], g)[0].tolist()
               for _ in range(n_requests)]
    # warm-up: the same request stream served once, untimed (captures the step graph and
    # meets every admission group's prefill shape, so the allocator holds its buffers);
    # the timed run then serves it again with a fresh server on the same engine
    warm = DecodeServer(model, slots=slots)
    for pr in prompts:
        warm.submit(pr, max_new)
    warm.run()
    srv = DecodeServer(model, slots=slots, engine=warm.eng)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for pr in prompts:
        srv.submit(pr, max_new)
    out = srv.run()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    gen = sum(len(v) for v in out.values())
    return {"config": f"config5 model, {n_requests} requests (prompts 32-256 tokens, {max_new} new each), "
                      f"{slots} slots, greedy", "generated_tokens": gen, "wall_s": wall, "tok_per_s": gen / wall,
            "decode_steps": srv.steps, "prompt_tokens": sum(len(p) for p in prompts)}


def cpu_baseline(n_tokens: int = 256, threads: int = 0):
    """The CPU restatement of the reference path (full 24 layers + lm_head) on
    one sequence of n_tokens of the config-4 workload."""
    from mamba_integer_b200 import synth
    from oracle import model as om

    cfg = synth.model_config("c4")
    sd = synth.model_state_dict(cfg, synth.CONFIGS["c4"]["seed"])
    p = om.prepare(sd)
    ids = synth.input_ids("c4", GLOBAL_BATCH, SEQ_LEN)[:1, :n_tokens].numpy()
    om.forward(p, cfg, ids[:, :16], nthreads=threads)  # warm-up (page in the weights)
    t0 = time.perf_counter()
    om.forward(p, cfg, ids, nthreads=threads)
    dt = time.perf_counter() - t0
    return n_tokens / dt, dt, p, cfg


def run_reference(args, rank: int):
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    n_tokens = int(os.environ.get("MI_REF_SAMPLE_TOKENS", "128"))
    from mamba_integer_b200 import synth
    from oracle import model as om

    cfg = synth.model_config("c4")
    sd = synth.model_state_dict(cfg, synth.CONFIGS["c4"]["seed"])
    p = om.prepare(sd)
    ids = synth.input_ids("c4", GLOBAL_BATCH, SEQ_LEN)[:1, :n_tokens].numpy()
    for _ in range(args.warmup):
        om.forward(p, cfg, ids, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        om.forward(p, cfg, ids, nthreads=cores)
    dt = time.perf_counter() - t0
    v = args.steps * n_tokens / dt
    sample = f"1 sequence x {n_tokens} tokens of config 4 per step (24 layers + lm_head), all {cores} host threads"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32+int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH, "seq_len": SEQ_LEN, "sample": sample},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# fp32 operations of the fused scan per token (d_inner channels): per (channel, state) the
# decay sum, its clamp, 1 - decay, x*dt*B, h*decay, (1 - decay)*u, their sum and one FMA of
# h.C (8); per channel the dt_proj rescale (2), ste_clamp (4), squareplus with its 3 Newton
# steps and clamps (31), dt scale + clamp (5), x*dt (1) and the gate (6): 49
SCAN_FP32_OPS_PER_CHANNEL = 16 * 8 + 49


def scan_alu_roofline(T: int, avg_ms: float, sm_mhz, di: int = 1536):
    """The fused scan's fp32 issue roofline: its fp32 operations per launch over
    the time, against 148 SMs x 128 fp32 lanes x the median SM clock measured
    during the timed steps."""
    if not sm_mhz:
        return None
    ops = float(T) * di * SCAN_FP32_OPS_PER_CHANNEL
    achieved = ops / (avg_ms / 1000.0) / 1e12
    peak = 148 * 128 * float(sm_mhz) * 1e6 / 1e12
    return {"unit": "T fp32 op/s", "achieved": achieved, "peak": peak, "frac": achieved / peak,
            "ops_per_launch": ops, "peak_basis": f"148 SMs x 128 fp32 lanes x {sm_mhz:.0f} MHz (median under load)",
            "ops_basis": f"{SCAN_FP32_OPS_PER_CHANNEL} fp32 operations per (token, channel)"}


def parity_check(logits_seq0_last: torch.Tensor):
    """sha256 of sequence 0's last-position logits against the oracle's
    (tests/golden/bench_c4_seq0.json, made by tests/golden/make_bench_hash.py)."""
    import hashlib

    path = os.path.join(ROOT, "tests", "golden", "bench_c4_seq0.json")
    with open(path) as f:
        ref = json.load(f)
    got = hashlib.sha256(logits_seq0_last.detach().cpu().contiguous().numpy().tobytes()).hexdigest()
    return {"checked": "sha256 of sequence 0's last-position logits (fp32) after the timed steps",
            "oracle_sha256": ref["last_logits_sha256"], "sha256": got, "match": got == ref["last_logits_sha256"]}


# ---- single-kernel workloads for profiler captures (nothing timed) -------------------------
def _pw_config2(dev, launches: int) -> None:
    from mamba_integer_b200 import _lib, synth

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


def _pw_config3(dev, launches: int, packed: bool) -> None:
    from mamba_integer_b200 import kernels, synth

    A, _, Wq, _ = synth.bitlinear_inputs()
    A, Wq = A.to(dev), Wq.to(dev)
    C = torch.empty(A.shape[0], Wq.shape[0], dtype=torch.int32, device=dev)
    Wp = kernels.pack_ternary(Wq) if packed else None
    for _ in range(launches):
        if packed:
            kernels.bitlinear_packed(A, Wp, out=C)
        else:
            kernels.bitlinear_i8(A, Wq, out=C)


def _pw_config3_norm_sqp(dev, launches: int) -> None:
    from mamba_integer_b200 import kernels, synth

    A, a_scale, Wq, ws = synth.bitlinear_inputs()
    gamma, step = (t.to(dev) for t in synth.bitlinear_norm_params(Wq.shape[0]))
    A, Wq, a_scale = A.to(dev), Wq.to(dev), a_scale.to(dev)
    Wp = kernels.pack_ternary(Wq)
    w_sc = torch.tensor([ws], dtype=torch.float32, device=dev)
    for _ in range(launches):
        kernels.bitlinear_packed_norm_sqp(A, Wp, a_scale, w_sc, gamma, step)


def _pw_config4_in_proj(dev, launches: int) -> None:
    """One layer's in_proj of the config-4 prefill at full size: int8 A
    [131072, 768] x packed ternary W [3072, 768] -> fp32 [131072, 3072] with
    the BitLinear rescale."""
    from mamba_integer_b200 import kernels, synth

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


def _pw_config5_step(dev, launches: int) -> None:
    """Decode steps of 256 streams after a short prompt (the per-step work does
    not depend on the prompt length), launched eagerly, without a CUDA graph."""
    from mamba_integer_b200 import kernels, synth
    from mamba_integer_b200.decode import DecodeEngine
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel

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


PROFILE_WORKLOADS = {
    "config2": lambda dev, k: _pw_config2(dev, k),
    "config3": lambda dev, k: _pw_config3(dev, k, packed=False),
    "config3-packed": lambda dev, k: _pw_config3(dev, k, packed=True),
    "config3-norm-sqp": lambda dev, k: _pw_config3_norm_sqp(dev, k),
    "config4-in_proj": lambda dev, k: _pw_config4_in_proj(dev, k),
    "config5-step": lambda dev, k: _pw_config5_step(dev, k),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config-2 scan / config-3 GEMM / config-5 decode lines")
    # smaller shapes for profiling captures only (the reported workload is 64 x 2048)
    ap.add_argument("--batch", type=int, default=GLOBAL_BATCH)
    ap.add_argument("--seq", type=int, default=SEQ_LEN)
    ap.add_argument("--scan-split", type=int, default=0, choices=[0, 1, 2, 3, 4, 8],
                    help="fused-scan variant: 1/2/4/8 lanes per channel, 3 = pipelined (0 = automatic)")
    ap.add_argument("--profile-workload", choices=sorted(PROFILE_WORKLOADS),
                    help="run one kernel class of a benchmark configuration for a profiler capture and exit")
    ap.add_argument("--launches", type=int, default=2, help="launches of --profile-workload")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.profile_workload:
        from mamba_integer_b200 import _lib

        PROFILE_WORKLOADS[args.profile_workload](dev, args.launches)
        torch.cuda.synchronize()
        print(f"{args.profile_workload}: {args.launches} launches, device error word {_lib.device_error()}")
        return

    import torch.distributed as dist

    from mamba_integer_b200 import _lib, synth
    from mamba_integer_b200 import distributed as mdist
    from mamba_integer_b200.engine import launches_per_forward
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel

    if world > 1:
        mdist.init_from_env("nccl", timeout_s=120)

    _lib.load()
    cfg = synth.model_config("c4")
    sd = synth.model_state_dict(cfg, synth.CONFIGS["c4"]["seed"])
    model = MambaIntegerModel(cfg)
    model.load_state_dict(sd)
    model = model.to(dev).eval()
    eng = model.engine()
    eng.scan_split = args.scan_split
    gb, sl = args.batch, args.seq
    ids_all = synth.input_ids("c4", gb, sl)
    lo, hi = mdist.shard_range(gb, world, rank)
    ids_host = ids_all[lo:hi].contiguous().pin_memory()
    ids_dev = ids_host.to(dev)
    b_local = hi - lo
    T_local = b_local * sl
    V = cfg["vocab_size"]
    logits = torch.empty(b_local, sl, V, dtype=torch.float32, device=dev)
    gather = mdist.LastLogitsGather(gb, V, device=dev) if world > 1 else None

    def step(ids):
        eng.forward(ids, logits=logits)
        if gather is not None:
            gather(logits[:, -1, :])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with torch.no_grad():
        for _ in range(args.warmup):
            step(ids_dev)
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            barrier()
            s0.record()
            for _ in range(args.steps):
                step(ids_dev)
            s1.record()
            barrier()
        ms = s0.elapsed_time(s1)
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        value = gb * sl * args.steps / (ms / 1000.0)
        parity = None
        if rank == 0 and (gb, sl) == (GLOBAL_BATCH, SEQ_LEN):
            parity = parity_check(logits[0, -1, :])

        # end to end through the public API: pinned host ids -> device, forward,
        # last-position logits -> pinned host
        last_host = torch.empty(b_local, V, dtype=torch.float32).pin_memory()
        e2e_steps = args.steps
        # one untimed pass so the logits allocation of the API call is cached
        out = model(ids_host.to(dev, non_blocking=True))
        last_host.copy_(out[:, -1, :], non_blocking=True)
        del out
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            ids_d = ids_host.to(dev, non_blocking=True)
            out = model(ids_d)
            last_host.copy_(out[:, -1, :], non_blocking=True)
            del out
        e1.record()
        barrier()
        ems = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e_val = gb * sl * e2e_steps / (float(ems.item()) / 1000.0)

        # per-kernel CUDA-event timing of one more forward (outside the timed region), and at
        # N > 1 the gather alone, so that a step splits into kernels, gather and the rest
        tim = EventTimer()
        eng.forward(ids_dev, logits=logits, timer=tim)
        per_k = tim.per_kernel()
        step_split = None
        if gather is not None:
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            for _ in range(5):
                gather(logits[:, -1, :])
            g1.record()
            barrier()
            gather_ms = g0.elapsed_time(g1) / 5
            fwd = sum(sum(v) for v in per_k.values())
            step_split = {"step_ms": ms / args.steps, "kernels_ms": fwd, "gather_ms": gather_ms,
                          "rest_ms": ms / args.steps - fwd - gather_ms,
                          "note": "rank 0's kernels and gather, CUDA events; rest = launch gaps and barrier skew"}
        secondary = None
        if not args.no_secondary:
            del logits
            torch.cuda.empty_cache()
            if world == 1:
                secondary = secondary_metrics(dev)
                secondary["decode"] = decode_metrics(dev)
                secondary["server"] = server_metrics(dev)
            else:
                secondary = {"decode": decode_metrics(dev, world=world, rank=rank)}

    hbm, bf16, src = peaks()
    totals = {k: sum(v) for k, v in per_k.items()}
    dom = max(totals, key=totals.get)
    bound, work = algorithmic_work(dom, T_local)
    avg_ms = totals[dom] / len(per_k[dom])
    if bound == "tensor":
        achieved = work / (avg_ms / 1000.0) / 1e12
        peak = 2.0 * bf16  # dense int8 peak taken as 2x the measured dense bf16 (nominal ratio 4.5/2.25)
        unit = "TOP/s"
    else:
        achieved = work / (avg_ms / 1000.0) / 1e9
        peak = hbm
        unit = "GB/s"
    clocks = clk.summary()
    roof = {"kernel": dom, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak, "traffic": measured_traffic(dom, T_local), "peak_source": src,
            "avg_launch_ms": avg_ms}
    if dom == "ssm_scan":
        # the scan is bound by its exact fp32 work, not by HBM: achieved/peak/frac above are its
        # HBM bytes (the unit this line reports for memory kernels), the alu block its issue roofline
        roof["bound"] = "alu"
        roof["frac_basis"] = "algorithmic HBM bytes per launch / measured copy bandwidth"
        roof["alu"] = scan_alu_roofline(T_local, avg_ms, clocks.get("sm_mhz"))
    fwd_ms = sum(totals.values())
    breakdown = {k: {"ms": round(v, 3), "share": round(v / fwd_ms, 4), "launches": len(per_k[k])}
                 for k, v in sorted(totals.items(), key=lambda kv: -kv[1])}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        n_tok = int(os.environ.get("MI_CPU_SAMPLE_TOKENS", "2048"))
        v_cpu, dt_cpu, _, _ = cpu_baseline(n_tok, cores)
        cpu = {"value": v_cpu, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"1 sequence x {n_tok} tokens of config 4 (24 layers + lm_head), oracle C port, "
                         f"{dt_cpu:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32+int8", "data": "synthetic",
            "config": {"workload": WORKLOAD if (gb, sl) == (GLOBAL_BATCH, SEQ_LEN) else f"profiling_b{gb}x{sl}",
                       "global_batch": gb, "seq_len": sl,
                       "parallelism": f"batch split {world} (distributed.shard_range)" if world > 1 else "single GPU",
                       "l2": "working set (>= 1.6 GB per activation buffer) far larger than L2; no flush needed"},
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(ids_host.numel() * 8),
                    "d2h_bytes_per_step": int(b_local * V * 4)},
            "gpu_launches": launches_per_forward(cfg["n_layer"]) * args.steps,
            "roofline": roof,
            "kernel_breakdown": breakdown,
            "step_split": step_split,
            "parity": parity,
            "clocks": clocks,
            "cpu_baseline": cpu,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
