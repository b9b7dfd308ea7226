"""Parity at the sizes bench.py times, bit for bit against the CPU oracle.

The kernels choose variants by shape (the fused scan by sequence length, the
GEMMs their tile widths and scheduler order by M and N), so these run the
GPU at the benchmarked shapes themselves and compare what the oracle can
afford at those shapes:

* config 4 (24 layers, d_model 768, vocab 32768) at the full 64 x 2048 batch
  and at the per-GPU batches of 2, 4 and 8 GPUs (32, 16, 8 sequences):
  sequence 0's full [2048, 32768] logits against the oracle's hash
  (tests/golden/bench_c4_seq0.json) and, at 64, the last sequence's full
  logits against a live oracle run;
* config 2 (integer scan, 8 x 4096 x 2048 x 16) in full: every y and final h;
* config 3 (BitLinear, M 16384, K 2048, N 8192, int8 and 2-bit packed
  weights): every row of 512 seeded columns, plus every 128-row tile's first
  row across all 8192 columns (the persistent scheduler's late tiles);
* config 5 (24 layers, d_model 1024) with all 256 streams and their
  512-token prompts on the GPU, then 8 greedy steps from the CUDA graph:
  four streams' logits at every step against the oracle's full forward over
  prompt + generated tokens, and their greedy ids.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _nthreads() -> int:
    return os.cpu_count() or 1


@pytest.fixture(scope="module")
def c4_model(cuda_dev):
    from mamba_integer_b200 import synth
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    cfg = synth.model_config("c4")
    sd = synth.model_state_dict(cfg, synth.CONFIGS["c4"]["seed"])
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    return cfg, sd, m.to(cuda_dev).eval()


def _oracle_seq(cfg, sd, ids_row):
    from oracle import model as om
    return om.forward(om.prepare(sd), cfg, ids_row[None, :], nthreads=_nthreads())[0]


def test_config4_full_depth_logits_bit_exact(cuda_dev, c4_model):
    from mamba_integer_b200 import synth
    cfg, sd, m = c4_model
    with open(os.path.join(GOLD, "bench_c4_seq0.json")) as f:
        fx = json.load(f)
    ids = synth.input_ids("c4", 64, 2048)
    assert _sha(ids[0].numpy()) == fx["ids_sha256"]
    eng = m.engine()
    logits = torch.empty(64, 2048, cfg["vocab_size"], dtype=torch.float32, device=cuda_dev)
    with torch.no_grad():
        eng.forward(ids.to(cuda_dev), logits=logits)
    seq0 = logits[0].cpu().numpy()
    last = logits[63].cpu().numpy()
    del logits
    torch.cuda.empty_cache()
    if _sha(seq0) != fx["logits_sha256"]:
        ref = _oracle_seq(cfg, sd, ids[0].numpy())
        ne = seq0.view(np.uint32) != ref.view(np.uint32)
        raise AssertionError(f"sequence 0: {int(ne.sum())} of {ne.size} logits differ from the oracle")
    assert _sha(seq0[-1]) == fx["last_logits_sha256"]
    ref63 = _oracle_seq(cfg, sd, ids[63].numpy())
    ne = last.view(np.uint32) != ref63.view(np.uint32)
    assert not ne.any(), f"sequence 63: {int(ne.sum())} of {ne.size} logits differ from the oracle"


@pytest.mark.parametrize("batch", [32, 16, 8])
def test_config4_per_gpu_batches_bit_exact(cuda_dev, c4_model, batch):
    # the batch one GPU holds when the 64 sequences are split over 2, 4 and 8 GPUs
    from mamba_integer_b200 import synth
    cfg, _, m = c4_model
    with open(os.path.join(GOLD, "bench_c4_seq0.json")) as f:
        fx = json.load(f)
    ids = synth.input_ids("c4", 64, 2048)[:batch]
    logits = torch.empty(batch, 2048, cfg["vocab_size"], dtype=torch.float32, device=cuda_dev)
    with torch.no_grad():
        m.engine().forward(ids.to(cuda_dev), logits=logits)
    assert _sha(logits[0].cpu().numpy()) == fx["logits_sha256"], f"batch {batch}: sequence 0 differs from the oracle"


def test_config2_full_size_bit_exact(cuda_dev):
    from mamba_integer_b200 import _lib, synth
    from oracle import lib as orc
    x, B, C, n = synth.scan_i32_inputs()  # 8 x 4096 x 2048, N 16
    bsz, L, D = x.shape
    y_ref, h_ref = orc.scan_i32(x.numpy(), B.numpy(), C.numpy(), n.numpy(), 15, nthreads=_nthreads())
    assert np.abs(y_ref).max() < 2 ** 31
    xd, Bd, Cd, nd = (t.to(cuda_dev) for t in (x, B, C, n))
    h = torch.zeros(bsz, D, 16, dtype=torch.int32, device=cuda_dev)
    y = torch.empty(bsz, L, D, dtype=torch.int32, device=cuda_dev)  # the int32 output bench.py times
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.mi_scan_i32(xd.data_ptr(), Bd.data_ptr(), Cd.data_ptr(), nd.data_ptr(), 15, y.data_ptr(), None,
                               h.data_ptr(), bsz, L, D, 16, st), "mi_scan_i32")
    assert _lib.device_error(st) == 0
    assert np.array_equal(y.cpu().numpy(), y_ref.astype(np.int32))
    assert np.array_equal(h.cpu().numpy(), h_ref)


@pytest.mark.parametrize("packed", [False, True])
def test_config3_full_size_bit_exact(cuda_dev, packed):
    from mamba_integer_b200 import _lib, kernels, synth
    from oracle import lib as orc
    A, _, Wq, _ = synth.bitlinear_inputs()  # M 16384, K 2048, N 8192
    M, K = A.shape
    N = Wq.shape[0]
    Ad, Wd = A.to(cuda_dev), Wq.to(cuda_dev)
    out = torch.empty(M, N, dtype=torch.int32, device=cuda_dev)
    if packed:
        kernels.bitlinear_packed(Ad, kernels.pack_ternary(Wd), out=out)
    else:
        kernels.bitlinear_i8(Ad, Wd, out=out)
    assert _lib.device_error() == 0
    An, Wn = A.numpy(), Wq.numpy()
    cols = np.sort(np.random.default_rng(5).choice(N, 512, replace=False))
    rows = np.arange(0, M, 128)
    ref_cols = orc.gemm_i8_i32(An, Wn[cols], nthreads=_nthreads())
    ref_rows = orc.gemm_i8_i32(An[rows], Wn, nthreads=_nthreads())
    got = out.cpu().numpy()
    assert np.array_equal(got[:, cols], ref_cols), "sampled columns differ"
    assert np.array_equal(got[rows], ref_rows), "tile first rows differ"


def test_config5_full_depth_decode_bit_exact(cuda_dev):
    from mamba_integer_b200 import kernels, synth
    from mamba_integer_b200.decode import DecodeEngine
    from mamba_integer_b200.mamba_integer_model import MambaIntegerModel
    from oracle import model as om
    c = synth.CONFIGS["c5"]
    cfg = synth.model_config("c5")
    sd = synth.model_state_dict(cfg, c["seed"])
    m = MambaIntegerModel(cfg)
    m.load_state_dict(sd)
    m = m.to(cuda_dev).eval()
    prompt = synth.input_ids("c5", c["batch"], c["seq_len"])  # 256 streams x 512 tokens
    watch = [0, 85, 170, 255]
    n_new = 8
    eng = DecodeEngine(m)  # the CUDA-graph step bench.py times
    logits = eng.start(prompt.to(cuda_dev))
    got_logits = [logits[watch].cpu().numpy()]
    kernels.argmax_rows(logits, out=eng.ws.next_ids)
    gen = []
    for _ in range(n_new):
        gen.append(eng.ws.next_ids[watch].cpu().numpy())
        got_logits.append(eng.step(eng.ws.next_ids)[watch].cpu().numpy())
    gen = np.stack(gen, 1)  # [4, n_new]
    seq = np.concatenate([prompt[watch].numpy(), gen], axis=1)
    ref = om.forward(om.prepare(sd), cfg, seq, nthreads=_nthreads())  # [4, 520, V]
    L = prompt.shape[1]
    for t in range(n_new + 1):
        r = ref[:, L - 1 + t, :]
        ne = got_logits[t].view(np.uint32) != r.view(np.uint32)
        assert not ne.any(), f"step {t}: {int(ne.sum())} logits differ from the full recompute"
        if t < n_new:
            assert (gen[:, t] == np.argmax(r, axis=-1)).all(), f"step {t}: greedy ids differ"
