"""BitLinear with the BitShift-norm + squareplus epilogue
on the GPU, bit for bit against the oracle (oracle/mi_oracle.c:
orc_bitlinear_norm_sqp): the int32 accumulators, the exact row sums and the
fp32 outputs, at small and ragged shapes and at config 3's full size."""
import numpy as np
import pytest
import torch

from oracle import lib as orc

pytestmark = pytest.mark.gpu


def _run(cuda_dev, A, Wq, a_scale, w_scale, gamma, step):
    from mamba_integer_b200 import kernels
    dev = cuda_dev
    Wp = kernels.pack_ternary(Wq.to(dev))
    ws = torch.tensor([w_scale], dtype=torch.float32, device=dev)
    st = torch.tensor([step], dtype=torch.float32, device=dev)
    stats = torch.full((A.shape[0], 2), 12345, dtype=torch.int64, device=dev)  # stale contents: zeroed by the call
    acc, out = kernels.bitlinear_packed_norm_sqp(A.to(dev), Wp, a_scale.to(dev), ws, gamma.to(dev), st,
                                                 stats_ws=stats)
    return acc.cpu().numpy(), out.cpu().numpy(), stats.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(300, 512, 256), (128, 96, 64), (257, 4096, 1024), (1000, 2048, 2048)])
def test_norm_sqp_matches_oracle(cuda_dev, M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    A = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    A[3] = 0  # an all-zero row: variance 0
    Wq = torch.randint(-1, 2, (N, K), generator=g, dtype=torch.int8)
    a_scale = torch.logspace(-5, 0, M).to(torch.float32)  # every power-of-two band
    gamma = (1.0 + 0.1 * torch.randn(N, generator=g)).to(torch.float32)
    acc, out, stats = _run(cuda_dev, A, Wq, a_scale, 2.0 ** -6, gamma, 0.875)
    acc_ref = orc.gemm_i8_i32(A.numpy(), Wq.numpy())
    assert np.array_equal(acc, acc_ref)
    out_ref, stats_ref = orc.bitlinear_norm_sqp(acc_ref, a_scale.numpy(), 2.0 ** -6, gamma.numpy(), 0.875)
    assert np.array_equal(stats, stats_ref)
    ne = out.view(np.uint32) != out_ref.view(np.uint32)
    assert not ne.any(), f"{int(ne.sum())} outputs differ"


def test_norm_sqp_config3_full_size(cuda_dev):
    from mamba_integer_b200 import synth
    A, a_scale, Wq, w_scale = synth.bitlinear_inputs()  # M 16384, K 2048, N 8192
    gamma, step = synth.bitlinear_norm_params()
    acc, out, stats = _run(cuda_dev, A, Wq, a_scale, w_scale, gamma, float(step[0]))
    rows = np.concatenate([np.arange(0, 16384, 128), np.arange(127, 16384, 1024)])
    acc_ref = orc.gemm_i8_i32(A.numpy()[rows], Wq.numpy())
    assert np.array_equal(acc[rows], acc_ref)
    out_ref, stats_ref = orc.bitlinear_norm_sqp(acc_ref, a_scale.numpy()[rows], w_scale, gamma.numpy(), float(step[0]))
    assert np.array_equal(stats[rows], stats_ref)
    assert np.array_equal(out[rows].view(np.uint32), out_ref.view(np.uint32))
    # every row's sums agree with its accumulators (the atomics over 32 tiles)
    a64 = acc.astype(np.int64)
    assert np.array_equal(stats[:, 0], a64.sum(1))
    assert np.array_equal(stats[:, 1], (a64 * a64).sum(1))


def test_norm_sqp_rejects_too_large_n_times_k(cuda_dev):
    from mamba_integer_b200 import _lib
    lib = _lib.load()
    t = torch.zeros(64, device=cuda_dev)
    p = t.data_ptr()
    # N * K = 2^25 > 2^24: the exact int64 statistics could overflow -> unsupported, nothing launched
    rc = lib.mi_bitlinear_packed_norm_sqp(p, 4096, p, p, p, p, p, p, 8192, p, 8192, p, 16, 8192, 4096, None)
    assert rc == -2
