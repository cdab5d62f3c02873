"""Tensor-core batched projection (vb_matmul_nt_tc: TMA + tcgen05.mma + TMEM)
against the exact (f64) product of the same operands, and the CPU oracle.

C = A . W^T for M activation rows: the batched form of matmul_nt
(ops.cpp:42-70) and matmul_nt_q8 (quant.cpp:43-70).  The operands are bf16
hi+lo splits (exact int8 weights), so the result tracks the f32 reference to
~2^-16 of the products' magnitude: the tolerance is 2e-5 * sum_k |a_k w_k|
per element (values ~0.6, sums of |products| ~20, so ~4e-4 absolute at most,
about 100x below the logits tolerance) plus a floor of 1e-6.  Shapes cover
the batched-step projections (q|k|v 4096, o 1024 x 2048, gate|up 6144,
down 1024 x 3072), a partial 128-row tile, K of one chunk, M of 1, 7, 64,
and several 64-row activation tiles (65, and 1000 rows as in a prefill).
"""
import numpy as np
import pytest

import oracle
import vb200

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

SHAPES = [  # (M, N, K)
    (64, 4096, 1024),
    (64, 1024, 2048),
    (64, 6144, 1024),
    (64, 1024, 3072),
    (7, 200, 64),
    (1, 384, 512),
    (33, 1000, 1024),
    (65, 1024, 2048),     # two activation tiles, the second of one row
    (1000, 3072, 1024),   # prefill-sized: wide tiles (128 activation x 256 weight rows)
    (300, 1000, 2048),    # wide tiles with partial activation and weight tiles
    (128, 256, 64),       # one wide tile, one K step
]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bound(A, W):
    return 2e-5 * (np.abs(A).astype(np.float64) @ np.abs(W).astype(np.float64).T) + 1e-6


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_f32_weights(M, N, K):
    A = vb200.synth_normal(M * K, 1000 + M + K, 1.0).reshape(M, K)
    W = vb200.synth_normal(N * K, 2000 + N + K, 0.02).reshape(N, K)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    vb200.matmul_nt_tc(dev(A), dev(W), C)
    got = host(C).astype(np.float64)
    exact = A.astype(np.float64) @ W.astype(np.float64).T
    err = np.abs(got - exact)
    assert np.all(err <= bound(A, W)), f"max err {err.max():.3e}"
    # the oracle's sequential f32 sum differs from the exact sum by its own rounding
    assert np.max(np.abs(got - oracle.matmul_nt(A, W))) < 1e-3


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_int8_weights(M, N, K):
    A = vb200.synth_normal(M * K, 3000 + M + K, 1.0).reshape(M, K)
    W = vb200.synth_normal(N * K, 4000 + N + K, 0.02).reshape(N, K)
    q, sc = oracle.quantize_rows(W)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    vb200.matmul_nt_tc(dev(A), dev(q), C, scales=dev(sc))
    got = host(C).astype(np.float64)
    exact = (A.astype(np.float64) @ q.astype(np.float64).T) * sc.astype(np.float64)[None, :]
    deq = q.astype(np.float64) * sc[:, None]
    err = np.abs(got - exact)
    assert np.all(err <= bound(A, deq)), f"max err {err.max():.3e}"
    assert np.max(np.abs(got - oracle.matmul_nt_q8(A, q, sc))) < 1e-3


def test_tc_gemm_rejects_bad_shapes():
    A2 = torch.zeros((4, 100), dtype=torch.float32, device="cuda")
    W2 = torch.zeros((128, 100), dtype=torch.float32, device="cuda")
    C2 = torch.zeros((4, 128), dtype=torch.float32, device="cuda")
    with pytest.raises(vb200.VBError):
        vb200.matmul_nt_tc(A2, W2, C2)
