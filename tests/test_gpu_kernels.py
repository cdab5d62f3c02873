"""Kernel-level parity of the sm_100a kernels against the CPU oracle.

Shapes are the Qwen3-0.6B decode shapes: the GEMV microbenchmark
(1024->2048 q, 1024->1024 k/v, 2048->1024 o, 1024->3072 gate/up,
3072->1024 down, 1024->151936 lm_head) in f32 and INT8, and the isolated GQA
attention sweep (16 Q / 8 KV heads, D=128, KV length 512..32768, batch 1 and
32).  Every call goes through the C ABI (vb200 -> libverbum_b200.so).

Tolerances: INT8 quantisation is compared bit for bit; RoPE is bit-exact by
construction (the same float operations); GEMV outputs within 1e-4 absolute
(values ~0.6 in magnitude, an f32 summation-order difference); attention
within 2e-5.
"""
import numpy as np
import pytest

import oracle
import vb200

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GEMV_SHAPES = [("q", 1024, 2048), ("k", 1024, 1024), ("o", 2048, 1024), ("gate", 1024, 3072),
               ("down", 3072, 1024), ("lm_head", 1024, 151936), ("odd", 528, 40)]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def weights(N, K, seed):
    return vb200.synth_normal(N * K, seed, 0.02).reshape(N, K)


def xvec(M, K, seed):
    return np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)


@pytest.mark.parametrize("name,K,N", GEMV_SHAPES, ids=[s[0] for s in GEMV_SHAPES])
def test_gemv_f32(name, K, N):
    W = weights(N, K, 100 + K + N)
    x = xvec(1, K, 1)
    y = torch.empty(1, N, device="cuda")
    vb200.matmul_nt_f32(dev(x), dev(W), y)
    ref = oracle.matmul_nt(x, W)
    assert np.max(np.abs(host(y) - ref)) < 1e-4


@pytest.mark.parametrize("name,K,N", GEMV_SHAPES, ids=[s[0] for s in GEMV_SHAPES])
def test_quantize_and_gemv_q8(name, K, N):
    W = weights(N, K, 200 + K + N)
    W[0, :] = 0.0
    dW = dev(W)
    q = torch.empty(N, K, dtype=torch.int8, device="cuda")
    s = torch.empty(N, device="cuda")
    vb200.quantize_rows(dW, q, s)
    q_ref, s_ref = oracle.quantize_rows(W)
    assert np.array_equal(host(q), q_ref)
    assert np.array_equal(host(s).view(np.uint32), s_ref.view(np.uint32))
    if K % 16:
        return
    x = xvec(1, K, 2)
    y = torch.empty(1, N, device="cuda")
    vb200.matmul_nt_q8(dev(x), q, s, y)
    assert np.max(np.abs(host(y) - oracle.matmul_nt_q8(x, q_ref, s_ref))) < 1e-4


@pytest.mark.parametrize("M", [2, 3, 64])
@pytest.mark.parametrize("q8", [False, True])
def test_batched_matmul(M, q8):
    K, N = 1024, 3072
    W = weights(N, K, 300 + M)
    x = xvec(M, K, 3)
    y = torch.empty(M, N, device="cuda")
    if q8:
        q_ref, s_ref = oracle.quantize_rows(W)
        vb200.matmul_nt_q8(dev(x), dev(q_ref), dev(s_ref), y)
        ref = oracle.matmul_nt_q8(x, q_ref, s_ref)
    else:
        vb200.matmul_nt_f32(dev(x), dev(W), y)
        ref = oracle.matmul_nt(x, W)
    assert np.max(np.abs(host(y) - ref)) < 1e-4


def test_rmsnorm_rows():
    x = xvec(5, 1024, 4) * 3
    w = (1 + 0.1 * xvec(1, 1024, 5)[0]).astype(np.float32)
    out = torch.empty(5, 1024, device="cuda")
    vb200.rmsnorm(dev(x), dev(w), out, 1e-6)
    ref = oracle.rmsnorm(x, w, 1e-6)
    got = host(out)
    assert np.max(np.abs(got - ref)) < 1e-6
    assert np.mean(got == ref) > 0.99  # double sum of squares as the reference: ~all bits equal


def test_rmsnorm_many_rows():
    # 1024 rows and more take the warp-per-row form (8 rows per CTA)
    x = xvec(1027, 1024, 14) * 3
    w = (1 + 0.1 * xvec(1, 1024, 15)[0]).astype(np.float32)
    out = torch.empty(1027, 1024, device="cuda")
    vb200.rmsnorm(dev(x), dev(w), out, 1e-6)
    ref = oracle.rmsnorm(x, w, 1e-6)
    got = host(out)
    assert np.max(np.abs(got - ref)) < 1e-6
    assert np.mean(got == ref) > 0.99


def test_rope_bitexact():
    c, s = oracle.rope_table(128, 4096, 1e6)
    for pos in (0, 7, 4095):
        x = xvec(16, 128, 6 + pos)
        dx = dev(x)
        vb200.rope(dx, dev(c), dev(s), pos)
        assert np.array_equal(host(dx), oracle.apply_rope(x, pos, c, s))


def test_silu_mul_add_cache_append():
    g = xvec(1, 3072, 7)[0] * 4
    u = xvec(1, 3072, 8)[0]
    dg = dev(g)
    vb200.silu_mul(dg, dev(u))
    assert np.max(np.abs(host(dg) - oracle.silu_mul(g, u))) < 1e-5
    a, b = xvec(1, 1024, 9)[0], xvec(1, 1024, 10)[0]
    da = dev(a)
    vb200.add(da, dev(b))
    assert np.array_equal(host(da), a + b)
    kc = torch.zeros(8, 1024, device="cuda")
    vc = torch.zeros(8, 1024, device="cuda")
    kn, vn = xvec(1, 1024, 11)[0], xvec(1, 1024, 12)[0]
    vb200.cache_append(kc, vc, dev(kn), dev(vn), 5)
    assert np.array_equal(host(kc)[5], kn) and np.array_equal(host(vc)[5], vn)
    assert not host(kc)[4].any()


def test_argmax_ties_lowest_index():
    lg = np.zeros((3, 151936), np.float32)
    lg[0, [7, 99, 151935]] = 5.0
    lg[1] = xvec(1, 151936, 13)[0]
    lg[2, :] = -np.inf
    out = torch.empty(3, dtype=torch.int32, device="cuda")
    vb200.argmax_rows(dev(lg), out)
    got = host(out)
    assert got[0] == 7 and got[1] == oracle.argmax(lg[1]) and got[2] == 0


@pytest.mark.parametrize("n", [1, 5, 40, 200, 512, 2048, 8192, 32768])
def test_attn_decode_reference_layout(n):
    """vb_attn_decode on the reference's [n, KVH*D] cache (generate.cpp:73-105)."""
    H, KVH, D = 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(n)
    q = torch.randn(H, D, device="cuda", generator=g)
    kc = torch.randn(n, KVH * D, device="cuda", generator=g)
    vc = torch.randn(n, KVH * D, device="cuda", generator=g)
    out = torch.empty(H, D, device="cuda")
    vb200.attn_decode(q, kc, vc, out, H, KVH, D, n)
    ref = oracle.attention_decode(host(q), host(kc), host(vc), H, KVH, D, n)
    assert np.max(np.abs(host(out) - ref)) < 2e-5


@pytest.mark.parametrize("n", [512, 2048, 8192, 32768])
def test_attn_decode_batched_b32(n):
    """Config-4 batch 32, cache laid out [B, n, KVH, D]; ragged lengths."""
    B, H, KVH, D = 32, 16, 8, 128
    g = torch.Generator(device="cuda").manual_seed(1000 + n)
    q = torch.randn(B, H, D, device="cuda", generator=g)
    k = torch.randn(B, n, KVH, D, device="cuda", generator=g)
    v = torch.randn(B, n, KVH, D, device="cuda", generator=g)
    lens_h = np.full(B, n, np.int32)
    lens_h[1] = 1
    lens_h[2] = max(1, n // 3 + 1)
    lens = dev(lens_h)
    out = torch.empty(B, H, D, device="cuda")
    ws = torch.empty(vb200.attn_workspace_bytes(B, H, n) // 4 + 1, device="cuda")
    vb200.attn_decode_batched(q, k, v, out, lens, B, H, KVH, D, n, n * KVH * D, KVH * D, D, ws)
    got = host(out)
    for b in (0, 1, 2, B - 1):
        ref = oracle.attention_decode(host(q[b]), host(k[b].reshape(n, KVH * D)),
                                      host(v[b].reshape(n, KVH * D)), H, KVH, D, int(lens_h[b]))
        assert np.max(np.abs(got[b] - ref)) < 2e-5, b
