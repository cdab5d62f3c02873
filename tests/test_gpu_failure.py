"""Failure paths of the bounded device waits.

The reference aborts the process on any CUDA error (CUDA_CHECK,
kernels/cuda_ops.cu:9-16).  Here every spin in a kernel -- on an mbarrier, a
tagged exchange word, a stage of the copy ring -- gives up after 2 s of
%globaltimer, records where, lets the copies and MMAs its CTA issued land,
releases its tensor memory and returns; the host reports VB_ERR_TIMEOUT and
the engine stays usable.

These tests make a wait run out without faulting anything: the library's
test hook (vb_debug_arm_fault) arms one launch to wait for something nothing
produces -- an exchange word no CTA writes (the clustered decode step) or a
stage no copy fills (the tensor-core GEMM).  Each test then checks the status
and the message, and that the next call computes the right answer again.
"""
import time

import numpy as np
import pytest

import oracle
import vb200
import vbsynth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_clustered_step_wait_runs_out_and_the_engine_recovers():
    cfg = vbsynth.qwen3_config(num_hidden_layers=2, vocab_size=4096)  # full widths: path 2
    w = vbsynth.make_weights(cfg, seed=17)
    prompt = vbsynth.prompt_ids(6, 18, cfg["vocab_size"])
    e = vb200.Engine(cfg).load(w)
    e.quantize()
    e.reset_cache(32)
    assert e.path() == 2
    e.step(int(prompt[0]))
    vb200.debug_arm_fault(1)
    t0 = time.time()
    with pytest.raises(vb200.VBError) as ei:
        e.step(int(prompt[1]))
    took = time.time() - t0
    assert ei.value.code == -8, ei.value
    # the message names the wait that gave up first (the armed gather, barring
    # a peer whose own wait began within microseconds of it)
    assert "timed out" in ei.value.msg and "[code" in ei.value.msg, ei.value.msg
    assert 1.5 < took < 30.0, took  # the 2 s bound, not an endless wait
    assert e.cache_len() == 1       # the failed step did not count
    # the same engine, from a fresh cache, matches the oracle again
    o = oracle.OracleModel(cfg, w)
    o.quantize()
    o.reset_cache(32)
    e.reset_cache(32)
    for t in prompt:
        d = float(np.max(np.abs(o.step(int(t)) - e.step(int(t)))))
        assert d <= 1e-2, d
    assert e.graph_nodes() == 1
    o.close()
    e.close()


def test_tensor_core_gemm_wait_runs_out_and_the_next_call_is_right():
    g = np.random.default_rng(5)
    M, N, K = 8, 512, 1024
    A = g.standard_normal((M, K)).astype(np.float32)
    Wf = (g.standard_normal((N, K)) * 0.02).astype(np.float32)
    q, sc = oracle.quantize_rows(Wf)
    dA, dq, dsc = (torch.from_numpy(x).cuda() for x in (A, q, sc))
    C = torch.zeros(M, N, device="cuda")
    vb200.debug_arm_fault(2)
    t0 = time.time()
    with pytest.raises(vb200.VBError) as ei:
        vb200.matmul_nt_tc(dA, dq, C, scales=dsc)
    took = time.time() - t0
    assert ei.value.code == -8 and "bounded wait" in ei.value.msg, ei.value
    assert 1.5 < took < 30.0, took
    # one-shot: the next call runs normally and is right
    vb200.matmul_nt_tc(dA, dq, C, scales=dsc)
    torch.cuda.synchronize()
    ref = (A.astype(np.float64) @ q.astype(np.float64).T) * sc.astype(np.float64)
    bound = 2e-5 * (np.abs(A).astype(np.float64) @ np.abs(q.astype(np.float64)).T) * sc + 1e-6
    assert np.all(np.abs(C.cpu().numpy() - ref) <= bound)


def test_disarming_leaves_launches_alone():
    g = np.random.default_rng(6)
    A = torch.from_numpy(g.standard_normal((4, 256)).astype(np.float32)).cuda()
    W = torch.from_numpy((g.standard_normal((128, 256)) * 0.02).astype(np.float32)).cuda()
    C = torch.zeros(4, 128, device="cuda")
    vb200.debug_arm_fault(2)
    vb200.debug_arm_fault(0)
    vb200.matmul_nt_tc(A, W, C)  # no timeout
    with pytest.raises(vb200.VBError):
        vb200.debug_arm_fault(7)
