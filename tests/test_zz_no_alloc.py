"""vb_attn_decode_noalloc: decode attention for callers that cannot allocate.

Callers such as a framework that owns all device memory through a budgeted
pool, or a plugin whose enqueue path may not allocate, use this entry point
instead of vb_attn_decode (which cudaMalloc's its scratch on first use).  Its
scratch is a fixed array compiled into the library.  This test drives it
through the C ABI and checks it against vb_attn_decode within the attention
tolerance of the other GPU tests, on two calls in a row (the second with a
shorter cache, so leftovers of the first call would show), at long contexts
where the split count is capped to fit the static buffer, and checks that a
head count needing more than the static buffer for one split is refused.  It sits in its own file
named to be collected last, and works alone in a fresh process too: its first
call also performs the one-time address lookup for the device.
"""
import numpy as np
import pytest

import vb200

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

H, KVH, D = 16, 8, 128


def _inputs(n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(H, D, device="cuda", generator=g)
    kc = torch.randn(n, KVH * D, device="cuda", generator=g)
    vc = torch.randn(n, KVH * D, device="cuda", generator=g)
    return q, kc, vc


def _compare(n, seed):
    q, kc, vc = _inputs(n, seed)
    got = torch.empty(H, D, device="cuda")
    vb200.attn_decode_noalloc(q, kc, vc, got, H, KVH, D, n)
    ref = torch.empty(H, D, device="cuda")
    vb200.attn_decode(q, kc, vc, ref, H, KVH, D, n)
    torch.cuda.synchronize()
    return float((got - ref).abs().max())


def test_noalloc_matches_allocating_entry_point_twice():
    for call, n in enumerate((4096, 777)):
        diff = _compare(n, 900 + call)
        assert np.isfinite(diff) and diff <= 2e-5, (call, n, diff)


def test_noalloc_long_contexts_run_with_capped_splits():
    # 16/8 heads: past ~16k positions the allocating entry point uses more
    # splits (up to 148, of >= 128 positions) than the 1 MiB array holds (124);
    # the no-alloc one caps the split count (longer splits) and must still
    # agree.  40960 is the model's max_position_embeddings; 15872 is the last
    # length whose split count fits, 16000 the first that is capped.
    for n in (15872, 16000, 32768, 40960):
        diff = _compare(n, n)
        assert np.isfinite(diff) and diff <= 2e-5, (n, diff)
        torch.cuda.empty_cache()


def test_noalloc_refuses_heads_beyond_the_static_buffer():
    # one split of 2048 heads needs 2048 x 132 floats + 512 B > 1 MiB, so the
    # size check refuses it before anything is launched (GQA group 2 is a
    # shape the attention kernels take, so only the size check can refuse it)
    h, kvh, n = 2048, 1024, 4
    q = torch.zeros(h, D, device="cuda")
    kc = torch.zeros(n, kvh * D, device="cuda")
    vc = torch.zeros(n, kvh * D, device="cuda")
    out = torch.zeros(h, D, device="cuda")
    with pytest.raises(vb200.VBError) as ei:
        vb200.attn_decode_noalloc(q, kc, vc, out, h, kvh, D, n)
    assert ei.value.code == -9 and "static buffer" in ei.value.msg
