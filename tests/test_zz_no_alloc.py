"""vb_attn_decode_noalloc: decode attention for callers that cannot allocate.

Callers such as a framework that owns all device memory through a budgeted
pool, or a plugin whose enqueue path may not allocate, use this entry point
instead of vb_attn_decode (which cudaMalloc's its scratch on first use).  Its
scratch is a fixed array compiled into the library.  This test drives it
through the C ABI and checks it against vb_attn_decode within the attention
tolerance of the other GPU tests, on two calls in a row (the second with a
shorter cache, so leftovers of the first call would show), and checks that a
shape needing more than the static buffer is refused.  It sits in its own file
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


def test_noalloc_matches_allocating_entry_point_twice():
    for call, n in enumerate((4096, 777)):
        q, kc, vc = _inputs(n, 900 + call)
        got = torch.empty(H, D, device="cuda")
        vb200.attn_decode_noalloc(q, kc, vc, got, H, KVH, D, n)
        ref = torch.empty(H, D, device="cuda")
        vb200.attn_decode(q, kc, vc, ref, H, KVH, D, n)
        torch.cuda.synchronize()
        diff = float((got - ref).abs().max())
        assert np.isfinite(diff) and diff <= 2e-5, (call, n, diff)


def test_noalloc_refuses_shapes_beyond_the_static_buffer():
    h, kvh, n = 64, 1, 40000  # 592 splits x 64 heads x 130 floats: ~19.7 MB
    q = torch.zeros(h, D, device="cuda")
    kc = torch.zeros(n, kvh * D, device="cuda")
    vc = torch.zeros(n, kvh * D, device="cuda")
    out = torch.zeros(h, D, device="cuda")
    with pytest.raises(vb200.VBError) as ei:
        vb200.attn_decode_noalloc(q, kc, vc, out, h, kvh, D, n)
    assert ei.value.code == -9 and "static buffer" in ei.value.msg
