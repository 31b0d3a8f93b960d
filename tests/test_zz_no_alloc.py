"""The allocation-free decode attention entry point, called through the C ABI.

krk_k_rope_kv_attn_decode_noalloc exists for callers that cannot hand the
library device scratch memory (a host that binds only the C header and has no
CUDA allocator of its own, or a process whose device memory belongs to another
allocator or a fixed budget).  Its results must equal those of
krk_k_rope_kv_attn_decode given a caller-allocated scratch buffer, on two calls
in a row (the second call sees whatever the first left in the shared fixed
scratch), and it must refuse sizes beyond its fixed scratch.  This file is
collected last so that a run stopping at the first failure has run every other
test already; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from krikil_rs_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from krikil_rs_b200._lib import INVALID, OK, lib  # noqa: E402

DEV = torch.device("cuda:0")
ATOL, RTOL = 1e-4, 1e-5  # the attention tolerance of the other GPU tests


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _with_buffer(q, k, v, kc, vc, pos, b, h, dh, ctx, split, stream):
    work = torch.empty(int(lib.krk_attn_work_floats(b, h, dh, ctx, split)), device=DEV)
    out = torch.empty_like(q)
    rc = lib.krk_k_rope_kv_attn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                       pos.data_ptr(), out.data_ptr(), work.data_ptr(), b, h, dh, ctx, split,
                                       10000.0, stream)
    assert rc == OK, lib.krk_last_error()
    return out


def _no_alloc(q, k, v, kc, vc, pos, b, h, dh, ctx, split, stream):
    out = torch.empty_like(q)
    rc = lib.krk_k_rope_kv_attn_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(),
                                               vc.data_ptr(), pos.data_ptr(), out.data_ptr(), b, h, dh, ctx, split,
                                               10000.0, stream)
    assert rc == OK, lib.krk_last_error()
    return out


@pytest.mark.parametrize("b,h,dh,ctx,split", [
    (64, 8, 64, 2048, 256),  # the [64,8,2048,64] decode benchmark shape: generic split kernel, narrow merge
    (16, 8, 64, 2048, 64),   # warp-per-16-keys split kernel and the wide merge (32 splits per sequence)
], ids=["split256", "split64-wide-merge"])
def test_no_alloc_matches_buffered_entry_point_twice(b, h, dh, ctx, split):
    assert lib.krk_attn_work_floats(b, h, dh, ctx, split) <= (1 << 20)
    q, k, v, pos, kc, vc = synth.attn_decode_inputs(b, h, dh, ctx, seed=0)
    stream = torch.cuda.current_stream().cuda_stream
    kc_a, vc_a, kc_b, vc_b = _t(kc), _t(vc), _t(kc), _t(vc)
    rng = np.random.default_rng(7)
    for call in range(2):
        if call == 1:  # new tokens one position further on
            pos = np.minimum(pos + 1, ctx - 1).astype(np.int32)
            q, k, v = (rng.standard_normal((b, h, dh)).astype(np.float32) for _ in range(3))
        gq, gk, gv, gp = _t(q), _t(k), _t(v), _t(pos)
        ref = _with_buffer(gq, gk, gv, kc_a, vc_a, gp, b, h, dh, ctx, split, stream)
        got = _no_alloc(gq, gk, gv, kc_b, vc_b, gp, b, h, dh, ctx, split, stream)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=ATOL, rtol=RTOL,
                                   err_msg=f"call {call}")
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)


def test_no_alloc_runs_on_the_streams_device_and_keeps_the_callers_device():
    """A stream of device 0 passed while device 0 is current: the call succeeds
    and the current device is unchanged afterwards (with one GPU the stream's
    device is always the current one; the lookup path is the same)."""
    b, h, dh, ctx, split = 4, 8, 64, 512, 64
    q, k, v, pos, kc, vc = synth.attn_decode_inputs(b, h, dh, ctx, seed=3)
    s = torch.cuda.Stream(device=DEV)
    gq, gk, gv, gp, gkc, gvc = (_t(a) for a in (q, k, v, pos, kc, vc))
    before = torch.cuda.current_device()
    got = _no_alloc(gq, gk, gv, gkc, gvc, gp, b, h, dh, ctx, split, s.cuda_stream)
    s.synchronize()
    assert torch.cuda.current_device() == before
    ref = _with_buffer(gq, gk, gv, _t(kc), _t(vc), gp, b, h, dh, ctx, split, s.cuda_stream)
    s.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), atol=ATOL, rtol=RTOL)


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    b, h, dh, ctx, split = 1024, 8, 76, 8192, 64
    assert lib.krk_attn_work_floats(b, h, dh, ctx, split) > (1 << 20)
    dummy = torch.zeros(16, device=DEV)
    p = dummy.data_ptr()
    rc = lib.krk_k_rope_kv_attn_decode_noalloc(p, p, p, p, p, p, p, b, h, dh, ctx, split, 10000.0,
                                               torch.cuda.current_stream().cuda_stream)
    assert rc == INVALID
    msg = lib.krk_last_error().decode()
    assert "scratch" in msg and str(1 << 20) in msg
