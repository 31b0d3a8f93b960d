"""Per-kernel parity of the CUDA library (through its C ABI) against the CPU
oracle, on seeded inputs.  Tolerances are written per test; the projections
are bit-exact by construction."""
import numpy as np
import pytest

import oracle as O
from krikil_rs_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from krikil_rs_b200 import _lib, kernels as K  # noqa: E402

DEV = torch.device("cuda:0")


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def np_(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ------------------------------------------------------------- projections
@pytest.mark.parametrize("m,n,k", [(64, 32, 32), (128, 2720, 608), (64, 608, 1216), (192, 608, 2432),
                                   (64, 2048, 608), (256, 1824, 608)])
@pytest.mark.parametrize("out_fm", [False, True])
@pytest.mark.parametrize("tile", [0, 16, 32, 64])
def test_gemm_bit_exact_vs_reference_dot(m, n, k, out_fm, tile):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    ref = O.gemm_transb(a, w)  # each element = the reference dot (src/math.rs:89-124)
    c = K.gemm(cu(a.T.copy()), cu(w.T.copy()), 0, out_fm, tile_rows=tile)
    got = np_(c).T if out_fm else np_(c)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("tile", [16, 32, 64])
def test_gemm_residual_and_gelu_epilogues(tile):
    rng = np.random.default_rng(1)
    m, n, k = 128, 608, 2432
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    res = rng.standard_normal((n, m)).astype(np.float32)
    ref = O.gemm_transb(a, w)
    c = cu(res.copy())
    K.gemm(cu(a.T.copy()), cu(w.T.copy()), 1, True, c, tile_rows=tile)
    np.testing.assert_array_equal(np_(c), res + ref.T)
    cb = cu(res.T.copy())
    K.gemm(cu(a.T.copy()), cu(w.T.copy()), 1, False, cb, tile_rows=tile)
    np.testing.assert_array_equal(np_(cb), res.T + ref)
    g = np_(K.gemm(cu(a.T.copy()), cu(w.T.copy()), 2, True, tile_rows=tile))
    gref = np.vectorize(O.gelu, otypes=[np.float32])(ref.T)
    np.testing.assert_allclose(g, gref, atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("m,n,k", [(1024, 2720, 608), (2048, 608, 2432)])
@pytest.mark.parametrize("tile", [16, 32, 64])
def test_gemm_many_waves_all_epilogues(m, n, k, tile):
    """Decode shapes with several tiles per SM (1360-5440 tiles): every output
    of every wave equals the reference dot, in both output layouts, and the
    residual and GELU epilogues apply to every tile."""
    rng = np.random.default_rng(m + n + k + tile)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    ref = O.gemm_transb(a, w)
    at, wt = cu(a.T.copy()), cu(w.T.copy())
    np.testing.assert_array_equal(np_(K.gemm(at, wt, 0, False, tile_rows=tile)), ref)
    np.testing.assert_array_equal(np_(K.gemm(at, wt, 0, True, tile_rows=tile)).T, ref)
    res = rng.standard_normal((n, m)).astype(np.float32)
    c = cu(res.copy())
    K.gemm(at, wt, 1, True, c, tile_rows=tile)
    np.testing.assert_array_equal(np_(c), res + ref.T)
    g = np_(K.gemm(at, wt, 2, False, tile_rows=tile))
    np.testing.assert_allclose(g, np.vectorize(O.gelu, otypes=[np.float32])(ref), atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("n,k", [(2720, 608), (608, 2432), (32, 32)])
def test_gemm_few_rows_form(m, n, k):
    """tile_rows 1, the decode form for up to 8 sequences (one thread per
    output column and dot lane, only the m real rows of a 64-wide operand):
    bitwise the reference dot in both layouts, with the residual epilogue, and
    the GELU epilogue within its tolerance; no padded row is written."""
    rng = np.random.default_rng(m * 31 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    ref = O.gemm_transb(a, w)
    at = np.zeros((k, 64), np.float32)
    at[:, :m] = a.T
    g_at, g_wt = cu(at), cu(w.T.copy())
    lib, st = _lib.lib, torch.cuda.current_stream().cuda_stream

    def run(epi, fm, c):
        ldc = c.shape[1]
        rc = lib.krk_k_gemm_tiled(g_at.data_ptr(), 64, g_wt.data_ptr(), n, c.data_ptr(), ldc, m, n, k, epi, int(fm), 1, st)
        assert rc == _lib.OK, lib.krk_last_error()
        return np_(c)

    marker = np.float32(-7.0)
    got = run(0, False, cu(np.full((8, n), marker, np.float32)))
    np.testing.assert_array_equal(got[:m], ref)
    assert (got[m:] == marker).all()
    got = run(0, True, cu(np.full((n, 64), marker, np.float32)))
    np.testing.assert_array_equal(got[:, :m], ref.T)
    assert (got[:, m:] == marker).all()
    res = rng.standard_normal((n, 64)).astype(np.float32)
    got = run(1, True, cu(res.copy()))
    np.testing.assert_array_equal(got[:, :m], res[:, :m] + ref.T)
    np.testing.assert_array_equal(got[:, m:], res[:, m:])
    got = run(2, False, cu(np.zeros((8, n), np.float32)))
    np.testing.assert_allclose(got[:m], np.vectorize(O.gelu, otypes=[np.float32])(ref), atol=1e-6, rtol=1e-5)


def test_gemm_rejects_bad_shapes():
    from krikil_rs_b200._lib import KrikilError
    with pytest.raises(KrikilError):
        K.gemm(torch.zeros(32, 60, device=DEV), torch.zeros(32, 32, device=DEV))


@pytest.mark.parametrize("m,n,k", [(64, 32, 32), (64, 64, 288), (128, 2720, 608), (64, 608, 1216),
                                   (192, 608, 2432), (64, 1824, 608), (128, 2432, 608),
                                   # the wide form (M % 256 == 0): block sums added in C
                                   (256, 32, 32), (256, 64, 288), (256, 2720, 608), (512, 608, 2432),
                                   (256, 1824, 608), (768, 608, 1216)])
def test_gemm_sgemm_order_bit_exact(m, n, k):
    """krk_k_gemm_sgemm_order against the oracle's restatement of
    matrixmultiply 0.3.11's sgemm order (the reference's prefill GEMM,
    src/math.rs:188-211), bitwise, at the prefill projection shapes and at K
    one K-block past a 256-long block; the dot-order kernel rounds differently."""
    rng = np.random.default_rng(m * 5 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    w = (0.02 * rng.standard_normal((n, k))).astype(np.float32)
    with O.prefill_gemm_order("matrixmultiply"):
        ref = O.gemm_transb(a, w)
    a_t, w_t = cu(a.T.copy()), cu(w.T.copy())
    np.testing.assert_array_equal(np_(K.gemm_sgemm_order(a_t, w_t)), ref)
    if k >= 64:
        assert not np.array_equal(np_(K.gemm(a_t, w_t)), ref)


@pytest.mark.parametrize("m", [64, 256])
def test_gemm_sgemm_order_known_answer(m):
    """One float32 FMA chain per 256-long block of K: 1 + 2^-24 + 2^-24 - 1 in
    one block gives 0 (each 2^-24 absorbed), split over two blocks 2^-23."""
    a = np.zeros((m, 512), np.float32)
    a[0, [0, 1, 2, 3]] = [1.0, 2.0 ** -24, 2.0 ** -24, -1.0]
    a[1, [0, 1, 256, 257]] = [1.0, -1.0, 2.0 ** -24, 2.0 ** -24]
    w = np.ones((32, 512), np.float32)
    c = np_(K.gemm_sgemm_order(cu(a.T.copy()), cu(w.T.copy())))
    assert (c[0] == 0.0).all() and (c[1] == np.float32(2.0 ** -23)).all() and not c[2:].any()


def test_gemm_sgemm_order_rejects_bad_shapes():
    from krikil_rs_b200._lib import KrikilError
    with pytest.raises(KrikilError):  # M not a multiple of 64
        K.gemm_sgemm_order(torch.zeros(32, 96, device=DEV), torch.zeros(32, 32, device=DEV))
    with pytest.raises(KrikilError):  # K not a multiple of 32
        K.gemm_sgemm_order(torch.zeros(40, 64, device=DEV), torch.zeros(40, 32, device=DEV))


# ------------------------------------------------------------- norms
@pytest.mark.parametrize("kdim,m,ld", [(608, 64, 64), (1216, 37, 64), (608, 1, 64), (608, 1024, 1024),
                                       (100, 13, 16)])
def test_rmsnorm_feature_major(kdim, m, ld):
    """The sum of squares runs as 32 ordered partials and a fixed tree instead
    of the reference's one sequential chain: the same to within a few ulps of
    the scale (relative 2e-6 here), and identical for a column whatever its
    batch or position in the block."""
    rng = np.random.default_rng(kdim + m)
    x = (rng.standard_normal((ld, kdim)) * rng.uniform(0.1, 3.0, (ld, 1))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(kdim)).astype(np.float32)
    eps = 1e-6 if kdim == 608 else 1e-5
    out = np_(K.rmsnorm_fm(cu(x.T.copy()), cu(w), eps, m))
    for col in range(m):
        np.testing.assert_allclose(out[:, col], O.rms_norm(x[col], w, eps), rtol=2e-6, atol=1e-7)
    # a column's result does not depend on the rest of its block or batch
    alone = np_(K.rmsnorm_fm(cu(x[m - 1:m].T.copy()), cu(w), eps, 1))
    np.testing.assert_array_equal(alone[:, 0], out[:, m - 1])


def test_rmsnorm_rows():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((1000, 512)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    np.testing.assert_allclose(np_(K.rmsnorm_rows(cu(x), cu(w), 1e-6)), O.rms_norm_rows(x, w, 1e-6),
                               atol=1e-5, rtol=1e-5)


def test_gated_rmsnorm_residual_full_size():
    """Config: x,z,res ~N(0,1) [16384,512], w ~N(1,0.1), eps 1e-5."""
    x, z, res, w = synth.fused_norm_inputs()
    got = np_(K.gated_rmsnorm_residual(cu(x), cu(z), cu(res), cu(w), 1e-5))
    ref = O.gated_rmsnorm_residual(x, z, res, w, 1e-5)
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-5)
    assert np.abs(got - ref).max() < 1e-5


@pytest.mark.parametrize("dim", [128, 256, 1024])
def test_gated_rmsnorm_residual_dims(dim):
    x, z, res, w = synth.fused_norm_inputs(rows=33, dim=dim, seed=dim)
    got = np_(K.gated_rmsnorm_residual(cu(x), cu(z), cu(res), cu(w), 1e-5))
    np.testing.assert_allclose(got, O.gated_rmsnorm_residual(x, z, res, w, 1e-5), atol=1e-5, rtol=1e-5)


# ------------------------------------------------------------- pointwise / embed
@pytest.mark.parametrize("op,fn", [(0, O.silu), (1, O.softplus), (2, O.gelu)])
def test_pointwise(op, fn):
    x = np.concatenate([np.linspace(-30, 30, 5001), [0.0, -0.0, 20.0, 20.000002, -87.0, 88.0]]).astype(np.float32)
    got = np_(K.pointwise(op, cu(x)))
    ref = np.array([fn(float(v)) for v in x], np.float32)
    np.testing.assert_allclose(got, ref, atol=1e-6, rtol=2e-6)


def test_embed_exact():
    rng = np.random.default_rng(2)
    wte = rng.standard_normal((2048, 608)).astype(np.float32)
    tok = np.array([0, 2047, 5, 5, 1000], np.uint32)
    out = np_(K.embed(cu(tok.view(np.int32)), cu(wte), ld=64))
    np.testing.assert_array_equal(out[:, :5].T, wte[tok])
    assert not out[:, 5:].any()


# ------------------------------------------------------------- Mamba2
def _ssd_case(bsz, t, nh=16, seed=0, state_scale=1.0):
    x, bm, cm, dt, cs, ssm = synth.conv_ssd_inputs(bsz, t, nh=nh, seed=seed, state_scale=state_scale)
    params = synth.conv_ssd_params(nh=nh, seed=seed)
    return x, bm, cm, dt, cs, ssm, params


def test_conv_ssd_step_full_size():
    """Config: batch 256, 16 heads x 64, d_state 128, conv state [256,1024,3]."""
    x, bm, cm, dt, cs, ssm, (cw, cb, dtb, an, dsk) = _ssd_case(256, 1)
    g_cs, g_ssm = cu(cs), cu(ssm)
    y = K.conv_ssd_step(cu(x[:, 0]), cu(bm[:, 0]), cu(cm[:, 0]), cu(dt[:, 0]), g_cs, cu(cw), cu(cb), g_ssm,
                        cu(dtb), cu(an), cu(dsk))
    o_cs, o_ssm = cs.copy(), ssm.copy()
    yr = O.conv_ssd_step(x[:, 0].copy(), bm[:, 0].copy(), cm[:, 0].copy(), dt[:, 0].copy(), o_cs, cw, cb, dtb,
                         an, dsk, o_ssm)
    np.testing.assert_array_equal(np_(g_cs), o_cs)  # conv state is a pure shift
    np.testing.assert_allclose(np_(g_ssm), o_ssm, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(np_(y), yr, atol=1e-4, rtol=1e-5)


def test_conv_ssd_step_repeated_steps():
    x, bm, cm, dt, cs, ssm, (cw, cb, dtb, an, dsk) = _ssd_case(8, 6, seed=3)
    g_cs, g_ssm = cu(cs), cu(ssm)
    o_cs, o_ssm = cs.copy(), ssm.copy()
    for t in range(6):
        y = K.conv_ssd_step(cu(x[:, t]), cu(bm[:, t]), cu(cm[:, t]), cu(dt[:, t]), g_cs, cu(cw), cu(cb), g_ssm,
                            cu(dtb), cu(an), cu(dsk))
        yr = O.conv_ssd_step(x[:, t].copy(), bm[:, t].copy(), cm[:, t].copy(), dt[:, t].copy(), o_cs, cw, cb,
                             dtb, an, dsk, o_ssm)
        np.testing.assert_allclose(np_(y), yr, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(np_(g_ssm), o_ssm, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("bsz,t", [(3, 1), (2, 31), (2, 33), (4, 100)])
def test_conv_ssd_scan_vs_oracle(bsz, t):
    x, bm, cm, dt, cs, ssm, (cw, cb, dtb, an, dsk) = _ssd_case(bsz, t, seed=t)
    g_cs, g_ssm = cu(cs), cu(ssm)
    y = K.conv_ssd_scan(cu(x), cu(bm), cu(cm), cu(dt), g_cs, cu(cw), cu(cb), g_ssm, cu(dtb), cu(an), cu(dsk))
    o_cs, o_ssm = cs.copy(), ssm.copy()
    yr = O.conv_ssd_scan(x, bm, cm, dt, o_cs, cw, cb, dtb, an, dsk, o_ssm)
    np.testing.assert_array_equal(np_(g_cs), o_cs)
    np.testing.assert_allclose(np_(g_ssm), o_ssm, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(np_(y), yr, atol=1e-4, rtol=1e-5)


def test_conv_ssd_scan_equals_repeated_steps():
    """The prefill scan and T single steps implement the same recurrence."""
    x, bm, cm, dt, cs, ssm, (cw, cb, dtb, an, dsk) = _ssd_case(4, 40, seed=9)
    s_cs, s_ssm = cu(cs), cu(ssm)
    ys = K.conv_ssd_scan(cu(x), cu(bm), cu(cm), cu(dt), s_cs, cu(cw), cu(cb), s_ssm, cu(dtb), cu(an), cu(dsk))
    t_cs, t_ssm = cu(cs), cu(ssm)
    yt = [np_(K.conv_ssd_step(cu(x[:, i]), cu(bm[:, i]), cu(cm[:, i]), cu(dt[:, i]), t_cs, cu(cw), cu(cb), t_ssm,
                              cu(dtb), cu(an), cu(dsk))) for i in range(40)]
    np.testing.assert_allclose(np_(ys), np.stack(yt, 1), atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(np_(s_ssm), np_(t_ssm), atol=1e-4, rtol=1e-5)


def test_conv_ssd_scan_split_invariance_full_size():
    """Config shapes (B=256, T=2048): one 2048-token scan equals two 1024-token
    scans carrying the state (bitwise: chunk boundaries coincide), and sampled
    sequences match the oracle's sequential recurrence."""
    bsz, t = 256, 2048
    x, bm, cm, dt, cs, ssm, (cw, cb, dtb, an, dsk) = _ssd_case(bsz, t, seed=11, state_scale=0.0)
    gx, gb, gc, gd = cu(x), cu(bm), cu(cm), cu(dt)
    a_cs, a_ssm = cu(cs), cu(ssm)
    ya = K.conv_ssd_scan(gx, gb, gc, gd, a_cs, cu(cw), cu(cb), a_ssm, cu(dtb), cu(an), cu(dsk))
    b_cs, b_ssm = cu(cs), cu(ssm)
    h = t // 2
    y1 = K.conv_ssd_scan(gx[:, :h].contiguous(), gb[:, :h].contiguous(), gc[:, :h].contiguous(),
                         gd[:, :h].contiguous(), b_cs, cu(cw), cu(cb), b_ssm, cu(dtb), cu(an), cu(dsk))
    y2 = K.conv_ssd_scan(gx[:, h:].contiguous(), gb[:, h:].contiguous(), gc[:, h:].contiguous(),
                         gd[:, h:].contiguous(), b_cs, cu(cw), cu(cb), b_ssm, cu(dtb), cu(an), cu(dsk))
    assert torch.equal(ya, torch.cat([y1, y2], 1))
    assert torch.equal(a_ssm, b_ssm) and torch.equal(a_cs, b_cs)
    ya_h, ssm_h = np_(ya), np_(a_ssm)
    for b in (0, 255):
        o_cs, o_ssm = cs[b:b + 1].copy(), ssm[b:b + 1].copy()
        yr = O.conv_ssd_scan(x[b:b + 1], bm[b:b + 1], cm[b:b + 1], dt[b:b + 1], o_cs, cw, cb, dtb, an, dsk, o_ssm)
        np.testing.assert_allclose(ya_h[b:b + 1], yr, atol=1e-4, rtol=1e-5)
        np.testing.assert_allclose(ssm_h[b:b + 1], o_ssm, atol=1e-4, rtol=1e-5)


# ------------------------------------------------------------- attention
@pytest.mark.parametrize("split", [0, 64, 128, 256, 512, 2048])
def test_rope_kv_attn_decode_full_size(split):
    """Config: q,k,v [64,8,1,64], positions ~U[0,2048), cache [64,8,2048,64].
    split 0 is the cluster kernel (eight CTAs per sequence and head merged in
    distributed shared memory, no scratch)."""
    q, k, v, pos, kc, vc = synth.attn_decode_inputs()
    g_kc, g_vc = cu(kc), cu(vc)
    out = K.rope_kv_attn_decode(cu(q), cu(k), cu(v), g_kc, g_vc, cu(pos), split=split)
    o_kc, o_vc = kc.copy(), vc.copy()
    ref = O.rope_kv_attn_decode(q, k, v, o_kc, o_vc, pos)
    np.testing.assert_allclose(np_(out), ref, atol=1e-4, rtol=1e-5)
    gk, gv = np_(g_kc), np_(g_vc)
    for b in range(64):
        np.testing.assert_allclose(gk[b, :, pos[b]], o_kc[b, :, pos[b]], atol=1e-5, rtol=1e-5)
        np.testing.assert_array_equal(gv[b, :, pos[b]], o_vc[b, :, pos[b]])
        np.testing.assert_array_equal(gk[b, :, : pos[b]], kc[b, :, : pos[b]])  # history untouched


@pytest.mark.parametrize("split", [0, 64, 128, 256])
@pytest.mark.parametrize("dh,ctx,posv", [(76, 16, [0, 15, 7]), (64, 300, [0, 63, 64, 299]), (76, 700, [699, 1, 256]),
                                         (64, 200, [15, 16, 17, 47, 48, 127, 128, 199]),
                                         (76, 200, [15, 16, 31, 32, 63, 64, 65, 191]),
                                         (64, 2048, [0, 1, 127, 128, 129, 1000, 2046, 2047]),
                                         (76, 1100, [1099, 511, 512, 513, 1024, 8, 136, 1087])])
def test_rope_kv_attn_decode_edges(dh, ctx, posv, split):
    """First slot, last slot, 16-key warp and split boundaries, head dim 76 (19
    float4s); for the cluster kernel (split 0) positions at the boundaries of
    its per-CTA ranges (multiples of 8 x 16 keys) and of its 16-key groups."""
    rng = np.random.default_rng(dh + ctx)
    bsz, nh = len(posv), 8
    q = rng.standard_normal((bsz, nh, dh)).astype(np.float32)
    k = rng.standard_normal((bsz, nh, dh)).astype(np.float32)
    v = rng.standard_normal((bsz, nh, dh)).astype(np.float32)
    kc = rng.standard_normal((bsz, nh, ctx, dh)).astype(np.float32)
    vc = rng.standard_normal((bsz, nh, ctx, dh)).astype(np.float32)
    pos = np.array(posv, np.int32)
    g_kc, g_vc = cu(kc), cu(vc)
    out = K.rope_kv_attn_decode(cu(q), cu(k), cu(v), g_kc, g_vc, cu(pos), split=split)
    o_kc, o_vc = kc.copy(), vc.copy()
    ref = O.rope_kv_attn_decode(q, k, v, o_kc, o_vc, pos)
    np.testing.assert_allclose(np_(out), ref, atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(np_(g_kc), o_kc, atol=1e-5, rtol=1e-5)  # appended roped k, history untouched
    np.testing.assert_array_equal(np_(g_vc), o_vc)


@pytest.mark.parametrize("dh,layout,lens,start", [
    (76, "model", [1, 17, 40], [0, 5, 100]),   # model dims: a one-row sequence, ragged blocks, nonzero starts
    (64, "bhtd", [9, 64, 3], [0, 0, 250]),     # the synthetic cache layout, a block boundary at 64 rows
    (76, "model", [300, 2], [0, 1500]),        # many 8-row blocks; a short sequence deep in its cache
])
def test_rope_kv_attn_prefill_vs_oracle(dh, layout, lens, start):
    """Prefill RoPE + KV append + causal attention (src/model.rs:486-548) through
    krk_k_rope_kv_attn_prefill, against the oracle run row by row: row i of a
    sequence is the decode step at position start + i over the keys before it
    (the reference's prefill and step attention share dot, softmax and PV
    order).  Appended K within the RoPE tolerance, V bitwise, history untouched."""
    rng = np.random.default_rng(sum(lens) + dh)
    S, H = len(lens), 8
    ctx = max(s0 + n for s0, n in zip(start, lens)) + 3
    rows = sum(lens)
    qkv = rng.standard_normal((rows, 3 * H * dh)).astype(np.float32)
    kc = rng.standard_normal((S, H, ctx, dh)).astype(np.float32)
    vc = rng.standard_normal((S, H, ctx, dh)).astype(np.float32)

    o_kc, o_vc = kc.copy(), vc.copy()
    ref = np.empty((rows, H, dh), np.float32)
    r = 0
    for s in range(S):
        for i in range(lens[s]):
            q, k, v = (a[None] for a in qkv[r].reshape(3, H, dh))
            pos = np.array([start[s] + i], np.int32)
            ref[r] = O.rope_kv_attn_decode(q, k, v, o_kc[s:s + 1], o_vc[s:s + 1], pos)[0]
            r += 1

    def to_dev(c):
        return cu(c.transpose(0, 2, 1, 3).reshape(S, ctx, H * dh)) if layout == "model" else cu(c)

    def from_dev(c):
        c = np_(c)
        return c.reshape(S, ctx, H, dh).transpose(0, 2, 1, 3) if layout == "model" else c

    g_kc, g_vc = to_dev(kc), to_dev(vc)
    out = K.rope_kv_attn_prefill(cu(qkv), g_kc, g_vc, lens, start, H, dh, cache_layout=layout)
    np.testing.assert_allclose(np_(out).reshape(rows, H, dh), ref, atol=1e-4, rtol=1e-5)
    gk, gv = from_dev(g_kc), from_dev(g_vc)
    for s in range(S):
        new = slice(start[s], start[s] + lens[s])
        np.testing.assert_allclose(gk[s, :, new], o_kc[s, :, new], atol=1e-5, rtol=1e-5)
        np.testing.assert_array_equal(gv[s, :, new], o_vc[s, :, new])
        np.testing.assert_array_equal(gk[s, :, :start[s]], kc[s, :, :start[s]])  # history untouched
        np.testing.assert_array_equal(gv[s, :, start[s] + lens[s]:], vc[s, :, start[s] + lens[s]:])


def test_rope_kv_attn_prefill_rejects_bad_tables():
    """Argument errors come back as KRK_INVALID before any launch."""
    assert K.attn_prefill_rows(100, 76) == 8 and K.attn_prefill_rows(100, 80) == 0
    qkv = torch.zeros((4, 3 * 8 * 76), device=DEV)
    kc = torch.zeros((1, 8, 16, 76), device=DEV)
    with pytest.raises(_lib.KrikilError):
        _lib.check(_lib.lib.krk_k_rope_kv_attn_prefill(qkv.data_ptr(), qkv.shape[1], kc.data_ptr(), kc.data_ptr(),
                                                       0, 0, 0, None, None, 1, 4, 8, 76, 1e4, None, 1, 1, 4,
                                                       qkv.data_ptr(), 608, 1, None))  # rows_per_block 1, not 8
    big = 100000  # one row's scores of this many keys exceed shared memory
    with pytest.raises(_lib.KrikilError):
        _lib.check(_lib.lib.krk_k_rope_kv_attn_prefill(qkv.data_ptr(), qkv.shape[1], kc.data_ptr(), kc.data_ptr(),
                                                       0, 0, 0, None, None, 1, 4, 8, 76, 1e4, None, 1,
                                                       K.attn_prefill_rows(big, 76), big, qkv.data_ptr(), 608, 1,
                                                       None))
    with pytest.raises(_lib.KrikilError):  # a cache 4 bytes off its 16-byte alignment
        _lib.check(_lib.lib.krk_k_rope_kv_attn_prefill(qkv.data_ptr(), qkv.shape[1], kc.data_ptr() + 4,
                                                       kc.data_ptr(), 0, 0, 0, None, None, 1, 4, 8, 76, 1e4, None,
                                                       1, 8, 4, qkv.data_ptr(), 608, 1, None))
    torch.cuda.synchronize()


@pytest.mark.parametrize("split,ctx", [(64, 2048), (128, 700), (256, 2048), (512, 2048), (384, 2000),
                                       (64, 64 * 65)])
def test_rope_kv_attn_decode_split_merge(split, ctx):
    """Split partials through the work buffer, up to 65 splits: the buffer
    starts as garbage and is reused across calls with other positions; every
    call must match the oracle."""
    rng = np.random.default_rng(split + ctx)
    bsz, nh, dh = 5, 3, 64
    kc = rng.standard_normal((bsz, nh, ctx, dh)).astype(np.float32)
    vc = rng.standard_normal((bsz, nh, ctx, dh)).astype(np.float32)
    g_kc, g_vc = cu(kc), cu(vc)
    work = torch.from_numpy(rng.integers(-2**31, 2**31, K.attn_work_floats(bsz, nh, dh, ctx, split),
                                         dtype=np.int64).astype(np.int32)).to(DEV).view(torch.float32)
    for call in range(3):
        q, k, v = (rng.standard_normal((bsz, nh, dh)).astype(np.float32) for _ in range(3))
        pos = np.array([ctx - 1 - call, call, ctx // 2, split - 1 + call, split + call], np.int32)
        out = K.rope_kv_attn_decode(cu(q), cu(k), cu(v), g_kc, g_vc, cu(pos), split=split, work=work)
        ref = O.rope_kv_attn_decode(q, k, v, kc, vc, pos)  # updates kc / vc like the device call
        np.testing.assert_allclose(np_(out), ref, atol=1e-4, rtol=1e-5)


def test_copy_wait_timeout_sets_status_and_context_survives():
    """The bounded wait of the attention's K/V copies, made to run out on a
    barrier whose copy is never issued: the kernel returns, the status word has
    bit 0 set, and the context keeps working (the same wait with its copy
    issued succeeds, and an attention call afterwards matches the oracle)."""
    src = torch.arange(4, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.wait_probe(src, status, polls=256, copy=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    K.wait_probe(None, status, polls=256, copy=False)
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    status.zero_()
    K.wait_probe(src, status, polls=256, copy=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    from krikil_rs_b200._lib import KrikilError
    with pytest.raises(KrikilError):
        K.wait_probe(src[1:], status, polls=256, copy=True)  # not 16-byte aligned: refused before launch
    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal((2, 2, 64)).astype(np.float32) for _ in range(3))
    kc, vc = (rng.standard_normal((2, 2, 128, 64)).astype(np.float32) for _ in range(2))
    pos = np.array([5, 127], np.int32)
    out = K.rope_kv_attn_decode(cu(q), cu(k), cu(v), cu(kc), cu(vc), cu(pos), split=64)
    np.testing.assert_allclose(np_(out), O.rope_kv_attn_decode(q, k, v, kc.copy(), vc.copy(), pos), atol=1e-4,
                               rtol=1e-5)


# ------------------------------------------------------------- sampling
@pytest.mark.parametrize("temp,top_p,top_k,pen",[(0.7, 0.95, 50, 1.2), (1.0, 1.0, 0, 1.0), (0.5, 0.5, 0, 1.0),
                                                  (1.3, 0.9, 5, 1.5), (2.0, 1.0, 2048, 1.0)])
def test_stochastic_sample_matches_oracle(temp, top_p, top_k, pen):
    """krk_k_sample against the oracle's Sampler::sample restatement: 6 rows, 40
    picks each from the rows' own seeded streams (crossing ChaCha block
    boundaries), the picks fed back into the penalty set."""
    rng_np = np.random.default_rng(21)
    B, V = 6, 2048
    lg = (rng_np.standard_normal((B, V)) * 3).astype(np.float32)
    ctx = [list(rng_np.integers(0, V, 20)) for _ in range(B)]
    seen = np.zeros((B, V // 32), np.uint32)
    for b in range(B):
        for t in ctx[b]:
            seen[b, t >> 5] |= np.uint32(1 << (t & 31))
    seeds = [3, 99, 2**40 + 7, 0, 12345, 2**63]
    orng = [O.Rng(s_) for s_ in seeds]
    st = np.stack([O.Rng(s_).state for s_ in seeds]).astype(np.uint32)
    g_lg, g_seen, g_st = cu(lg), torch.from_numpy(seen.view(np.int32)).to("cuda"), torch.from_numpy(st.view(np.int32)).to("cuda")
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    for it in range(40):
        rc = _lib.lib.krk_k_sample(g_lg.data_ptr(), V, V, B, g_seen.data_ptr(), temp, top_p, top_k, pen,
                                   g_st.data_ptr(), tok.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.OK
        got = np_(tok).view(np.uint32).tolist()
        for b in range(B):
            want = O.sample(lg[b], ctx[b], temp, top_p, top_k, pen, orng[b])
            assert got[b] == want, (it, b, got[b], want)
            ctx[b].append(want)
    np.testing.assert_array_equal(np_(g_st).view(np.uint32), np.stack([r.state for r in orng]))

def test_greedy_matches_sampler():
    rng = np.random.default_rng(6)
    lg = rng.standard_normal((5, 2048)).astype(np.float32)
    lg[1, 100] = lg[1, 700] = 50.0  # tie: the lower index wins
    lg[2, :] = np.nan
    lg[2, 3] = 1.0
    lg[3, :] = -np.inf
    tok = np_(K.greedy(cu(lg)))
    assert [int(t) for t in tok] == [O.sample_greedy(lg[i], []) for i in range(5)]
    assert tok[1] == 100 and tok[3] == 0
    seen = np.zeros((5, 64), np.uint32)
    ctx = [[int(np.argmax(lg[0]))], [100, 5], [], [1], list(range(0, 2048, 3))]
    for b, c in enumerate(ctx):
        for t in c:
            seen[b, t // 32] |= np.uint32(1 << (t % 32))
    tok = np_(K.greedy(cu(lg), cu(seen.view(np.int32)), 1.2))
    assert [int(t) for t in tok] == [O.sample_greedy(lg[i], ctx[i], 1.2) for i in range(5)]
