"""Per-kernel entry points of the C ABI on torch CUDA tensors.

torch only provides device memory and the current stream here; every op is one
of this library's sm_100a kernels (krk_k_* in include/krikil_cuda.h).
"""
from __future__ import annotations

import itertools
from typing import Optional

import torch

from ._lib import check, lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _f32(*ts):
    for t in ts:
        if t is None:
            continue
        if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
            raise ValueError("expected contiguous float32 CUDA tensors")


def rmsnorm_rows(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _f32(x, w)
    y = torch.empty_like(x)
    check(lib.krk_k_rmsnorm_rows(x.data_ptr(), w.data_ptr(), eps, x.shape[0], x.shape[1], y.data_ptr(), _stream()))
    return y


def rmsnorm_fm(x_t: torch.Tensor, w: torch.Tensor, eps: float, m: Optional[int] = None) -> torch.Tensor:
    """x_t: feature-major [K, ld]; normalises columns 0..m-1."""
    _f32(x_t, w)
    k, ld = x_t.shape
    out = torch.zeros_like(x_t)
    check(lib.krk_k_rmsnorm_fm(x_t.data_ptr(), ld, w.data_ptr(), eps, k, m or ld, out.data_ptr(), ld, _stream()))
    return out


def gated_rmsnorm_residual(x, z, res, w, eps: float, y=None) -> torch.Tensor:
    _f32(x, z, res, w, y)
    if y is None:
        y = torch.empty_like(x)
    check(lib.krk_k_gated_rmsnorm_residual(x.data_ptr(), z.data_ptr(), res.data_ptr(), w.data_ptr(), eps,
                                           x.shape[0], x.shape[1], y.data_ptr(), _stream()))
    return y


def gemm(a_t: torch.Tensor, w_t: torch.Tensor, epilogue: int = 0, out_fm: bool = False,
         c: Optional[torch.Tensor] = None, tile_rows: int = 0) -> torch.Tensor:
    """C = A . W^T with a_t = A^T [K, M] and w_t = W^T [K, N]; tile_rows 0/16/32/64."""
    _f32(a_t, w_t, c)
    k, m = a_t.shape
    k2, n = w_t.shape
    assert k == k2
    if c is None:
        c = torch.empty((n, m) if out_fm else (m, n), device=a_t.device, dtype=torch.float32)
    check(lib.krk_k_gemm_tiled(a_t.data_ptr(), m, w_t.data_ptr(), n, c.data_ptr(), c.shape[1], m, n, k, epilogue,
                               int(out_fm), tile_rows, _stream()))
    return c


def embed(tok: torch.Tensor, wte: torch.Tensor, ld: Optional[int] = None) -> torch.Tensor:
    _f32(wte)
    vocab, k = wte.shape
    m = tok.numel()
    out = torch.zeros((k, ld or m), device=wte.device, dtype=torch.float32)
    check(lib.krk_k_embed(tok.data_ptr(), wte.data_ptr(), vocab, k, m, out.data_ptr(), out.shape[1], _stream()))
    return out


def pointwise(op: int, x: torch.Tensor) -> torch.Tensor:
    _f32(x)
    y = torch.empty_like(x)
    check(lib.krk_k_pointwise(op, x.data_ptr(), y.data_ptr(), x.numel(), _stream()))
    return y


def conv_ssd_step(x, bm, cm, dt, conv_state, conv_w, conv_b, ssm, dt_bias, a_neg, dsk, y=None) -> torch.Tensor:
    """x [B,H*P], bm/cm [B,N], dt [B,H]; conv_state [B,H*P,3] and ssm [B,H,P,N]
    updated in place; returns y [B,H*P]."""
    _f32(x, bm, cm, dt, conv_state, conv_w, conv_b, ssm, dt_bias, a_neg, dsk, y)
    b, h, p, n = ssm.shape
    if y is None:
        y = torch.empty((b, h * p), device=x.device, dtype=torch.float32)
    check(lib.krk_k_conv_ssd_step(x.data_ptr(), bm.data_ptr(), cm.data_ptr(), dt.data_ptr(), conv_state.data_ptr(),
                                  conv_w.data_ptr(), conv_b.data_ptr(), ssm.data_ptr(), dt_bias.data_ptr(),
                                  a_neg.data_ptr(), dsk.data_ptr(), y.data_ptr(), b, h, p, n, _stream()))
    return y


def conv_ssd_scan(x, bm, cm, dt, conv_state, conv_w, conv_b, ssm, dt_bias, a_neg, dsk, y=None) -> torch.Tensor:
    """x [B,T,H*P], bm/cm [B,T,N], dt [B,T,H]; states updated in place; y [B,T,H*P]."""
    _f32(x, bm, cm, dt, conv_state, conv_w, conv_b, ssm, dt_bias, a_neg, dsk, y)
    b, h, p, n = ssm.shape
    t = x.shape[1]
    if y is None:
        y = torch.empty((b, t, h * p), device=x.device, dtype=torch.float32)
    check(lib.krk_k_conv_ssd_scan(x.data_ptr(), bm.data_ptr(), cm.data_ptr(), dt.data_ptr(), conv_state.data_ptr(),
                                  conv_w.data_ptr(), conv_b.data_ptr(), ssm.data_ptr(), dt_bias.data_ptr(),
                                  a_neg.data_ptr(), dsk.data_ptr(), y.data_ptr(), b, t, h, p, n, _stream()))
    return y


def attn_work_floats(b: int, h: int, dh: int, ctx: int, split: int = 0) -> int:
    return int(lib.krk_attn_work_floats(b, h, dh, ctx, split))


def wait_probe(src16, status, polls: int, copy: bool) -> None:
    """krk_k_wait_probe: the bounded copy wait with (copy) or without its copy;
    bit 0 of status (int32, device) is set when the wait runs out."""
    check(lib.krk_k_wait_probe(src16.data_ptr() if src16 is not None else None, polls, int(copy),
                               status.data_ptr(), _stream()))


def rope_kv_attn_decode(q, k, v, kc, vc, pos, split: int = 0, theta: float = 10000.0, work=None, out=None):
    """q,k,v [B,H,dh]; kc,vc [B,H,ctx,dh] (updated at pos); pos int32 [B].
    split 0: the cluster kernel (no scratch); split > 0: splits of that many
    keys merged through `work` (allocated here when not given)."""
    _f32(q, k, v, kc, vc, work, out)
    b, h, dh = q.shape
    ctx = kc.shape[2]
    if out is None:
        out = torch.empty_like(q)
    if work is None:
        work = torch.empty(max(1, attn_work_floats(b, h, dh, ctx, split)), device=q.device, dtype=torch.float32)
    check(lib.krk_k_rope_kv_attn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                        pos.data_ptr(), out.data_ptr(), work.data_ptr(), b, h, dh, ctx, split, theta,
                                        _stream()))
    return out


def gemm_sgemm_order(a_t: torch.Tensor, w_t: torch.Tensor) -> torch.Tensor:
    """C = A . W^T (a_t = A^T [K, M], w_t = W^T [K, N]) summed in the order of
    matrixmultiply's sgemm (the reference's prefill GEMM)."""
    _f32(a_t, w_t)
    k, m = a_t.shape
    k2, n = w_t.shape
    assert k == k2
    c = torch.empty((m, n), device=a_t.device, dtype=torch.float32)
    check(lib.krk_k_gemm_sgemm_order(a_t.data_ptr(), m, w_t.data_ptr(), n, c.data_ptr(), n, m, n, k, _stream()))
    return c


def attn_prefill_rows(kmax: int, dh: int) -> int:
    return int(lib.krk_k_attn_prefill_rows(kmax, dh))


def rope_kv_attn_prefill(qkv, kc, vc, lens, start, H: int, dh: int, theta: float = 10000.0,
                         cache_layout: str = "model"):
    """Packed prefill rows of len(lens) sequences: qkv [rows, 3*H*dh] (q rotated
    in place), sequence s starting at position start[s] of its cache.  Caches:
    "model" [S, ctx, H*dh] (the model's layout) or "bhtd" [S, H, ctx, dh].
    Builds the row-block table as the model does and returns out [rows, H*dh]."""
    _f32(qkv, kc, vc)
    lens = [int(x) for x in lens]
    start = [int(x) for x in start]
    S, rows = len(lens), sum(lens)
    if cache_layout == "model":
        ctx = kc.shape[1]
        c_sb, c_sh, c_st = ctx * H * dh, dh, H * dh
    else:
        ctx = kc.shape[2]
        c_sb, c_sh, c_st = H * ctx * dh, ctx * dh, dh
    kmax = max(s0 + n for s0, n in zip(start, lens))
    rpb = attn_prefill_rows(kmax, dh)
    blocks = [(s, r0) for s in range(S) for r0 in range(0, lens[s], rpb)]
    dev = qkv.device
    cu = torch.tensor([0] + list(itertools.accumulate(lens)), dtype=torch.int32, device=dev)
    st = torch.tensor(start, dtype=torch.int32, device=dev)
    blk = torch.tensor(blocks, dtype=torch.int32, device=dev).reshape(-1)
    out = torch.zeros((rows, H * dh), device=dev, dtype=torch.float32)
    check(lib.krk_k_rope_kv_attn_prefill(qkv.data_ptr(), qkv.shape[1], kc.data_ptr(), vc.data_ptr(), c_sb, c_sh,
                                         c_st, cu.data_ptr(), st.data_ptr(), S, rows, H, dh, theta, blk.data_ptr(),
                                         len(blocks), rpb, kmax, out.data_ptr(), H * dh, 1, _stream()))
    return out


def greedy(logits: torch.Tensor, seen: Optional[torch.Tensor] = None, penalty: float = 1.0) -> torch.Tensor:
    _f32(logits)
    b, v = logits.shape
    tok = torch.empty(b, device=logits.device, dtype=torch.int32)
    check(lib.krk_k_greedy(logits.data_ptr(), v, v, b, seen.data_ptr() if seen is not None else None, penalty,
                           tok.data_ptr(), _stream()))
    return tok
