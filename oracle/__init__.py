"""ctypes front-end of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
package, and only as the checker; the CUDA library never calls it.  The C source
(krikil_oracle.c) restates src/math.rs, src/model.rs and src/sampler.rs of
krikil-rs; see its header for what is and is not pinned.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os
import subprocess
from typing import Dict, List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

HIDDEN, VOCAB, INTER, NLAYERS = 608, 2048, 2432, 8
DXBC, DCONV, MHEADS, MHDIM, DSTATE = 1472, 4, 19, 64, 128
OK, BAD_TOKEN, CONTEXT_OVERFLOW, EMPTY = 0, 1, 2, 3


def build() -> str:
    src = os.path.join(_HERE, "krikil_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    if not os.path.exists(_LIB_PATH):
        build()
    return C.CDLL(_LIB_PATH)


lib = _load()
_fp = C.POINTER(C.c_float)
_u32p = C.POINTER(C.c_uint32)
_i32p = C.POINTER(C.c_int32)


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_fp)


for _name in ("orc_silu", "orc_softplus", "orc_gelu"):
    getattr(lib, _name).restype = C.c_float
    getattr(lib, _name).argtypes = [C.c_float]
lib.orc_dot.restype = C.c_float
lib.orc_dot.argtypes = [_fp, _fp, C.c_int]
lib.orc_rms_norm.argtypes = [_fp, _fp, C.c_float, _fp, C.c_int]
lib.orc_rms_norm_inplace.argtypes = [_fp, _fp, C.c_float, C.c_int]
lib.orc_gemv.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int]
lib.orc_gemm_transb.argtypes = [_fp, _fp, _fp, C.c_int, C.c_int, C.c_int]
lib.orc_set_prefill_gemm_order.argtypes = [C.c_int]
lib.orc_prefill_gemm_order.restype = C.c_int
lib.orc_softmax_inplace.argtypes = [_fp, C.c_int]
lib.orc_apply_rope.argtypes = [_fp, _fp, C.c_int, C.c_int, C.c_int, C.c_float]
lib.orc_precompute_a.argtypes = [_fp, _fp, C.c_int]
lib.orc_sample_greedy.restype = C.c_uint32
lib.orc_sample_greedy.argtypes = [_fp, C.c_int, _u32p, C.c_int, C.c_float, _fp]
lib.orc_gated_rmsnorm_residual.argtypes = [_fp, _fp, _fp, _fp, C.c_float, _fp, C.c_int64, C.c_int]
lib.orc_rms_norm_rows.argtypes = [_fp, _fp, C.c_float, _fp, C.c_int64, C.c_int]
lib.orc_rope_kv_attn_decode.argtypes = [_fp, _fp, _fp, _fp, _fp, _i32p, _fp] + [C.c_int] * 4 + [C.c_float]
lib.orc_conv_ssd_step.argtypes = [_fp] * 12 + [C.c_int] * 4
lib.orc_conv_ssd_scan.argtypes = [_fp] * 12 + [C.c_int] * 5
lib.orc_chacha_block.argtypes = [_u32p, C.c_int, _u32p]
lib.orc_rng_seed.argtypes = [C.c_uint64, _u32p]
lib.orc_rng_next_u32.restype = C.c_uint32
lib.orc_rng_next_u32.argtypes = [_u32p]
lib.orc_rng_f32.restype = C.c_float
lib.orc_rng_f32.argtypes = [_u32p]
lib.orc_sample.restype = C.c_uint32
lib.orc_sample.argtypes = [_fp, C.c_int, _u32p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, _u32p]
lib.orc_num_threads.restype = C.c_int
lib.orc_set_num_threads.argtypes = [C.c_int]


class _Layer(C.Structure):
    _fields_ = [(n, _fp) for n in (
        "ln_w", "in_proj_w", "conv1d_w", "conv1d_b", "dt_bias", "a_neg_exp", "d", "norm_w", "out_proj_w",
        "ln1_w", "wqkv_w", "wo_w", "ln2_w", "fc1_w", "fc2_w")]


class _Model(C.Structure):
    _fields_ = [("wte", _fp), ("lnf_w", _fp), ("layers", _Layer * NLAYERS)]


class _State(C.Structure):
    _fields_ = [("conv", _fp * NLAYERS), ("ssm", _fp * NLAYERS), ("kc", _fp * NLAYERS), ("vc", _fp * NLAYERS),
                ("cur_len", C.c_int64 * NLAYERS), ("context_limit", C.c_int64), ("current_pos", C.c_int64)]


lib.orc_forward_prefill.restype = C.c_int
lib.orc_forward_prefill.argtypes = [C.POINTER(_Model), C.POINTER(_State), _u32p, C.c_int, _fp]
lib.orc_forward_step.restype = C.c_int
lib.orc_forward_step.argtypes = [C.POINTER(_Model), C.POINTER(_State), C.c_uint32, _fp]
lib.orc_state_reset.argtypes = [C.POINTER(_State)]


# ----------------------------------------------------------------- primitives
def silu(x: float) -> float: return lib.orc_silu(x)
def softplus(x: float) -> float: return lib.orc_softplus(x)
def gelu(x: float) -> float: return lib.orc_gelu(x)


def dot(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a, np.float32); b = np.ascontiguousarray(b, np.float32)
    return lib.orc_dot(_p(a), _p(b), a.size)


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib.orc_rms_norm(_p(x), _p(w), eps, _p(out), x.size)
    return out


def rms_norm_rows(x, w, eps):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib.orc_rms_norm_rows(_p(x), _p(w), eps, _p(out), x.shape[0], x.shape[1])
    return out


def gemv(w, x):
    w = np.ascontiguousarray(w, np.float32); x = np.ascontiguousarray(x, np.float32)
    out = np.empty(w.shape[0], np.float32)
    lib.orc_gemv(_p(w), _p(x), _p(out), w.shape[0], w.shape[1])
    return out


def gemm_transb(a, b):
    a = np.ascontiguousarray(a, np.float32); b = np.ascontiguousarray(b, np.float32)
    out = np.empty((a.shape[0], b.shape[0]), np.float32)
    lib.orc_gemm_transb(_p(a), _p(b), _p(out), a.shape[0], a.shape[1], b.shape[0])
    return out


PREFILL_GEMM_ORDERS = {"dot": 0, "matrixmultiply": 1}


@contextlib.contextmanager
def prefill_gemm_order(order: str):
    """Run the block with the prefill projections (gemm_transb,
    src/math.rs:188-211) summed in ``order``: "dot" is the gemv dot order of
    src/math.rs:70-124 (the default, and the CUDA projections' order);
    "matrixmultiply" is the restated order of matrixmultiply 0.3.11's sgemm,
    the crate the reference calls there (256-long K blocks, one FMA
    accumulator per element within a block, blocks added in order)."""
    old = lib.orc_prefill_gemm_order()
    lib.orc_set_prefill_gemm_order(PREFILL_GEMM_ORDERS[order])
    try:
        yield
    finally:
        lib.orc_set_prefill_gemm_order(old)


def softmax(x):
    x = np.array(x, np.float32)
    lib.orc_softmax_inplace(_p(x), x.size)
    return x


def apply_rope(q, k, pos, nh, hd, theta=10000.0):
    q = np.array(q, np.float32); k = np.array(k, np.float32)
    lib.orc_apply_rope(_p(q), _p(k), pos, nh, hd, theta)
    return q, k


def sample_greedy(logits, context: Sequence[int], penalty: float = 1.0) -> int:
    lg = np.ascontiguousarray(logits, np.float32)
    ctx = np.ascontiguousarray(np.array(context, dtype=np.uint32))
    scratch = np.empty_like(lg)
    return int(lib.orc_sample_greedy(_p(lg), lg.size, ctx.ctypes.data_as(_u32p), ctx.size, penalty, _p(scratch)))


# ------------------------------------------------------- stochastic sampling
def chacha_block(words: Sequence[int], rounds: int) -> List[int]:
    """The ChaCha block function on 16 input words (test hook)."""
    inp = np.ascontiguousarray(np.array(words, dtype=np.uint32))
    out = np.empty(16, np.uint32)
    lib.orc_chacha_block(inp.ctypes.data_as(_u32p), rounds, out.ctypes.data_as(_u32p))
    return out.tolist()


class Rng:
    """StdRng::seed_from_u64(seed) restated (see krikil_oracle.c): ten u32 words,
    the ChaCha12 key and the index of the next keystream word."""

    def __init__(self, seed: int):
        self.state = np.zeros(10, np.uint32)
        lib.orc_rng_seed(seed & 0xFFFFFFFFFFFFFFFF, self.state.ctypes.data_as(_u32p))

    def next_u32(self) -> int:
        return int(lib.orc_rng_next_u32(self.state.ctypes.data_as(_u32p)))

    def gen_f32(self) -> float:
        return float(lib.orc_rng_f32(self.state.ctypes.data_as(_u32p)))


def sample(logits, context: Sequence[int], temperature: float, top_p: float, top_k: int, penalty: float,
           rng: Rng) -> int:
    """Sampler::sample (src/sampler.rs:43-152); temperature <= 1e-6 is the greedy branch."""
    if temperature <= 1e-6:
        return sample_greedy(logits, context, penalty)
    lg = np.ascontiguousarray(logits, np.float32)
    ctx = np.ascontiguousarray(np.array(context, dtype=np.uint32))
    return int(lib.orc_sample(_p(lg), lg.size, ctx.ctypes.data_as(_u32p), ctx.size, temperature, top_p, top_k,
                              penalty, rng.state.ctypes.data_as(_u32p)))


# ------------------------------------------------------- synthetic layer ops
def gated_rmsnorm_residual(x, z, res, w, eps):
    y = np.empty_like(x)
    lib.orc_gated_rmsnorm_residual(_p(x), _p(z), _p(res), _p(w), eps, _p(y), x.shape[0], x.shape[1])
    return y


def rope_kv_attn_decode(q, k, v, kc, vc, pos, theta=10000.0):
    """Updates kc, vc in place; returns out [B,H,Dh]."""
    bsz, nh, dh = q.shape
    out = np.empty_like(q)
    pos = np.ascontiguousarray(pos, np.int32)
    lib.orc_rope_kv_attn_decode(_p(q), _p(k), _p(v), _p(kc), _p(vc), pos.ctypes.data_as(_i32p), _p(out),
                                bsz, nh, dh, kc.shape[2], theta)
    return out


def conv_ssd_step(x, bm, cm, dt, conv_state, conv_w, conv_b, dt_bias, a_neg, dsk, ssm):
    """x [B,nh*p], bm/cm [B,n], dt [B,nh]; conv_state [B,nh*p,3] and ssm [B,nh,p,n]
    are updated in place; returns y [B,nh*p]."""
    bsz, nh, p, n = ssm.shape
    y = np.empty((bsz, nh * p), np.float32)
    lib.orc_conv_ssd_step(_p(x), _p(bm), _p(cm), _p(dt), _p(conv_state), _p(conv_w), _p(conv_b), _p(dt_bias),
                          _p(a_neg), _p(dsk), _p(ssm), _p(y), bsz, nh, p, n)
    return y


def conv_ssd_scan(x, bm, cm, dt, conv_state, conv_w, conv_b, dt_bias, a_neg, dsk, ssm):
    """x [B,T,nh*p] ...; states updated in place; returns y [B,T,nh*p]."""
    bsz, nh, p, n = ssm.shape
    t = x.shape[1]
    y = np.empty((bsz, t, nh * p), np.float32)
    lib.orc_conv_ssd_scan(_p(x), _p(bm), _p(cm), _p(dt), _p(conv_state), _p(conv_w), _p(conv_b), _p(dt_bias),
                          _p(a_neg), _p(dsk), _p(ssm), _p(y), bsz, t, nh, p, n)
    return y


# ---------------------------------------------------------------- full model
class OracleModel:
    """Mirror of ``PebbleModel`` (src/model.rs:112-117) over a weights dict."""

    def __init__(self, weights: Dict[str, np.ndarray]):
        self._keep: List[np.ndarray] = []
        self.s = _Model()

        def ptr(name):
            a = np.ascontiguousarray(weights[name], np.float32)
            self._keep.append(a)
            return _p(a)

        self.s.wte = ptr("wte.weight")
        self.s.lnf_w = ptr("lnf.weight")
        for i in range(NLAYERS):
            L = self.s.layers[i]
            p = f"blocks.{i}."
            if i % 4 < 3:
                for f, n in (("ln_w", "ln.weight"), ("in_proj_w", "mixer.in_proj.weight"),
                             ("conv1d_w", "mixer.conv1d.weight"), ("conv1d_b", "mixer.conv1d.bias"),
                             ("dt_bias", "mixer.dt_bias"), ("d", "mixer.D"), ("norm_w", "mixer.norm.weight"),
                             ("out_proj_w", "mixer.out_proj.weight")):
                    setattr(L, f, ptr(p + n))
                alog = np.ascontiguousarray(weights[p + "mixer.A_log"], np.float32)
                aneg = np.empty_like(alog)
                lib.orc_precompute_a(_p(alog), _p(aneg), alog.size)
                self._keep += [alog, aneg]
                L.a_neg_exp = _p(aneg)
            else:
                for f, n in (("ln1_w", "ln1.weight"), ("wqkv_w", "wqkv.weight"), ("wo_w", "wo.weight"),
                             ("ln2_w", "ln2.weight"), ("fc1_w", "fc1.weight"), ("fc2_w", "fc2.weight")):
                    setattr(L, f, ptr(p + n))


class OracleState:
    """Mirror of ``PebbleState`` (src/model.rs:196-230)."""

    def __init__(self, max_ctx: int = 2048):
        self.s = _State()
        self.conv, self.ssm, self.kc, self.vc = {}, {}, {}, {}
        for i in range(NLAYERS):
            if i % 4 < 3:
                self.conv[i] = np.zeros((DXBC, DCONV), np.float32)
                self.ssm[i] = np.zeros((MHEADS, MHDIM, DSTATE), np.float32)
                self.s.conv[i] = _p(self.conv[i]); self.s.ssm[i] = _p(self.ssm[i])
            else:
                self.kc[i] = np.zeros((max_ctx, HIDDEN), np.float32)
                self.vc[i] = np.zeros((max_ctx, HIDDEN), np.float32)
                self.s.kc[i] = _p(self.kc[i]); self.s.vc[i] = _p(self.vc[i])
        self.s.context_limit = max_ctx
        self.s.current_pos = 0

    @property
    def current_pos(self) -> int: return self.s.current_pos

    @property
    def context_limit(self) -> int: return self.s.context_limit

    def cur_len(self, layer: int) -> int: return self.s.cur_len[layer]

    def reset(self): lib.orc_state_reset(C.byref(self.s))


class OracleError(RuntimeError):
    def __init__(self, code: int):
        super().__init__({BAD_TOKEN: "token id exceeds vocab size", CONTEXT_OVERFLOW: "context limit exceeded",
                          EMPTY: "cannot prefill empty sequence"}.get(code, f"status {code}"))
        self.code = code


def forward_prefill(model: OracleModel, state: OracleState, tokens) -> np.ndarray:
    toks = np.ascontiguousarray(np.array(tokens, dtype=np.uint32))
    logits = np.empty(VOCAB, np.float32)
    rc = lib.orc_forward_prefill(C.byref(model.s), C.byref(state.s), toks.ctypes.data_as(_u32p), toks.size,
                                 _p(logits))
    if rc:
        raise OracleError(rc)
    return logits


def forward_step(model: OracleModel, state: OracleState, token: int) -> np.ndarray:
    logits = np.empty(VOCAB, np.float32)
    rc = lib.orc_forward_step(C.byref(model.s), C.byref(state.s), int(token) & 0xFFFFFFFF, _p(logits))
    if rc:
        raise OracleError(rc)
    return logits


def generate_sample(model: OracleModel, state: OracleState, prompt, max_new_tokens: int, temperature: float,
                    top_p: float, top_k: int, repetition_penalty: float, seed: int, eos: Optional[int] = 0):
    """GenerationEngine::generate_with_callback (src/generate.rs:65-114) with a
    Sampler seeded by `seed` (src/sampler.rs:35-40).  ``eos=None`` ignores EOS."""
    state.reset()
    rng = Rng(seed)
    all_tokens = [int(t) for t in prompt]
    lg = forward_prefill(model, state, prompt)
    nxt = sample(lg, all_tokens, temperature, top_p, top_k, repetition_penalty, rng)
    out = []
    while len(out) < max_new_tokens:
        if eos is not None and nxt == eos:
            break
        out.append(nxt)
        all_tokens.append(nxt)
        if state.current_pos >= state.context_limit:
            break
        lg = forward_step(model, state, nxt)
        nxt = sample(lg, all_tokens, temperature, top_p, top_k, repetition_penalty, rng)
    return out


def generate_greedy(model: OracleModel, state: OracleState, prompt, max_new_tokens: int,
                    repetition_penalty: float = 1.0, eos: Optional[int] = 0, keep_logits: bool = False):
    """The greedy branch of GenerationEngine::generate_with_callback
    (src/generate.rs:65-114): reset, prefill, sample, then step/sample per token.
    ``eos=None`` ignores EOS (benchmark mode).  Returns (tokens, [logits...])."""
    state.reset()
    all_tokens = [int(t) for t in prompt]
    lg = forward_prefill(model, state, prompt)
    logits = [lg] if keep_logits else []
    nxt = sample_greedy(lg, all_tokens, repetition_penalty)
    out = []
    while len(out) < max_new_tokens:
        if eos is not None and nxt == eos:
            break
        out.append(nxt)
        all_tokens.append(nxt)
        if state.current_pos >= state.context_limit:
            break
        lg = forward_step(model, state, nxt)
        if keep_logits:
            logits.append(lg)
        nxt = sample_greedy(lg, all_tokens, repetition_penalty)
    return out, logits
