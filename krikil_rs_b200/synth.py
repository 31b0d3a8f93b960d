"""Seeded synthetic weights and inputs for the Pebble-25M architecture.

The real Pebble-25M checkpoint is not distributed with krikil-rs, so every test
and benchmark runs on random-init weights with the checkpoint's tensor names and
shapes (the names are the ones ``PebbleModel::load_safetensors`` reads,
src/model.rs:256-294; the dims are those of config.json / src/model.rs:12-30).

Initialisation (seeded ``numpy.random.default_rng(seed)``, tensors drawn in the
order of ``tensor_specs()``):
  * linear and embedding weights ~ N(0, 0.02)
  * norm weights (ln, ln1, ln2, lnf, mixer.norm) = 1
  * A_log ~ U(0, ln 16);  dt_bias ~ N(0, 0.1)
  * D = 1;  conv1d.weight ~ N(0, 0.02) stored [1472, 1, 4];  conv1d.bias = 0
``perturb=True`` draws the constant tensors instead (norm weights ~ N(1, 0.1),
D ~ N(1, 0.1), conv bias ~ N(0, 0.1)) so that tests see every weight used.

The safetensors reader/writer here is a minimal implementation of the format
(8-byte little-endian header length, JSON header, raw little-endian data).
"""
from __future__ import annotations

import json
import math
import os
import struct
import tempfile
from typing import Dict, List, Tuple

import numpy as np

# config.json of the reference (dims are also hard-coded at src/model.rs:12-30)
CONFIG = {
    "vocab_size": 2048,
    "hidden_size": 608,
    "intermediate_size": 2432,
    "num_hidden_layers": 8,
    "num_attention_heads": 8,
    "rope_theta": 10000.0,
    "rms_norm_eps": 1e-6,
    "max_position_embeddings": 2048,
    "block_pattern": "mmma|mmma",
    "mamba2": {"d_conv": 4, "d_state": 128, "expand": 2, "headdim": 64},
}

HIDDEN = 608
VOCAB = 2048
INTER = 2432
NLAYERS = 8
NHEADS = 8
HDIM = 76
DSTATE = 128
DCONV = 4
DINNER = 1216
MHDIM = 64
MHEADS = 19
DINPROJ = 2707
DXBC = 1472
EOS_TOKEN = 0


def is_mamba(layer: int) -> bool:
    """Layer i is Mamba2 if i % 4 < 3, else attention (src/model.rs:207, :261)."""
    return layer % 4 < 3


def tensor_specs() -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape, init) in load order (src/model.rs:256-294)."""
    specs = [("wte.weight", (VOCAB, HIDDEN), "normal02"), ("lnf.weight", (HIDDEN,), "ones")]
    for i in range(NLAYERS):
        p = f"blocks.{i}."
        if is_mamba(i):
            specs += [
                (p + "ln.weight", (HIDDEN,), "ones"),
                (p + "mixer.in_proj.weight", (DINPROJ, HIDDEN), "normal02"),
                (p + "mixer.conv1d.weight", (DXBC, 1, DCONV), "normal02"),
                (p + "mixer.conv1d.bias", (DXBC,), "zeros"),
                (p + "mixer.dt_bias", (MHEADS,), "dt_bias"),
                (p + "mixer.A_log", (MHEADS,), "a_log"),
                (p + "mixer.D", (MHEADS,), "ones"),
                (p + "mixer.norm.weight", (DINNER,), "ones"),
                (p + "mixer.out_proj.weight", (HIDDEN, DINNER), "normal02"),
            ]
        else:
            specs += [
                (p + "ln1.weight", (HIDDEN,), "ones"),
                (p + "wqkv.weight", (3 * HIDDEN, HIDDEN), "normal02"),
                (p + "wo.weight", (HIDDEN, HIDDEN), "normal02"),
                (p + "ln2.weight", (HIDDEN,), "ones"),
                (p + "fc1.weight", (INTER, HIDDEN), "normal02"),
                (p + "fc2.weight", (HIDDEN, INTER), "normal02"),
            ]
    return specs


def make_weights(seed: int = 0, perturb: bool = False) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out: Dict[str, np.ndarray] = {}
    for name, shape, init in tensor_specs():
        if init == "normal02":
            a = rng.normal(0.0, 0.02, shape)
        elif init == "a_log":
            a = rng.uniform(0.0, math.log(16.0), shape)
        elif init == "dt_bias":
            a = rng.normal(0.0, 0.1, shape)
        elif init == "ones":
            a = rng.normal(1.0, 0.1, shape) if perturb else np.ones(shape)
        elif init == "zeros":
            a = rng.normal(0.0, 0.1, shape) if perturb else np.zeros(shape)
        else:  # pragma: no cover
            raise ValueError(init)
        out[name] = np.ascontiguousarray(a, dtype=np.float32)
    return out


def save_safetensors(path: str, tensors: Dict[str, np.ndarray]) -> None:
    header = {}
    off = 0
    blobs = []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr, dtype="<f4")
        n = arr.nbytes
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + n]}
        blobs.append(arr.tobytes())
        off += n
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


def load_safetensors(path: str) -> Dict[str, np.ndarray]:
    with open(path, "rb") as f:
        buf = f.read()
    (hlen,) = struct.unpack("<Q", buf[:8])
    header = json.loads(buf[8 : 8 + hlen])
    base = 8 + hlen
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        out[name] = np.frombuffer(buf[base + a : base + b], dtype="<f4").reshape(meta["shape"]).copy()
    return out


def weights_file(seed: int = 0, perturb: bool = False, directory: str | None = None) -> str:
    """Write (once) and return the path of a seeded synthetic checkpoint."""
    directory = directory or os.environ.get("KRIKIL_SYNTH_DIR") or os.path.join(
        tempfile.gettempdir(), "krikil_synth")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"pebble25m_seed{seed}{'_perturbed' if perturb else ''}.safetensors")
    if not os.path.exists(path):
        save_safetensors(path, make_weights(seed, perturb))
    return path


# ---------------------------------------------------------------------------
# Synthetic inputs of the per-kernel benchmark shapes
# ---------------------------------------------------------------------------

def fused_norm_inputs(rows: int = 16384, dim: int = 512, seed: int = 0):
    """x, z, res ~ N(0,1) [rows, dim]; w ~ N(1, 0.1) [dim]; eps 1e-5."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, dim), dtype=np.float32)
    z = rng.standard_normal((rows, dim), dtype=np.float32)
    res = rng.standard_normal((rows, dim), dtype=np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    return x, z, res, w


def attn_decode_inputs(bsz: int = 64, nh: int = 8, dh: int = 64, ctx: int = 2048, seed: int = 0, fill=True):
    """q,k,v ~ N(0,1) [B,H,Dh]; positions ~ U[0, ctx); cache [B,H,ctx,Dh] ~ N(0,1)
    up to each position (zeros above)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((bsz, nh, dh), dtype=np.float32)
    k = rng.standard_normal((bsz, nh, dh), dtype=np.float32)
    v = rng.standard_normal((bsz, nh, dh), dtype=np.float32)
    pos = rng.integers(0, ctx, bsz).astype(np.int32)
    kc = np.zeros((bsz, nh, ctx, dh), dtype=np.float32)
    vc = np.zeros((bsz, nh, ctx, dh), dtype=np.float32)
    if fill:
        for b in range(bsz):
            kc[b, :, : pos[b]] = rng.standard_normal((nh, pos[b], dh), dtype=np.float32)
            vc[b, :, : pos[b]] = rng.standard_normal((nh, pos[b], dh), dtype=np.float32)
    return q, k, v, pos, kc, vc


def conv_ssd_params(nh: int = 16, p: int = 64, seed: int = 0):
    """Per-channel/per-head parameters: conv_w ~ N(0, 0.5) [nh*p, 4],
    conv_b ~ N(0, 0.1), dt_bias ~ N(0, 0.1), A = -exp(U(0, ln16)), D ~ N(1, 0.1)."""
    rng = np.random.default_rng(seed + 1000)
    nch = nh * p
    conv_w = rng.normal(0.0, 0.5, (nch, 4)).astype(np.float32)
    conv_b = rng.normal(0.0, 0.1, nch).astype(np.float32)
    dt_bias = rng.normal(0.0, 0.1, nh).astype(np.float32)
    a_neg = (-np.exp(rng.uniform(0.0, math.log(16.0), nh))).astype(np.float32)
    dsk = rng.normal(1.0, 0.1, nh).astype(np.float32)
    return conv_w, conv_b, dt_bias, a_neg, dsk


def conv_ssd_inputs(bsz: int = 256, t: int = 1, nh: int = 16, p: int = 64, n: int = 128, seed: int = 0,
                    state_scale: float = 1.0):
    """x ~ N(0,1) [B,T,nh*p]; B, C ~ N(0,1) [B,T,n]; dt_raw ~ N(0,1) [B,T,nh];
    conv state ~ N(0,1) [B,nh*p,3]; SSD state ~ N(0, state_scale) [B,nh,p,n]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((bsz, t, nh * p), dtype=np.float32)
    bm = rng.standard_normal((bsz, t, n), dtype=np.float32)
    cm = rng.standard_normal((bsz, t, n), dtype=np.float32)
    dt = rng.standard_normal((bsz, t, nh), dtype=np.float32)
    conv_state = rng.standard_normal((bsz, nh * p, 3), dtype=np.float32)
    ssm = (state_scale * rng.standard_normal((bsz, nh, p, n), dtype=np.float32)).astype(np.float32)
    return x, bm, cm, dt, conv_state, ssm


def decode_prompts(nseq: int = 1024, prompt_len: int = 128, seed: int = 1):
    """Prompts of `prompt_len` token ids ~ U[0, 2048) (seed 1)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, VOCAB, (nseq, prompt_len)).astype(np.uint32)
