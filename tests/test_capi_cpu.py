"""The C-ABI library on a machine without a GPU: it loads, exports every entry
point include/krikil_cuda.h declares, and reports file/format errors (which
the loader checks before touching a device) with the reference's messages."""
import ctypes as C
import os
import re
import struct

import numpy as np
import pytest

from krikil_rs_b200 import _lib, synth
from krikil_rs_b200._lib import KrikilError, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    with open(os.path.join(ROOT, "include", "krikil_cuda.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"KRK_API\s+[\w\s\*]+?\b(krk_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "krk_model_load" in names and "krk_k_gemm" in names and len(names) >= 29


def test_library_exports_every_declared_symbol():
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTED) >= set(_declared())


def test_checked_build_exports_the_same_symbols_and_says_so():
    """The checked build (make CHECKED=1) exports every declared entry point and
    reports itself as checked; the default build reports 0 and no check bits."""
    assert lib.krk_checked_build() == (1 if _lib.CHECKED else 0)
    bits = C.c_uint32(123)
    assert lib.krk_check_status(C.byref(bits), 1) == _lib.OK and bits.value == 0
    path = os.path.join(ROOT, "krikil_rs_b200", "lib", "libkrikil_cuda_checked.so")
    chk = C.CDLL(path)
    for name in _declared():
        assert hasattr(chk, name), name
    assert chk.krk_checked_build() == 1


def test_abi_version_and_status_strings():
    assert lib.krk_abi_version() == 1
    assert lib.krk_status_string(_lib.BAD_TOKEN) == b"token id exceeds vocab size"


def _load(path):
    h = C.c_void_p()
    return lib.krk_model_load(path.encode(), 0, C.byref(h)), lib.krk_last_error().decode()


def test_load_missing_file(tmp_path):
    rc, msg = _load(str(tmp_path / "nope.safetensors"))
    assert rc == _lib.IO and "Failed to open model file" in msg


def test_load_truncated_and_malformed(tmp_path):
    p = tmp_path / "t.safetensors"
    p.write_bytes(b"\x01\x02")
    assert _load(str(p))[0] == _lib.IO
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    rc, msg = _load(str(p))
    assert rc == _lib.IO and "header length exceeds file" in msg
    hdr = b'{"wte.weight": {"dtype": "F32", "shape": [2], "data_offsets": [0, 64]}}'
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
    rc, msg = _load(str(p))
    assert rc == _lib.IO and "exceed" in msg


def test_load_missing_tensor(tmp_path):
    w = {"wte.weight": np.zeros((2048, 608), np.float32)}
    p = str(tmp_path / "m.safetensors")
    synth.save_safetensors(p, w)
    rc, msg = _load(p)
    assert rc == _lib.NOT_FOUND and msg == "Tensor 'lnf.weight' not found in model"


def test_load_wrong_size_and_dtype(tmp_path):
    w = synth.make_weights(0)
    w["blocks.3.wo.weight"] = w["blocks.3.wo.weight"][:100]
    p = str(tmp_path / "m.safetensors")
    synth.save_safetensors(p, w)
    rc, msg = _load(p)
    assert rc == _lib.IO and "blocks.3.wo.weight" in msg
    # shapes are not checked (like the reference), only element counts:
    w = synth.make_weights(0)
    w["blocks.0.mixer.conv1d.weight"] = w["blocks.0.mixer.conv1d.weight"].reshape(1472, 4)
    synth.save_safetensors(p, w)
    rc, msg = _load(p)
    assert rc in (_lib.OK, _lib.CUDA)  # CUDA when this machine has no GPU


def test_python_mirror_raises_krikil_error(tmp_path):
    from krikil_rs_b200 import PebbleModel
    with pytest.raises(KrikilError) as e:
        PebbleModel.load_safetensors(str(tmp_path / "missing"))
    assert e.value.status == _lib.IO


def test_synth_safetensors_roundtrip(tmp_path):
    w = synth.make_weights(0)
    assert len(w) == 2 + 6 * 9 + 2 * 6
    p = str(tmp_path / "w.safetensors")
    synth.save_safetensors(p, w)
    r = synth.load_safetensors(p)
    for k in w:
        np.testing.assert_array_equal(w[k], r[k])
    w2 = synth.make_weights(0)
    assert all(np.array_equal(w[k], w2[k]) for k in w)
    assert (w["blocks.0.mixer.A_log"] >= 0).all() and (w["blocks.0.mixer.A_log"] <= np.log(16)).all()


def test_rng_seed_state_matches_oracle():
    """krk_rng_seed_state (host) = the oracle's StdRng::seed_from_u64 restatement."""
    import oracle as O
    for seed in (0, 1, 42, 2**63 + 5, 2**64 - 1):
        st = np.zeros(10, np.uint32)
        assert lib.krk_rng_seed_state(seed, st.ctypes.data) == _lib.OK
        np.testing.assert_array_equal(st, O.Rng(seed).state)


def test_gemm_refuses_operands_past_32bit_offsets():
    """The projection indexes A^T and W^T with 32-bit element offsets, so
    K * lda or K * ldw of 2^31 or more is refused before anything touches a
    device (INVALID, where a launch on this machine would report CUDA)."""
    p = 16  # 16-byte aligned placeholder: the size check comes first
    assert lib.krk_k_gemm_tiled(p, 67108868, p, 32, p, 32, 32, 32, 32, 0, 0, 0, None) == _lib.INVALID
    assert lib.krk_k_gemm_tiled(p, 32, p, 67108868, p, 32, 32, 32, 32, 0, 0, 0, None) == _lib.INVALID


def test_gemm_tile_choice_small_batches():
    """The automatic projection tile height (host rule, B200's 148 SMs): at
    decode sizes the smallest of 16/32/64 rows whose grid fits in one wave,
    else 32 rows below 256 rows and 64 from there on.  Every height gives bitwise the same
    result (the GPU projection tests run each one)."""
    m64 = {608: 16, 1824: 32, 2048: 32, 2432: 64, 2720: 64}
    m128 = {608: 32, 1824: 64, 2048: 64, 2432: 32, 2720: 32}
    for m, table in ((64, m64), (128, m128)):
        for n, t in table.items():
            assert lib.krk_k_gemm_tile_rows(m, n) == t, (m, n)
    assert lib.krk_k_gemm_tile_rows(192, 608) == 32 and lib.krk_k_gemm_tile_rows(192, 2720) == 32
    assert lib.krk_k_gemm_tile_rows(1024, 608) == 64 and lib.krk_k_gemm_tile_rows(1024, 2720) == 64
    assert lib.krk_k_gemm_tile_rows(16384, 2720) == 64 and lib.krk_k_gemm_tile_rows(0, 32) == 0
