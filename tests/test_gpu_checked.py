"""The checked build (make CHECKED=1, loaded with KRIKIL_CHECKED=1): its kernels
test the preconditions on device data that the host cannot see before a
launch and report a violated one as a bit of the device status word read by
krk_check_status, skipping the access instead of making it (no trap, no
assert; the context stays usable).

Run in a child process, since a process loads one build of the library.  The
planted faults are device-side values that every build's kernels already
guard (a position at the context limit, a token id past the vocabulary):
the default build skips them silently, the checked build also reports them."""
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import ctypes as C
import numpy as np
import torch
import oracle as O
from krikil_rs_b200 import PebbleModel, PebbleState, synth, kernels as K
from krikil_rs_b200._lib import lib, CHECKED, CHECK_POSITION, CHECK_TOKEN, OK

assert CHECKED and lib.krk_checked_build() == 1

def status():
    torch.cuda.synchronize()
    b = C.c_uint32()
    assert lib.krk_check_status(C.byref(b), 1) == OK
    return b.value

dev = torch.device("cuda:0")
cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)

# 1. a clean generation: the oracle's tokens, no check bit
path = synth.weights_file(0)
gpu, orc = PebbleModel.load_safetensors(path), O.OracleModel(synth.load_safetensors(path))
rng = np.random.default_rng(4)
prompts = [rng.integers(0, 2048, n).astype(np.uint32).tolist() for n in (5, 37, 70)]
st = PebbleState(gpu, 128, batch=3)
got = gpu.generate_greedy(prompts, st, 20, repetition_penalty=1.1, stop_at_eos=False)
for b, p in enumerate(prompts):
    ref, _ = O.generate_greedy(orc, O.OracleState(128), p, 20, repetition_penalty=1.1, eos=None)
    assert got[b] == ref, b
assert status() == 0

# 2. decode attention with one position at the context limit: that (sequence,
# head) is skipped and reported, the others match the oracle
bsz, nh, dh, ctx = 4, 2, 64, 256
q, k, v = (rng.standard_normal((bsz, nh, dh)).astype(np.float32) for _ in range(3))
kc, vc = (rng.standard_normal((bsz, nh, ctx, dh)).astype(np.float32) for _ in range(2))
pos = np.array([10, ctx, 200, 63], np.int32)
for split in (0, 64, 256):
    out = K.rope_kv_attn_decode(cu(q), cu(k), cu(v), cu(kc), cu(vc), cu(pos), split=split)
    assert status() & CHECK_POSITION, split
    good = [0, 2, 3]
    ref = O.rope_kv_attn_decode(q[good], k[good], v[good], kc[good].copy(), vc[good].copy(), pos[good])
    np.testing.assert_allclose(out.cpu().numpy()[good], ref, atol=1e-4, rtol=1e-5)
    assert status() == 0

# 3. the embedding gather with a token id past the vocabulary: zeros, reported
wte = cu(rng.standard_normal((2048, 608)).astype(np.float32))
tok = torch.tensor([3, 2048, 7], dtype=torch.int32, device=dev)
out = torch.empty((608, 64), device=dev)
assert lib.krk_k_embed(tok.data_ptr(), wte.data_ptr(), 2048, 608, 3, out.data_ptr(), 64, None) == OK
assert status() & CHECK_TOKEN
o = out.cpu().numpy()
assert (o[:, 1] == 0).all() and np.array_equal(o[:, 0], wte.cpu().numpy()[3])
print("checked build ok")
'''


def test_checked_build_reports_device_faults_and_matches_the_oracle():
    env = dict(os.environ, KRIKIL_CHECKED="1", PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "checked build ok" in r.stdout
