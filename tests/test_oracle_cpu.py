"""The CPU oracle against the reference's own known-answer tests and against an
independent float64 model (no GPU)."""
import json
import os

import numpy as np
import pytest

import oracle as O
from tests.np_pebble import NpPebble

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


# ---- src/math.rs:266-297 ---------------------------------------------------
def test_dot_product_known_answer():
    a = np.array([1, 2, 3, 4, 5, 6, 7, 8, 9], np.float32)
    b = np.array([2, 1, 0, -1, 3, 2, 1, 0, -2], np.float32)
    assert abs(O.dot(a, b) - float((a * b).sum())) < 1e-5


def test_rms_norm_known_answer():
    out = O.rms_norm([1.0, 2.0, 3.0, 4.0], [1.0] * 4, 1e-6)
    rstd = 1.0 / np.sqrt(np.float32(30.0 / 4.0) + np.float32(1e-6))
    assert abs(out[0] - 1.0 * rstd) < 1e-5
    assert abs(out[3] - 4.0 * rstd) < 1e-5


def test_gelu_known_answer():
    assert abs(O.gelu(0.0)) < 1e-5
    assert abs(O.gelu(1.0) - 0.8413447) < 1e-4
    assert abs(O.gelu(-1.0) - (-0.1586553)) < 1e-4


# ---- src/sampler.rs:160-182 --------------------------------------------------
def test_greedy_sampling_known_answer():
    assert O.sample_greedy([1.0, 5.0, 3.0, 2.0], []) == 1


def test_repetition_penalty_known_answer():
    assert O.sample_greedy([1.0, 5.0, 3.0, 2.0], [1], penalty=3.0) == 2


def test_greedy_first_max_and_nan():
    assert O.sample_greedy([3.0, 7.0, 7.0, 1.0], []) == 1
    assert O.sample_greedy([np.nan, 2.0, np.nan], []) == 1
    assert O.sample_greedy([np.nan, np.nan], []) == 0
    assert O.sample_greedy([-np.inf, -np.inf], []) == 0
    # negative logits are multiplied by the penalty
    assert O.sample_greedy([-1.0, -1.5], [0], penalty=2.0) == 1


# ---- dot order: src/math.rs:89-124 -------------------------------------------
def test_dot_close_to_float64():
    rng = np.random.default_rng(3)
    for n in (8, 9, 76, 608, 1216, 2432, 13):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        ref = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
        assert abs(O.dot(a, b) - ref) < 1e-5 * max(1.0, float(np.abs(a * b).sum()))


def test_gemv_rows_threading_invariant():
    rng = np.random.default_rng(4)
    w = rng.standard_normal((300, 608)).astype(np.float32)
    x = rng.standard_normal(608).astype(np.float32)
    out = O.gemv(w, x)
    for r in (0, 63, 64, 299):
        assert out[r] == O.dot(w[r], x)  # bitwise: each row is one dot


# ---- full model vs independent float64 numpy ---------------------------------
@pytest.mark.parametrize("perturb", [False, True])
def test_oracle_model_matches_float64(perturb, synth_weights, synth_weights_perturbed):
    w = synth_weights_perturbed if perturb else synth_weights
    m = O.OracleModel(w)
    st = O.OracleState(64)
    ref = NpPebble(w, 64)
    toks = [5, 1999, 17, 300, 42, 7]
    lo = O.forward_prefill(m, st, toks)
    lr = ref.prefill(toks)
    np.testing.assert_allclose(lo, lr, atol=2e-5, rtol=1e-4)
    for t in (11, 2047, 0):
        np.testing.assert_allclose(O.forward_step(m, st, t), ref.step(t), atol=2e-5, rtol=1e-4)
    assert st.current_pos == len(toks) + 3
    np.testing.assert_allclose(st.ssm[0], ref.ssm[0], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(st.conv[4], ref.conv[4], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(st.kc[7][:9], ref.k[7][:9], atol=1e-5, rtol=1e-4)


def test_oracle_model_matches_float64_c1_prompt(synth_weights_perturbed):
    """The batch-1 workload's 32-token prompt (seed 0) and eight decode steps
    on the perturbed weights (norm weights, D and conv bias away from their
    constants), against the float64 model: longer contexts for the SSD and the
    attention cache than the short-prompt test."""
    w = synth_weights_perturbed
    m = O.OracleModel(w)
    st = O.OracleState(64)
    ref = NpPebble(w, 64)
    toks = np.random.default_rng(0).integers(0, O.VOCAB, 32).tolist()
    np.testing.assert_allclose(O.forward_prefill(m, st, toks), ref.prefill(toks), atol=2e-5, rtol=1e-4)
    for t in (199, 490, 0, 2047, 5, 5, 1024, 77):
        np.testing.assert_allclose(O.forward_step(m, st, t), ref.step(t), atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(st.ssm[5], ref.ssm[5], atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(st.conv[1], ref.conv[1], atol=1e-6, rtol=1e-5)
    np.testing.assert_allclose(st.kc[3][:40], ref.k[3][:40], atol=1e-5, rtol=1e-4)


def test_prefill_then_prefill_equals_one_prefill(synth_weights):
    """Prefill at a nonzero start (src/model.rs:495, :506) continues the sequence."""
    m = O.OracleModel(synth_weights)
    s1, s2 = O.OracleState(32), O.OracleState(32)
    toks = [9, 8, 7, 6, 5, 4, 3]
    a = O.forward_prefill(m, s1, toks)
    O.forward_prefill(m, s2, toks[:3])
    b = O.forward_prefill(m, s2, toks[3:])
    np.testing.assert_allclose(a, b, atol=1e-5, rtol=1e-5)
    assert s2.current_pos == 7 and s2.cur_len(3) == 7


def test_oracle_errors(synth_weights):
    m = O.OracleModel(synth_weights)
    st = O.OracleState(4)
    with pytest.raises(O.OracleError) as e:
        O.forward_prefill(m, st, [])
    assert e.value.code == O.EMPTY
    with pytest.raises(O.OracleError) as e:
        O.forward_prefill(m, st, [1, 2048])
    assert e.value.code == O.BAD_TOKEN
    assert st.current_pos == 0
    with pytest.raises(O.OracleError) as e:
        O.forward_prefill(m, st, [1, 2, 3, 4, 5])
    assert e.value.code == O.CONTEXT_OVERFLOW
    O.forward_prefill(m, st, [1, 2, 3, 4])
    with pytest.raises(O.OracleError) as e:
        O.forward_step(m, st, 1)
    assert e.value.code == O.CONTEXT_OVERFLOW
    with pytest.raises(O.OracleError) as e:
        O.forward_step(m, st, 5000)
    assert e.value.code == O.BAD_TOKEN
    st.reset()
    assert st.current_pos == 0 and not st.ssm[0].any()


def test_generate_greedy_loop_semantics(synth_weights):
    """src/generate.rs:86-110: count, context limit and determinism."""
    m = O.OracleModel(synth_weights)
    st = O.OracleState(16)
    out, _ = O.generate_greedy(m, st, [3, 1, 4, 1, 5], 20, eos=None)
    assert len(out) == 16 - 5 + 1  # stops once current_pos reaches the limit
    st2 = O.OracleState(16)
    out2, _ = O.generate_greedy(m, st2, [3, 1, 4, 1, 5], 20, eos=None)
    assert out == out2


# ---- prefill projections in matrixmultiply's summation order -----------------
def test_sgemm_order_gemm_close_to_float64():
    """The restated matrixmultiply 0.3.11 sgemm order (src/math.rs:188-211) is a
    correct product, and it rounds differently from the gemv dot order."""
    rng = np.random.default_rng(3)
    for m, k, n in ((5, 608, 37), (3, 1216, 19), (2, 2432, 11), (4, 100, 9), (3, 257, 5), (3, 256, 7),
                    (2, 512, 6)):
        a = rng.standard_normal((m, k), dtype=np.float32)
        b = rng.standard_normal((n, k), dtype=np.float32)
        exact = a.astype(np.float64) @ b.astype(np.float64).T
        with O.prefill_gemm_order("matrixmultiply"):
            mm = O.gemm_transb(a, b)
        dot = O.gemm_transb(a, b)
        bound = 4 * k * np.finfo(np.float32).eps * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64).T)
        assert np.all(np.abs(mm - exact) <= bound)
        assert np.all(np.abs(dot - exact) <= bound)
        assert not np.array_equal(mm, dot)
    # one block of K is a single FMA chain from zero; two blocks add their chains
    # (the two 2^-24 terms are absorbed one at a time by the running 1.0: the
    # exact sum 2^-23 comes out as 0; split over two blocks they survive)
    a = np.array([[1.0, 2.0 ** -24, 2.0 ** -24, -1.0]], np.float32)
    b = np.ones((1, 4), np.float32)
    with O.prefill_gemm_order("matrixmultiply"):
        assert O.gemm_transb(a, b)[0, 0] == 0.0
        a2 = np.zeros((1, 512), np.float32)
        a2[0, 0], a2[0, 256], a2[0, 257], a2[0, 1] = 1.0, 2.0 ** -24, 2.0 ** -24, -1.0
        assert O.gemm_transb(a2, np.ones((1, 512), np.float32))[0, 0] == np.float32(2.0 ** -23)
    assert O.lib.orc_prefill_gemm_order() == 0


def _prefill_and_generate(w, prompt, new, order):
    m = O.OracleModel(w)
    with O.prefill_gemm_order(order):
        st = O.OracleState(2048)
        logits = O.forward_prefill(m, st, prompt)
        ssm = {i: a.copy() for i, a in st.ssm.items()}
        conv = {i: a.copy() for i, a in st.conv.items()}
        kc = {i: a[:len(prompt)].copy() for i, a in st.kc.items()}
        toks, _ = O.generate_greedy(m, O.OracleState(2048), prompt, new, eos=None)
    return logits, ssm, conv, kc, toks


@pytest.mark.parametrize("case", ["c1", "c5"])
def test_prefill_in_matrixmultiply_order_within_tolerance(case, synth_weights):
    """The reference's prefill projections go through matrixmultiply::sgemm
    (src/math.rs:188-211, called at src/model.rs:387, 458, 484, 554, 570, 577);
    the CUDA path and the default oracle sum them in the gemv dot order.  With
    the sgemm order restated, the prefill logits stay within the logits
    tolerance (max-abs 1e-4 plus rel 1e-5), the SSD, conv and K states within
    the same tolerance, and the greedy streams that follow are identical.  c1:
    the 32-token prompt of the batch-1 workload (seed 0) and 64 tokens; c5: two
    of the 128-token prompts of the 1024-sequence workload (seed 1, the first
    and the last) and 32 tokens each."""
    from krikil_rs_b200 import synth
    if case == "c1":
        prompts, new = [np.random.default_rng(0).integers(0, O.VOCAB, 32).astype(np.uint32)], 64
    else:
        p = synth.decode_prompts()
        prompts, new = [p[0], p[-1]], 32
    for prompt in prompts:
        d = _prefill_and_generate(synth_weights, prompt, new, "dot")
        mm = _prefill_and_generate(synth_weights, prompt, new, "matrixmultiply")
        assert not np.array_equal(d[0], mm[0])  # the orders do differ
        np.testing.assert_allclose(mm[0], d[0], atol=1e-4, rtol=1e-5)
        for i in d[1]:
            np.testing.assert_allclose(mm[1][i], d[1][i], atol=1e-4, rtol=1e-5)
            np.testing.assert_allclose(mm[2][i], d[2][i], atol=1e-4, rtol=1e-5)
        for i in d[3]:
            np.testing.assert_allclose(mm[3][i], d[3][i], atol=1e-4, rtol=1e-5)
        assert mm[4] == d[4]


# ---- golden fixtures of the reference ----------------------------------------
def test_golden_fixtures_consistent():
    with open(os.path.join(GOLDEN, "reference_prefill_logits.json")) as f:
        pre = json.load(f)
    with open(os.path.join(GOLDEN, "reference_step_logits.json")) as f:
        stp = json.load(f)
    assert len(pre["logits"]) == 2048 and len(stp["logits"]) == 2048
    assert stp["tokens"] == pre["tokens"] + [stp["step_token"]]
    assert int(np.argmax(pre["logits"])) == stp["step_token"] == 199  # greedy continuation
    assert int(np.argmax(stp["logits"])) == 490


@pytest.mark.skipif(not os.environ.get("KRIKIL_PEBBLE_WEIGHTS"), reason="real Pebble-25M checkpoint not available")
def test_oracle_matches_reference_golden_logits():
    """src/model.rs:791-932 with the real weights: max-abs < 1e-4, same argmax."""
    from krikil_rs_b200 import synth
    w = synth.load_safetensors(os.environ["KRIKIL_PEBBLE_WEIGHTS"])
    m = O.OracleModel(w)
    with open(os.path.join(GOLDEN, "reference_prefill_logits.json")) as f:
        pre = json.load(f)
    with open(os.path.join(GOLDEN, "reference_step_logits.json")) as f:
        stp = json.load(f)
    st = O.OracleState(2048)
    lg = O.forward_prefill(m, st, pre["tokens"])
    assert np.abs(lg - np.array(pre["logits"], np.float32)).max() < 1e-4
    assert int(np.argmax(lg)) == int(np.argmax(pre["logits"]))
    lg2 = O.forward_step(m, st, stp["step_token"])
    assert np.abs(lg2 - np.array(stp["logits"], np.float32)).max() < 1e-4


# ---- stochastic sampler (src/sampler.rs:83-152) and its StdRng stream -------
def test_chacha_block_published_vectors():
    """The oracle's ChaCha block function (run with 20 rounds) against the
    published ChaCha20 vectors: the all-zero key/nonce keystream and RFC 7539
    section 2.3.2; ChaCha12, the reference's StdRng core, is the same code with
    12 rounds."""
    const = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574]
    out = O.chacha_block(const + [0] * 12, 20)
    assert out[:4] == [0xADE0B876, 0x903DF1A0, 0xE56A5D40, 0x28BD8653]
    key = [int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)]
    nonce = bytes.fromhex("000000090000004a00000000")
    words = const + key + [1] + [int.from_bytes(nonce[4 * i:4 * i + 4], "little") for i in range(3)]
    ser = b"".join(w.to_bytes(4, "little") for w in O.chacha_block(words, 20))
    assert ser[:16].hex() == "10f1e7e4d13b5915500fdd1fa32071c4"


def _rng_from_seed_bytes(seed: bytes, rounds: int):
    """A ChaCha generator keyed by a 32-byte seed (SeedableRng::from_seed of
    rand_chacha 0.3): key words little-endian, block counter and stream 0.
    With 12 rounds it is the oracle's Rng (orc_rng_next_u32); the 20-round
    form draws keystream words from the same block function."""
    key = [int.from_bytes(seed[4 * i:4 * i + 4], "little") for i in range(8)]
    if rounds == 12:
        r = O.Rng(0)
        r.state[:8] = key
        r.state[8:] = 0
        return r.next_u32
    const = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574]
    words = iter([])
    blk = [0]

    def next_u32():
        nonlocal words
        w = next(words, None)
        if w is None:
            words = iter(O.chacha_block(const + key + [blk[0], 0, 0, 0], 20))
            blk[0] += 1
            w = next(words)
        return w
    return next_u32


def _seed_bytes_from(next_u32) -> bytes:
    """SeedableRng::from_rng: 32 bytes taken with fill_bytes, i.e. the next
    eight keystream words in order."""
    return b"".join(next_u32().to_bytes(4, "little") for _ in range(8))


def test_stdrng_value_stability_vectors():
    """Known answers of the generators the reference's Sampler draws from
    (StdRng, src/sampler.rs:35-40 and :142): the value-stability vectors of
    rand 0.8 (StdRng = rand_chacha 0.3 ChaCha12Rng) and of rand_chacha 0.3
    (ChaCha20Rng): a generator from a 32-byte seed, its first output, then a
    generator seeded from its next 32 bytes and that one's first output.  They
    pin the key layout, the counter and stream words, StdRng's 12 rounds and the
    order in which the block generator hands out words (next_u64 = two words,
    low first).  rand_core 0.6's seed_from_u64 expansion (PCG32) has no such
    vector and stays restated only."""
    nxt = _rng_from_seed_bytes(bytes([1, 0, 0, 0, 23, 0, 0, 0, 200, 1, 0, 0, 210, 30, 0, 0] + [0] * 16), 12)
    x0 = nxt() | (nxt() << 32)
    nxt1 = _rng_from_seed_bytes(_seed_bytes_from(nxt), 12)
    x1 = nxt1() | (nxt1() << 32)
    assert [x0, x1] == [10719222850664546238, 14064965282130556830]

    seed = bytes([0] * 8 + [1] + [0] * 7 + [2] + [0] * 7 + [3] + [0] * 7)
    nxt = _rng_from_seed_bytes(seed, 20)
    assert nxt() == 137206642
    nxt1 = _rng_from_seed_bytes(_seed_bytes_from(nxt), 20)
    assert nxt1() == 1325750369


def test_rng_stream_deterministic_and_uniform():
    a, b = O.Rng(42), O.Rng(42)
    xs = [a.gen_f32() for _ in range(4000)]
    assert xs == [b.gen_f32() for _ in range(4000)]
    assert all(0.0 <= x < 1.0 for x in xs) and abs(np.mean(xs) - 0.5) < 0.02
    assert O.Rng(43).next_u32() != O.Rng(42).next_u32()


def test_sampling_deterministic_with_seed():
    """src/sampler.rs:185-201: two samplers with seed 42 pick the same token."""
    lg = np.array([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], np.float32)
    t1 = O.sample(lg, [], 0.7, 0.9, 10, 1.0, O.Rng(42))
    t2 = O.sample(lg, [], 0.7, 0.9, 10, 1.0, O.Rng(42))
    assert t1 == t2 and 0 <= t1 < 6


def test_sampling_filters_and_distribution():
    lg = np.array([0.5, 2.0, 1.0, -1.0, 1.5], np.float32)
    rng = O.Rng(7)
    assert {O.sample(lg, [], 1.0, 1.0, 1, 1.0, rng) for _ in range(50)} == {1}  # top-k 1 = argmax
    assert {O.sample(lg, [], 1.0, 1e-3, 0, 1.0, rng) for _ in range(50)} == {1}  # tiny top-p keeps one
    assert {O.sample(lg, [], 1.0, 0.9, 2, 1.0, rng) for _ in range(200)} <= {1, 4}
    counts = np.bincount([O.sample(lg, [], 1.0, 1.0, 0, 1.0, rng) for _ in range(20000)], minlength=5)
    p = np.exp(lg - lg.max())
    p /= p.sum()
    assert np.abs(counts / counts.sum() - p).max() < 0.015
    assert O.sample(lg, [1], 0.0, 1.0, 0, 3.0, rng) == 4  # temperature 0: greedy after the penalty
