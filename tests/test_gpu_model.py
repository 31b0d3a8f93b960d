"""Full-model parity of the CUDA library against the CPU oracle on seeded
random-init Pebble-25M weights: logits within max-abs 1e-4 / rel 1e-5
(|gpu - oracle| <= 1e-4 + 1e-5 |oracle|), identical greedy token streams, and
SSD / conv / KV state within the same tolerance."""
import numpy as np
import pytest

import oracle as O
from krikil_rs_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

from krikil_rs_b200 import (  # noqa: E402
    GenerationEngine, GenerationOptions, KrikilError, PebbleModel, PebbleState, SamplerConfig, _lib)

ATOL, RTOL = 1e-4, 1e-5


def close(a, b, what=""):
    np.testing.assert_allclose(a, b, atol=ATOL, rtol=RTOL, err_msg=what)


@pytest.fixture(scope="module", params=[False, True], ids=["seed0", "seed0-perturbed"])
def models(request):
    path = synth.weights_file(0, perturb=request.param)
    gpu = PebbleModel.load_safetensors(path)
    orc = O.OracleModel(synth.load_safetensors(path))
    return gpu, orc


def _prompt(n, seed=0):
    return np.random.default_rng(seed).integers(0, 2048, n).astype(np.uint32).tolist()


def test_forward_matches_oracle_c1(models):
    """Config: batch 1, 32 prompt ids, greedy 64 tokens, ctx 2048."""
    gpu, orc = models
    gs, os_ = PebbleState(gpu, 2048), O.OracleState(2048)
    prompt = _prompt(32)
    lg, lo = gpu.forward_prefill(prompt, gs), O.forward_prefill(orc, os_, prompt)
    close(lg, lo, "prefill logits")
    toks_g, toks_o = [], []
    ctx_g, ctx_o = list(prompt), list(prompt)
    for i in range(64):
        tg = O.sample_greedy(lg, ctx_g)
        to = O.sample_greedy(lo, ctx_o)
        if tg != to:
            top = np.sort(lo)[-2:]
            pytest.fail(f"token {i}: gpu {tg} oracle {to}; oracle top-2 gap {top[1] - top[0]:.3g}")
        toks_g.append(tg)
        toks_o.append(to)
        ctx_g.append(tg)
        ctx_o.append(to)
        lg, lo = gpu.forward_step(tg, gs), O.forward_step(orc, os_, to)
        close(lg, lo, f"step {i} logits")
    assert gs.current_pos == os_.current_pos == 32 + 64
    for layer in (0, 2, 6):
        close(gs.export(0, layer, 1), os_.ssm[layer], f"ssd state layer {layer}")
        close(gs.export(0, layer, 0), os_.conv[layer], f"conv state layer {layer}")
    for layer in (3, 7):
        close(gs.export(0, layer, 2)[:96], os_.kc[layer][:96], f"k cache layer {layer}")
        close(gs.export(0, layer, 3)[:96], os_.vc[layer][:96], f"v cache layer {layer}")


def test_generate_greedy_device_matches_oracle(models):
    gpu, orc = models
    prompts = [_prompt(n, seed=n) for n in (1, 7, 32, 130)]
    st = PebbleState(gpu, 256, batch=len(prompts))
    for pen, eos in ((1.0, False), (1.2, True)):
        got = gpu.generate_greedy(prompts, st, 40, repetition_penalty=pen, stop_at_eos=eos)
        for b, p in enumerate(prompts):
            ref, _ = O.generate_greedy(orc, O.OracleState(256), p, 40, repetition_penalty=pen,
                                       eos=0 if eos else None)
            assert got[b] == ref, (b, pen)
        # every pushed token is stepped (src/generate.rs:86-114)
        assert list(st.positions) == [len(p) + len(g) for p, g in zip(prompts, got)]


def test_generation_engine_mirror(models):
    gpu, orc = models
    eng = GenerationEngine(gpu)
    st = PebbleState(gpu, 64)
    opts = GenerationOptions(max_new_tokens=20, sampler_config=SamplerConfig(temperature=0.0,
                                                                               repetition_penalty=1.2))
    res = eng.generate(_prompt(10, 3), st, opts)
    ref, _ = O.generate_greedy(orc, O.OracleState(64), _prompt(10, 3), 20, repetition_penalty=1.2, eos=0)
    assert res.generated_tokens == ref
    assert res.tokens_per_second > 0


def test_context_limit_in_generation(models):
    gpu, orc = models
    st = PebbleState(gpu, 16, batch=2)
    got = gpu.generate_greedy([_prompt(5), _prompt(16, 1)], st, 40, stop_at_eos=False)
    assert len(got[0]) == 12 and len(got[1]) == 1
    assert list(st.positions) == [16, 16]
    ref, _ = O.generate_greedy(orc, O.OracleState(16), _prompt(5), 40, eos=None)
    assert got[0] == ref


def test_batched_ragged_prefill_and_steps(models):
    gpu, orc = models
    lens = [1, 5, 64, 65, 200]
    prompts = [_prompt(n, seed=100 + n) for n in lens]
    st = PebbleState(gpu, 512, batch=len(lens))
    lg = gpu.prefill_batch(prompts, st)
    ost = [O.OracleState(512) for _ in lens]
    for b, p in enumerate(prompts):
        close(lg[b], O.forward_prefill(orc, ost[b], p), f"prefill seq {b}")
    for step in range(3):
        toks = [(37 * b + 11 * step) % 2048 for b in range(len(lens))]
        lg = gpu.step_batch(toks, st)
        for b in range(len(lens)):
            close(lg[b], O.forward_step(orc, ost[b], toks[b]), f"step {step} seq {b}")
    assert list(st.positions) == [n + 3 for n in lens]
    close(st.export(4, 1, 1), ost[4].ssm[1])
    close(st.export(3, 7, 2)[:68], ost[3].kc[7][:68])


def test_prefill_continuation_and_reset(models):
    gpu, orc = models
    st = PebbleState(gpu, 128)
    p = _prompt(40, 7)
    a = gpu.forward_prefill(p[:25], st)
    b = gpu.forward_prefill(p[25:], st)
    os_ = O.OracleState(128)
    O.forward_prefill(orc, os_, p[:25])
    close(b, O.forward_prefill(orc, os_, p[25:]))
    st.reset()
    assert st.current_pos == 0
    c = gpu.forward_prefill(p[:25], st)
    np.testing.assert_array_equal(a, c)  # reset state reproduces the first call bitwise


def test_errors_leave_state_untouched(models):
    gpu, _ = models
    st = PebbleState(gpu, 8)
    with pytest.raises(KrikilError) as e:
        gpu.forward_prefill([], st)
    assert e.value.status == _lib.EMPTY and "Cannot prefill empty sequence" in str(e.value)
    with pytest.raises(KrikilError) as e:
        gpu.forward_prefill([1, 2048], st)
    assert e.value.status == _lib.BAD_TOKEN and "Token ID 2048 exceeds vocab size 2048" in str(e.value)
    with pytest.raises(KrikilError) as e:
        gpu.forward_prefill(list(range(9)), st)
    assert e.value.status == _lib.CONTEXT_OVERFLOW
    assert st.current_pos == 0
    gpu.forward_prefill(list(range(8)), st)
    with pytest.raises(KrikilError) as e:
        gpu.forward_step(3, st)
    assert e.value.status == _lib.CONTEXT_OVERFLOW and "Context limit 8 reached" in str(e.value)
    with pytest.raises(KrikilError) as e:
        gpu.forward_step(4096, st)
    assert e.value.status == _lib.BAD_TOKEN
    assert st.current_pos == 8


def test_c5_subset_token_streams(models):
    """Config shape of the batched decode (prompts of 128 ids, seed 1; 256 new
    tokens, EOS ignored) on 16 sequences; two checked in full against the oracle."""
    gpu, orc = models
    prompts = synth.decode_prompts(16, 128, seed=1)
    st = PebbleState(gpu, 2048, batch=16)
    got = gpu.generate_greedy([p.tolist() for p in prompts], st, 256, stop_at_eos=False)
    assert all(len(g) == 256 for g in got)
    for b in (0, 15):
        ref, _ = O.generate_greedy(orc, O.OracleState(2048), prompts[b].tolist(), 256, eos=None)
        assert got[b] == ref, b


def test_c5_benchmark_call_streams_match_oracle():
    """The decode benchmark's own call: 1024 sequences, prompts of 128 ids
    ~U[0,2048) (seed 1), 256 greedy tokens each with EOS ignored, context 2048,
    the decode in its default three parts (rows 0-383, 384-703, 704-1023) on
    seed-0 weights.  32 of the 1024 streams -- both ends of every part and
    spread over the batch -- equal the oracle's token for token."""
    path = synth.weights_file(0)
    gpu = PebbleModel.load_safetensors(path)
    orc = O.OracleModel(synth.load_safetensors(path))
    prompts = synth.decode_prompts(1024, 128, seed=1)
    st = PebbleState(gpu, 2048, batch=1024)
    got = gpu.generate_greedy([p.tolist() for p in prompts], st, 256, stop_at_eos=False)
    assert all(len(g) == 256 for g in got)
    picks = sorted(set(np.linspace(0, 1023, 22).astype(int).tolist()) |
                   {1, 127, 128, 383, 384, 385, 703, 704, 705, 1022})
    assert len(picks) == 32
    for b in picks:
        ref, _ = O.generate_greedy(orc, O.OracleState(2048), prompts[b].tolist(), 256, eos=None)
        if got[b] != ref:
            i = next(i for i, (x, y) in enumerate(zip(got[b], ref)) if x != y)
            pytest.fail(f"sequence {b}: first difference at token {i}: gpu {got[b][i]} oracle {ref[i]}")
    st.close()
    gpu.close()


def test_state_reuse_across_calls_of_growing_size(models):
    """One state serves generation calls whose prompts grow from a few tokens to
    several hundred (the pinned host tables, their device copy and the prompt
    buffer grow between calls) with a prefill and steps in between; every call
    gives exactly the tokens of the same call on a fresh state."""
    gpu, _ = models
    rng = np.random.default_rng(21)
    st = PebbleState(gpu, 1024, batch=6)
    for n_lo, n_hi, new in ((1, 6, 12), (200, 500, 9), (30, 90, 20)):
        prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(n_lo, n_hi, 6)]
        got = gpu.generate_greedy(prompts, st, new, repetition_penalty=1.2, stop_at_eos=False)
        fresh = PebbleState(gpu, 1024, batch=6)
        assert got == gpu.generate_greedy(prompts, fresh, new, repetition_penalty=1.2, stop_at_eos=False)
        fresh.close()
        # the plain API on the same state afterwards: continues from the generated positions
        pos = st.positions.copy()
        lg = gpu.step_batch([5, 6, 7, 8, 9, 10], st)
        assert np.all(st.positions == pos + 1) and lg.shape == (6, 2048)
    st.reset()
    lg = gpu.prefill_batch([[1, 2, 3]] * 6, st)
    fresh = PebbleState(gpu, 1024, batch=6)
    np.testing.assert_array_equal(lg, gpu.prefill_batch([[1, 2, 3]] * 6, fresh))


def test_large_batch_halves_match_single_sequences(models):
    """A batch of 256+ sequences decodes as two halves on two streams; every
    sequence's logits equal (bitwise) those of the same sequence run alone, on
    both sides of the split, and match the oracle."""
    gpu, orc = models
    bsz = 260
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 40, bsz)
    prompts = [rng.integers(0, 2048, n).astype(np.uint32).tolist() for n in lens]
    st = PebbleState(gpu, 64, batch=bsz)
    gpu.prefill_batch(prompts, st)
    picks = (0, 127, 128, 200, bsz - 1)
    alone = {b: PebbleState(gpu, 64) for b in picks}
    for b in picks:
        gpu.forward_prefill(prompts[b], alone[b])
    ost = O.OracleState(64)
    O.forward_prefill(orc, ost, prompts[bsz - 1])
    for step in range(3):
        toks = [(29 * b + 7 * step) % 2048 for b in range(bsz)]
        lg = gpu.step_batch(toks, st)
        for b in picks:
            np.testing.assert_array_equal(lg[b], gpu.forward_step(toks[b], alone[b]), err_msg=f"seq {b}")
        close(lg[bsz - 1], O.forward_step(orc, ost, toks[bsz - 1]), f"step {step}")
    got = gpu.generate_greedy(prompts, st, 6, stop_at_eos=False)
    for b in (3, 255):
        ref, _ = O.generate_greedy(orc, O.OracleState(64), prompts[b], 6, eos=None)
        assert got[b] == ref, b


def test_few_row_batches_match_tiled_batches(models):
    """Decode batches of up to 8 sequences compute their projections in the
    few-rows form (one thread per output column and dot lane, real rows only);
    their step logits and greedy tokens equal (bitwise) those of the same
    sequences inside a 70-sequence batch (64-row tiles), and the oracle's."""
    gpu, orc = models
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(1, 40, 70)]
    big = PebbleState(gpu, 96, batch=70)
    gpu.prefill_batch(prompts, big)
    few = PebbleState(gpu, 96, batch=6)
    sel = [0, 9, 33, 47, 60, 69]
    gpu.prefill_batch([prompts[b] for b in sel], few)
    for step in range(3):
        toks = [(17 * b + 5 * step) % 2048 for b in range(70)]
        lg_big = gpu.step_batch(toks, big)
        lg_few = gpu.step_batch([toks[b] for b in sel], few)
        for i, b in enumerate(sel):
            np.testing.assert_array_equal(lg_few[i], lg_big[b], err_msg=f"seq {b} step {step}")
    st_few, st_big = PebbleState(gpu, 96, batch=6), PebbleState(gpu, 96, batch=70)
    got_few = gpu.generate_greedy([prompts[b] for b in sel], st_few, 12, stop_at_eos=False)
    got_big = gpu.generate_greedy(prompts, st_big, 12, stop_at_eos=False)
    assert got_few == [got_big[b] for b in sel]
    ref, _ = O.generate_greedy(orc, O.OracleState(96), prompts[sel[2]], 12, eos=None)
    assert got_few[2] == ref


def test_profile_modes(models):
    """krk_state_profile: mode 1 times every kernel class (event pairs read back
    when the totals are read), mode 2 only whole calls."""
    gpu, _ = models
    st = PebbleState(gpu, 64, batch=4)
    prompts = [_prompt(5, seed=b) for b in range(4)]
    st.profile(True, per_kernel=True)
    gpu.generate_greedy(prompts, st, 4, stop_at_eos=False)
    p = st.profile_read()
    assert p["device_total"][0] > 0 and p["device_total"][1] == 1
    assert p["gemm"][1] > 0 and p["ssd_step"][1] > 0 and p["attn_decode"][1] > 0
    assert p["ssd_step"][2] == 4 * p["ssd_step"][1]  # 4 sequences per decode launch
    st.profile(True, per_kernel=False)
    gpu.generate_greedy(prompts, st, 4, stop_at_eos=False)
    p = st.profile_read()
    assert p["device_total"][0] > 0 and p["device_total"][1] == 1
    assert all(v[1] == 0 for k, v in p.items() if k != "device_total")
    st.profile(False)


def test_decode_streams_identical(models):
    """krk_state_set_decode_streams: a 520-sequence batch decoded on one stream,
    as two halves, or as three parts of 192 rows gives bitwise identical logits."""
    gpu, _ = models
    bsz = 520
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(1, 30, bsz)]
    out = []
    for n in (1, 2, 3, 4):
        st = PebbleState(gpu, 64, batch=bsz)
        st.set_decode_streams(n)
        gpu.prefill_batch(prompts, st)
        lg = [gpu.step_batch([(13 * b + s) % 2048 for b in range(bsz)], st) for s in range(2)]
        out.append(lg)
    for other in out[1:]:
        for a_, b_ in zip(out[0], other):
            np.testing.assert_array_equal(a_, b_)
    with pytest.raises(KrikilError):
        PebbleState(gpu, 8).set_decode_streams(5)


def test_multi_group_prefill_on_streams(models):
    """A 70-sequence prefill of ~49k tokens runs as several 16k-token groups on
    up to three streams with their own workspaces: its logits and the next
    decode step equal (bitwise) those of the same sequences prefilled ten at a
    time (one group each), and two of them match the oracle."""
    gpu, orc = models
    rng = np.random.default_rng(31)
    bsz, ctx = 70, 1024
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(600, 800, bsz)]
    assert sum(len(p) for p in prompts) > 2 * 16384  # three groups at least
    st = PebbleState(gpu, ctx, batch=bsz)
    lg = gpu.prefill_batch(prompts, st)
    nxt = [int(np.argmax(r)) for r in lg]
    lg2 = gpu.step_batch(nxt, st)
    for c0 in range(0, bsz, 10):
        sub = PebbleState(gpu, ctx, batch=10)
        np.testing.assert_array_equal(gpu.prefill_batch(prompts[c0:c0 + 10], sub), lg[c0:c0 + 10])
        np.testing.assert_array_equal(gpu.step_batch(nxt[c0:c0 + 10], sub), lg2[c0:c0 + 10])
    for b in (0, bsz - 1):
        ref = O.forward_prefill(orc, O.OracleState(ctx), prompts[b])
        np.testing.assert_allclose(lg[b], ref, atol=1e-4, rtol=1e-5)


def test_small_batch_step_graphs(models):
    """Decode steps of batches of one 64-row tile replay CUDA graphs, one per
    count of 512-key attention splits: a 120-token generation from a
    460-token prompt, crossing into the second split, a 40-sequence batch
    with ragged prompts, and a 6-sequence batch whose longer prompts reach the
    end of the context early (inactive sequences beside active ones), give
    exactly the tokens of the same calls launched kernel by kernel (per-kernel
    profiling turns the graphs and the chained launches of a few sequences'
    steps off), and the single sequence matches the oracle."""
    gpu, orc = models
    prompt = _prompt(460, 7)
    runs = []
    for profiled in (False, True):
        st = PebbleState(gpu, 1024)
        if profiled:
            st.profile(True)
        runs.append(gpu.generate_greedy([prompt], st, 120, repetition_penalty=1.2, stop_at_eos=False)[0])
    assert runs[0] == runs[1] and len(runs[0]) == 120
    ref, _ = O.generate_greedy(orc, O.OracleState(1024), prompt, 120, repetition_penalty=1.2, eos=None)
    assert runs[0] == ref
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(1, 90, 40)]
    outs = []
    for profiled in (False, True):
        st = PebbleState(gpu, 256, batch=40)
        if profiled:
            st.profile(True)
        outs.append(gpu.generate_sample(prompts, st, 70, 0.8, 0.9, 20, 1.1, list(range(40)), stop_at_eos=False))
    assert outs[0] == outs[1]
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in (100, 5, 77, 30, 120, 64)]
    outs = []
    for profiled in (False, True):
        st = PebbleState(gpu, 128, batch=6)
        if profiled:
            st.profile(True)
        outs.append(gpu.generate_sample(prompts, st, 60, 0.8, 0.9, 20, 1.1, list(range(6)), stop_at_eos=False))
    assert outs[0] == outs[1]
    assert [len(o) for o in outs[0]] == [29, 60, 52, 60, 9, 60]  # ctx - prompt + 1 where that is below 60


@pytest.mark.parametrize("bsz,parts", [(128, 3), (384, 3), (520, 2)])
def test_step_graphs_of_batches_in_parts(models, bsz, parts):
    """Decode steps of larger batches -- one stream at 128 sequences, three or
    two parts on their own streams with forks and joins at 384 and 520 -- also
    replay CUDA graphs: ragged prompts crossing several attention key-block
    counts give exactly the tokens of the same call launched kernel by kernel,
    and a graph captured for one part layout is dropped when the layout
    changes."""
    gpu, _ = models
    rng = np.random.default_rng(bsz)
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in rng.integers(1, 140, bsz)]
    outs = []
    for graphs in (True, False):
        st = PebbleState(gpu, 256, batch=bsz)
        st.set_decode_streams(parts)
        st.set_step_graphs(graphs)
        outs.append(gpu.generate_greedy(prompts, st, 40, repetition_penalty=1.1, stop_at_eos=False))
        if graphs:  # a new part layout: the captured graphs go, the results stay the same
            st.set_decode_streams(1)
            assert gpu.generate_greedy(prompts, st, 40, repetition_penalty=1.1, stop_at_eos=False) == outs[0]
        st.close()
    assert outs[0] == outs[1]


def test_generate_sample_device_matches_oracle(models):
    """krk_generate_sample against the oracle's generate loop with a seeded
    Sampler per sequence: identical token streams (ragged prompts, EOS on)."""
    gpu, orc = models
    prompts = [_prompt(n, seed=50 + n) for n in (3, 9, 17)]
    seeds = [42, 7, 2**33 + 1]
    st = PebbleState(gpu, 96, batch=len(prompts))
    for temp, top_p, top_k, pen in ((0.7, 0.95, 50, 1.2), (1.0, 1.0, 0, 1.0)):
        got = gpu.generate_sample(prompts, st, 12, temp, top_p, top_k, pen, seeds, stop_at_eos=True)
        for b, p in enumerate(prompts):
            ref = O.generate_sample(orc, O.OracleState(96), p, 12, temp, top_p, top_k, pen, seeds[b], eos=0)
            assert got[b] == ref, (b, temp)
    eng = GenerationEngine(gpu)
    st1 = PebbleState(gpu, 64)
    cfg = SamplerConfig(temperature=0.8, top_p=0.9, top_k=20, repetition_penalty=1.1, seed=5)
    res = eng.generate(prompts[0], st1, GenerationOptions(max_new_tokens=10, sampler_config=cfg))
    assert res.generated_tokens == O.generate_sample(orc, O.OracleState(64), prompts[0], 10, 0.8, 0.9, 20, 1.1, 5)


def test_generation_engine_with_tokenizer(models):
    """GenerationEngine::new(&model, &tokenizer) (src/generate.rs:41-133): each
    token's decode_token text goes to the callback and into generated_text."""
    import os
    from krikil_rs_b200.text import PebbleTokenizer
    gpu, orc = models
    tok = PebbleTokenizer.from_file(os.path.join(os.path.dirname(__file__), "golden", "tokenizer_small.json"))
    eng = GenerationEngine(gpu, tok)
    ids = tok.encode("user: Hello there assistant: ")
    for cfg in (SamplerConfig(temperature=0.0, repetition_penalty=1.2), SamplerConfig(seed=11)):
        seen = []
        res = eng.generate_with_callback(ids, PebbleState(gpu, 64), GenerationOptions(
            max_new_tokens=12, sampler_config=cfg, stream_stdout=False), seen.append)
        if cfg.temperature == 0.0:
            ref, _ = O.generate_greedy(orc, O.OracleState(64), ids, 12, repetition_penalty=1.2, eos=0)
        else:
            ref = O.generate_sample(orc, O.OracleState(64), ids, 12, 0.7, 0.95, 50, 1.2, 11)
        assert res.generated_tokens == ref
        assert seen == [tok.decode_token(t) for t in ref] and res.generated_text == "".join(seen)


def test_large_batch_generation_to_context_limit(models):
    """260 sequences (two decode streams) generating until the context limit,
    with EOS stops on: ragged positions near the end of the cache exercise the
    attention's key bound and the per-sequence stop bookkeeping."""
    gpu, orc = models
    bsz, ctx = 260, 40
    rng = np.random.default_rng(17)
    lens = rng.integers(1, ctx + 1, bsz)
    prompts = [rng.integers(0, 2048, int(n)).astype(np.uint32).tolist() for n in lens]
    st = PebbleState(gpu, ctx, batch=bsz)
    got = gpu.generate_greedy(prompts, st, 64, repetition_penalty=1.1, stop_at_eos=True)
    for b in (0, 129, 130, 259, int(np.argmax(lens)), int(np.argmin(lens))):
        ref, _ = O.generate_greedy(orc, O.OracleState(ctx), prompts[b], 64, repetition_penalty=1.1, eos=0)
        assert got[b] == ref, b
    for b in range(bsz):
        assert len(got[b]) <= ctx - lens[b] + 1
