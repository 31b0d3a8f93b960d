"""Python mirror of krikil-rs's model API over the C ABI.

Names and semantics follow the Rust library (src/model.rs, src/generate.rs,
src/sampler.rs): ``PebbleModel.load_safetensors``, ``forward_prefill``,
``forward_step``, ``PebbleState(model, max_ctx).reset()`` and
``GenerationEngine.generate``.  Errors raise ``KrikilError`` with the same
conditions and messages as the reference's ``anyhow`` errors.  Batched forms
(``prefill_batch``, ``step_batch``, ``generate_greedy``) run many independent
sequences in one state.
"""
from __future__ import annotations

import ctypes as C
import os
import time
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import KrikilError, check, lib

VOCAB_SIZE = 2048
HIDDEN_SIZE = 608
NUM_LAYERS = 8
EOS_TOKEN = 0


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


@dataclass
class PebbleConfig:
    """src/model.rs:32-84 (defaults; config.json is not read by the reference)."""

    vocab_size: int = 2048
    hidden_size: int = 608
    num_hidden_layers: int = 8
    num_attention_heads: int = 8
    intermediate_size: int = 2432
    max_position_embeddings: int = 2048
    block_pattern: str = "mmma|mmma"


class PebbleModel:
    """src/model.rs:112-117, with weights resident on one GPU."""

    def __init__(self, handle: int, device: int):
        self._h = C.c_void_p(handle)
        self.device = device
        self.config = PebbleConfig()

    @classmethod
    def load_safetensors(cls, path: str, device: int = 0) -> "PebbleModel":
        h = C.c_void_p()
        check(lib.krk_model_load(str(path).encode(), device, C.byref(h)))
        return cls(h.value, device)

    @property
    def stream(self) -> int:
        s = C.c_void_p()
        check(lib.krk_model_stream(self._h, C.byref(s)))
        return s.value or 0

    def close(self) -> None:
        if self._h:
            lib.krk_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -------------------------------------------------- reference API (batch 1)
    def forward_prefill(self, tokens: Sequence[int], state: "PebbleState") -> np.ndarray:
        """src/model.rs:316-368: last-token logits [2048]; advances current_pos."""
        return self.prefill_batch([tokens], state)[0]

    def forward_step(self, token: int, state: "PebbleState") -> np.ndarray:
        """src/model.rs:586-624: logits [2048] of one token; advances current_pos."""
        return self.step_batch([token], state)[0]

    # -------------------------------------------------------------- batched
    def prefill_batch(self, prompts: Sequence[Sequence[int]], state: "PebbleState",
                      want_logits: bool = True) -> Optional[np.ndarray]:
        if len(prompts) != state.batch:
            raise ValueError(f"{len(prompts)} prompts for a state of batch {state.batch}")
        lens = np.array([len(p) for p in prompts], dtype=np.int32)
        toks = _pack(prompts)
        out = np.empty((state.batch, VOCAB_SIZE), np.float32) if want_logits else None
        check(lib.krk_prefill(self._h, state._h, _ptr(toks) if toks.size else None, _ptr(lens),
                              _ptr(out) if out is not None else None))
        return out

    def step_batch(self, tokens: Sequence[int], state: "PebbleState", want_logits: bool = True) -> Optional[np.ndarray]:
        toks = _u32(tokens)
        if toks.size != state.batch:
            raise ValueError(f"{toks.size} tokens for a state of batch {state.batch}")
        out = np.empty((state.batch, VOCAB_SIZE), np.float32) if want_logits else None
        check(lib.krk_step(self._h, state._h, _ptr(toks), _ptr(out) if out is not None else None))
        return out

    def generate_greedy(self, prompts: Sequence[Sequence[int]], state: "PebbleState", max_new_tokens: int,
                        repetition_penalty: float = 1.0, stop_at_eos: bool = True) -> List[List[int]]:
        """Batched greedy generation with device-side sampling (see
        krk_generate_greedy); returns the generated ids of every sequence."""
        if len(prompts) != state.batch:
            raise ValueError(f"{len(prompts)} prompts for a state of batch {state.batch}")
        lens = np.array([len(p) for p in prompts], dtype=np.int32)
        toks = _pack(prompts)
        out = np.zeros((state.batch, max_new_tokens), np.uint32)
        n = np.zeros(state.batch, np.int32)
        check(lib.krk_generate_greedy(self._h, state._h, _ptr(toks) if toks.size else None, _ptr(lens),
                                      int(max_new_tokens), float(repetition_penalty), int(bool(stop_at_eos)),
                                      _ptr(out), _ptr(n)))
        return [out[b, : n[b]].tolist() for b in range(state.batch)]

    def generate_sample(self, prompts: Sequence[Sequence[int]], state: "PebbleState", max_new_tokens: int,
                        temperature: float, top_p: float = 1.0, top_k: int = 0, repetition_penalty: float = 1.0,
                        seeds: Optional[Sequence[int]] = None, stop_at_eos: bool = True) -> List[List[int]]:
        """Batched generation with the stochastic sampler on the device (see
        krk_generate_sample); sequence b draws from StdRng::seed_from_u64(seeds[b])."""
        if len(prompts) != state.batch:
            raise ValueError(f"{len(prompts)} prompts for a state of batch {state.batch}")
        if seeds is None:
            seeds = [int.from_bytes(os.urandom(8), "little") for _ in range(state.batch)]
        sd = np.ascontiguousarray(np.array([int(x) & 0xFFFFFFFFFFFFFFFF for x in seeds], dtype=np.uint64))
        if sd.size != state.batch:
            raise ValueError(f"{sd.size} seeds for a state of batch {state.batch}")
        lens = np.array([len(p) for p in prompts], dtype=np.int32)
        toks = _pack(prompts)
        out = np.zeros((state.batch, max_new_tokens), np.uint32)
        n = np.zeros(state.batch, np.int32)
        check(lib.krk_generate_sample(self._h, state._h, _ptr(toks) if toks.size else None, _ptr(lens),
                                      int(max_new_tokens), float(temperature), float(top_p), int(top_k),
                                      float(repetition_penalty), _ptr(sd), int(bool(stop_at_eos)), _ptr(out),
                                      _ptr(n)))
        return [out[b, : n[b]].tolist() for b in range(state.batch)]


def _u32(tokens) -> np.ndarray:
    a = np.asarray(tokens, dtype=np.int64)
    if a.size and (a.min() < 0 or a.max() > 0xFFFFFFFF):
        raise KrikilError(_lib.BAD_TOKEN, "Token ID out of u32 range")
    return np.ascontiguousarray(a.astype(np.uint32))


def _pack(prompts) -> np.ndarray:
    parts = [_u32(p) for p in prompts]
    return np.ascontiguousarray(np.concatenate(parts) if parts else np.zeros(0, np.uint32))


class PebbleState:
    """src/model.rs:196-230: per-sequence Mamba conv/SSD state and KV caches,
    here for ``batch`` independent sequences resident on the model's GPU."""

    def __init__(self, model: PebbleModel, max_ctx: int = 2048, batch: int = 1):
        h = C.c_void_p()
        check(lib.krk_state_create(model._h, int(batch), int(max_ctx), C.byref(h)))
        self._h = h
        self.model = model
        self.batch = int(batch)
        self.context_limit = int(max_ctx)

    def reset(self, mask: Optional[Sequence[bool]] = None) -> None:
        m = None if mask is None else np.ascontiguousarray(np.asarray(mask, dtype=np.uint8))
        check(lib.krk_state_reset(self._h, _ptr(m) if m is not None else None))

    @property
    def positions(self) -> np.ndarray:
        p = np.zeros(self.batch, np.int64)
        check(lib.krk_state_positions(self._h, _ptr(p)))
        return p

    @property
    def current_pos(self) -> int:
        return int(self.positions[0])

    def export(self, seq: int, layer: int, what: int) -> np.ndarray:
        """Layer state of one sequence: what 0 conv [1472,4], 1 SSD [19,64,128],
        2 K cache [ctx,608], 3 V cache [ctx,608]."""
        shapes = {0: (1472, 4), 1: (19, 64, 128), 2: (self.context_limit, 608), 3: (self.context_limit, 608)}
        out = np.empty(shapes[what], np.float32)
        check(lib.krk_state_export(self._h, seq, layer, what, _ptr(out), out.size))
        return out

    def set_decode_streams(self, n: int) -> None:
        """Decode batches of 256+ in up to n parts of whole 64-row tiles on their
        own streams (3 by default, at most 4); 1: decode and prefill on one stream."""
        check(lib.krk_state_set_decode_streams(self._h, int(n)))

    def set_step_graphs(self, enable: bool) -> None:
        """Replay each decode step of the generation loops as a CUDA graph (the
        default) or launch its kernels one by one; results are identical."""
        check(lib.krk_state_set_step_graphs(self._h, int(bool(enable))))

    def profile(self, enable: bool = True, per_kernel: bool = True) -> None:
        """Turn CUDA-event timing of later calls on/off (resets totals): per kernel
        class and whole calls, or (per_kernel=False) whole calls only."""
        check(lib.krk_state_profile(self._h, 0 if not enable else (1 if per_kernel else 2)))

    def profile_read(self) -> dict:
        """{class: (device ms, launches, decode sequences)} accumulated since
        profile().  Kernel times of the two decode streams may overlap."""
        out = {}
        for i, name in enumerate(_lib.PROF_CLASSES):
            ms, n, u = C.c_double(), C.c_int64(), C.c_int64()
            check(lib.krk_state_profile_read(self._h, i, C.byref(ms), C.byref(n)))
            check(lib.krk_state_profile_units(self._h, i, C.byref(u)))
            out[name] = (ms.value, n.value, u.value)
        return out

    def close(self) -> None:
        if self._h:
            lib.krk_state_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ generation
@dataclass
class SamplerConfig:
    """src/sampler.rs:5-26.  seed None draws a seed from the OS, as the
    reference's StdRng::from_entropy."""

    temperature: float = 0.7
    top_p: float = 0.95
    top_k: int = 50
    repetition_penalty: float = 1.2
    eos_token_id: int = EOS_TOKEN
    seed: Optional[int] = None


@dataclass
class GenerationOptions:
    """src/generate.rs:8-23."""

    max_new_tokens: int = 128
    sampler_config: SamplerConfig = field(default_factory=SamplerConfig)
    stream_stdout: bool = True  # print each token's text (needs the engine's tokenizer)


@dataclass
class GenerationResult:
    """src/generate.rs:25-34.  generated_text is the concatenated decode_token
    text of the generated tokens (empty without a tokenizer).  The device
    sampling loop runs prefill and decode in one call: its decode_duration
    covers both."""

    generated_tokens: List[int]
    prefill_duration: float
    decode_duration: float
    prompt_token_count: int
    generated_token_count: int
    tokens_per_second: float
    generated_text: str = ""


class GenerationEngine:
    """src/generate.rs:36-133 for one sequence.  With a tokenizer (the
    reference's GenerationEngine::new(&model, &tokenizer)) each token's text is
    streamed to stdout (options.stream_stdout), passed to on_token and
    collected in generated_text; without one, on_token receives token ids."""

    def __init__(self, model: PebbleModel, tokenizer=None):
        self.model = model
        self.tokenizer = tokenizer

    def generate_with_callback(self, prompt_tokens: Sequence[int], state: PebbleState, options: GenerationOptions,
                               on_token) -> GenerationResult:
        return self.generate(prompt_tokens, state, options, on_token)

    def _emitter(self, options: GenerationOptions, on_token, text: List[str]):
        tok = self.tokenizer

        def emit(t: int) -> None:
            if tok is None:
                if on_token:
                    on_token(t)
                return
            try:
                s = tok.decode_token(t)
            except KrikilError:  # src/generate.rs:89-92: a token that does not decode prints nothing
                s = ""
            if options.stream_stdout:
                import sys
                sys.stdout.write(s)
                sys.stdout.flush()
            if on_token:
                on_token(s)
            text.append(s)
        return emit

    def generate(self, prompt_tokens: Sequence[int], state: PebbleState, options: GenerationOptions,
                 on_token=None) -> GenerationResult:
        text: List[str] = []
        emit = self._emitter(options, on_token, text)
        sc = options.sampler_config
        if sc.temperature > 1e-6:
            # the whole loop on the device (krk_generate_sample), then the callbacks
            if state.batch != 1:
                raise ValueError("GenerationEngine.generate runs one sequence")
            if sc.eos_token_id != EOS_TOKEN:
                raise ValueError(f"the device loop stops at token {EOS_TOKEN}")
            t0 = time.perf_counter()
            out = self.model.generate_sample([list(prompt_tokens)], state, options.max_new_tokens, sc.temperature,
                                             sc.top_p, sc.top_k, sc.repetition_penalty,
                                             None if sc.seed is None else [sc.seed])[0]
            dt = time.perf_counter() - t0
            for t in out:
                emit(t)
            return GenerationResult(out, 0.0, dt, len(prompt_tokens), len(out), len(out) / dt if dt > 0 else 0.0,
                                    "".join(text))
        state.reset()
        all_tokens = list(int(t) for t in prompt_tokens)
        t0 = time.perf_counter()
        logits = self.model.forward_prefill(prompt_tokens, state)
        prefill = time.perf_counter() - t0
        nxt = greedy_host(logits, all_tokens, sc.repetition_penalty)
        out: List[int] = []
        t1 = time.perf_counter()
        while len(out) < options.max_new_tokens:
            if nxt == sc.eos_token_id:
                break
            out.append(nxt)
            all_tokens.append(nxt)
            emit(nxt)
            if state.current_pos >= state.context_limit:
                break
            logits = self.model.forward_step(nxt, state)
            nxt = greedy_host(logits, all_tokens, sc.repetition_penalty)
        dec = time.perf_counter() - t1
        return GenerationResult(out, prefill, dec, len(prompt_tokens), len(out), len(out) / dec if dec > 0 else 0.0,
                                "".join(text))


def greedy_host(logits: np.ndarray, context: Sequence[int], penalty: float) -> int:
    """src/sampler.rs:50-80 on host logits (used by GenerationEngine)."""
    lg = np.array(logits, dtype=np.float32)
    if abs(np.float32(penalty) - np.float32(1.0)) > np.float32(1e-4):
        p = np.float32(penalty)
        for t in set(int(c) for c in context):
            if t < lg.size:
                lg[t] = lg[t] / p if lg[t] > 0 else lg[t] * p
    # first maximum; NaN never wins and an all -inf/NaN row gives 0
    return int(np.argmax(np.where(np.isnan(lg), -np.inf, lg)))
