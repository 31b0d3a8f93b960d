"""Text front end: the tokenizer and the chat template, mirrors of
src/tokenizer.rs and src/template.rs over the C ABI of include/krikil_text.h
(native code in lib/libkrikil_cuda.so; no GPU involved).

    tok = PebbleTokenizer.from_file(PebbleTokenizer.resolve_path("model.safetensors", None))
    prompt = ChatTemplateEngine.default_template().render_user_prompt("What is the capital of France?")
    ids = tok.encode(prompt)
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from ._lib import INVALID, KrikilError, check, lib

DEFAULT_EOS_TOKEN_ID = 0  # src/tokenizer.rs:5
DEFAULT_CHAT_TEMPLATE = lib.krk_default_chat_template().decode()  # src/template.rs:7


def _read_string(call) -> str:
    """Runs call(buf, cap, len_ptr) under the size-query rule of krikil_text.h."""
    n = C.c_size_t(0)
    cap = 256
    while True:
        buf = C.create_string_buffer(cap + 1)
        rc = call(buf, cap + 1, C.byref(n))
        if rc == INVALID and n.value > cap:
            cap = n.value
            continue
        check(rc)
        return buf.raw[:n.value].decode("utf-8")


class PebbleTokenizer:
    """src/tokenizer.rs:7-80."""

    def __init__(self, handle: C.c_void_p, path: str):
        self._h = handle
        self.path = path

    @classmethod
    def from_file(cls, path) -> "PebbleTokenizer":
        h = C.c_void_p()
        check(lib.krk_tokenizer_load(os.fsencode(path), C.byref(h)))
        return cls(h, os.fspath(path))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            lib.krk_tokenizer_free(h)
            self._h = None

    def encode(self, text: str) -> List[int]:
        data = text.encode("utf-8")
        ids = np.empty(max(1, len(data)), dtype=np.uint32)
        n = C.c_size_t(0)
        check(lib.krk_tokenizer_encode(self._h, data, len(data), ids.ctypes.data, ids.size, C.byref(n)))
        return ids[:n.value].tolist()

    def _decode(self, tokens: Sequence[int], skip_special: bool) -> str:
        ids = np.ascontiguousarray(np.asarray(list(tokens), dtype=np.int64).astype(np.uint32))
        ptr = ids.ctypes.data if ids.size else None
        return _read_string(lambda b, cap, n: lib.krk_tokenizer_decode(self._h, ptr, ids.size, int(skip_special), b,
                                                                       cap, n))

    def decode(self, tokens: Sequence[int]) -> str:
        """Special tokens skipped (src/tokenizer.rs:34-38)."""
        return self._decode(tokens, True)

    def decode_token(self, token: int) -> str:
        """One token, special tokens kept (src/tokenizer.rs:40-44)."""
        return self._decode([token], False)

    def token_to_id(self, token: str) -> Optional[int]:
        v = C.c_int64(0)
        check(lib.krk_tokenizer_token_to_id(self._h, token.encode("utf-8"), C.byref(v)))
        return None if v.value < 0 else int(v.value)

    def eos_token_id(self) -> int:
        v = C.c_uint32(0)
        check(lib.krk_tokenizer_eos_token_id(self._h, C.byref(v)))
        return int(v.value)

    def vocab_size(self) -> int:
        v = C.c_size_t(0)
        check(lib.krk_tokenizer_vocab_size(self._h, C.byref(v)))
        return int(v.value)

    @staticmethod
    def resolve_path(model_path, explicit_tokenizer=None) -> str:
        """src/tokenizer.rs:54-79."""
        mp = os.fsencode(model_path)
        ex = None if explicit_tokenizer is None else os.fsencode(explicit_tokenizer)
        return _read_string(lambda b, cap, n: lib.krk_tokenizer_resolve_path(mp, ex, b, cap, n))


@dataclass
class ChatMessage:
    """src/template.rs:9-29."""
    role: str
    content: str

    @classmethod
    def user(cls, content: str) -> "ChatMessage":
        return cls("user", content)

    @classmethod
    def assistant(cls, content: str) -> "ChatMessage":
        return cls("assistant", content)


class ChatTemplateEngine:
    """src/template.rs:31-79."""

    def __init__(self, template_source: str):
        self.template_source = template_source

    @classmethod
    def from_file(cls, path) -> "ChatTemplateEngine":
        try:
            with open(path, encoding="utf-8") as f:
                return cls(f.read())
        except (OSError, UnicodeDecodeError) as e:
            raise KrikilError(4, f"Failed to read chat template from {os.fspath(path)}: {e}") from e

    @classmethod
    def default_template(cls) -> "ChatTemplateEngine":
        return cls(DEFAULT_CHAT_TEMPLATE)

    def render(self, messages: Sequence[ChatMessage], add_generation_prompt: bool) -> str:
        n = len(messages)
        roles = (C.c_char_p * max(1, n))(*[m.role.encode("utf-8") for m in messages])
        contents = (C.c_char_p * max(1, n))(*[m.content.encode("utf-8") for m in messages])
        src = self.template_source.encode("utf-8")
        return _read_string(lambda b, cap, k: lib.krk_chat_template_render(src, roles, contents, n,
                                                                           int(add_generation_prompt), b, cap, k))

    def render_user_prompt(self, prompt: str) -> str:
        return self.render([ChatMessage.user(prompt)], True)
