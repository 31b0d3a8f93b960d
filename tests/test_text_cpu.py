"""The text front end on the CPU: tokenizer (src/tokenizer.rs) and chat
template (src/template.rs), native code in the C-ABI library.

Pinned by golden vectors from the `tokenizers` crate itself (its Python
binding, tests/golden/make_text_golden.py) on a BPE trained for the tests and
on the Pebble-25M tokenizer.json, the reference's own known-answer tests
(src/tokenizer.rs:85-108, src/template.rs:82-96), and Jinja2 renderings of
the supported template constructs."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from krikil_rs_b200 import _lib
from krikil_rs_b200._lib import KrikilError, lib
from krikil_rs_b200.text import (DEFAULT_CHAT_TEMPLATE, DEFAULT_EOS_TOKEN_ID, ChatMessage, ChatTemplateEngine,
                                 PebbleTokenizer)

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, name), encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def small():
    return PebbleTokenizer.from_file(os.path.join(GOLDEN, "tokenizer_small.json")), _load("tokenizer_small_cases.json")


def _pebble_path():
    cases = _load("tokenizer_pebble_cases.json")
    p = os.environ.get("KRIKIL_PEBBLE_TOKENIZER", cases["source_path"])
    return (p if os.path.exists(p) else None), cases


def test_small_encode_matches_tokenizers_crate(small):
    tok, cases = small
    bad = [(c["text"], tok.encode(c["text"]), c["ids"]) for c in cases["encode"] if tok.encode(c["text"]) != c["ids"]]
    assert not bad, bad[:3]
    assert len(cases["encode"]) > 600


def test_small_decode_matches_tokenizers_crate(small):
    tok, cases = small
    for c in cases["decode"]:
        assert tok.decode(c["ids"]) == c["skip"], c["ids"]
        assert tok._decode(c["ids"], False) == c["keep"], c["ids"]
    for c in cases["decode_token"]:
        assert tok.decode_token(c["id"]) == c["text"], c["id"]


def test_small_added_tokens_and_sizes(small):
    tok, cases = small
    assert tok.eos_token_id() == cases["eos_token_id"] == 0
    assert tok.vocab_size() == cases["vocab_size"]
    tool = tok.token_to_id("<tool>")
    assert tool is not None and tok.token_to_id("no such token") is None
    # lstrip/rstrip: the spaces around "<tool>" belong to it
    assert tok.encode("x  <tool>  y") == tok.encode("x") + [tool] + tok.encode("y")
    # the special token is dropped by decode, kept by decode_token
    ids = tok.encode("a<|eos|>b")
    assert 0 in ids and tok.decode(ids) == "ab" and tok.decode_token(0) == "<|eos|>"


def test_pebble_reference_known_answer():
    """src/tokenizer.rs:85-108 on the Pebble-25M tokenizer.json."""
    path, _ = _pebble_path()
    if path is None:
        pytest.skip("Pebble-25M tokenizer.json not available")
    tok = PebbleTokenizer.from_file(path)
    assert tok.eos_token_id() == 0
    text = "user: What is the capital of France? assistant: "
    ids = tok.encode(text)
    assert ids == [397, 264, 26, 1270, 311, 263, 1530, 1360, 284, 420, 82, 549, 31, 842, 373, 419, 26, 221]
    assert tok.decode(ids) == text
    assert tok.vocab_size() == 2048


def test_pebble_golden_cases():
    path, cases = _pebble_path()
    if path is None:
        pytest.skip("Pebble-25M tokenizer.json not available")
    tok = PebbleTokenizer.from_file(path)
    for c in cases["encode"]:
        assert tok.encode(c["text"]) == c["ids"], c["text"]
    for c in cases["decode"]:
        assert tok.decode(c["ids"]) == c["skip"] and tok._decode(c["ids"], False) == c["keep"], c["ids"]


def test_encode_rejects_invalid_utf8(small):
    tok, _ = small
    ids = np.zeros(8, dtype=np.uint32)
    n = C.c_size_t(0)
    for raw in (b"\xff", b"a\xc3", b"\xed\xa0\x80", b"\xf4\x90\x80\x80", b"\xc0\xaf"):
        rc = lib.krk_tokenizer_encode(tok._h, raw, len(raw), ids.ctypes.data, ids.size, C.byref(n))
        assert rc == _lib.INVALID and b"Failed to encode text" in lib.krk_last_error()


def test_buffer_rules(small):
    tok, _ = small
    text = b"hello world, hello"
    n = C.c_size_t(0)
    assert lib.krk_tokenizer_encode(tok._h, text, len(text), None, 0, C.byref(n)) == _lib.OK
    need = n.value
    assert 0 < need <= len(text)
    small_buf = np.zeros(need - 1, dtype=np.uint32)
    assert lib.krk_tokenizer_encode(tok._h, text, len(text), small_buf.ctypes.data, small_buf.size,
                                    C.byref(n)) == _lib.INVALID
    ids = (C.c_uint32 * 2)(1, 2)
    ln = C.c_size_t(0)
    assert lib.krk_tokenizer_decode(tok._h, ids, 2, 1, None, 0, C.byref(ln)) == _lib.OK
    buf = C.create_string_buffer(ln.value)  # no room for the NUL: still fine
    assert lib.krk_tokenizer_decode(tok._h, ids, 2, 1, buf, ln.value, C.byref(ln)) == _lib.OK
    assert lib.krk_tokenizer_decode(tok._h, ids, 2, 1, buf, max(0, ln.value - 1), C.byref(ln)) == _lib.INVALID


def test_load_errors(tmp_path):
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(tmp_path / "missing.json")
    assert e.value.status == _lib.IO and "Failed to load tokenizer from" in e.value.message
    assert "No such file or directory" in e.value.message
    bad = tmp_path / "bad.json"
    bad.write_text('{"model": {"type": "WordPiece"}}')
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(bad)
    assert e.value.status == _lib.IO
    bad.write_text('{"model": ')
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(bad)
    assert "invalid JSON" in e.value.message


def test_unsupported_tokenizer_files_are_refused(tmp_path):
    """Only what the Pebble tokenizer uses is implemented; anything else fails
    at load with a message naming it rather than tokenizing differently."""
    import copy
    base = _load("tokenizer_small.json")
    cases = [("normalizer", {"type": "NFC"}, "normalizer"),
             ("pre_tokenizer", {"type": "Whitespace"}, "pre_tokenizer"),
             ("decoder", {"type": "WordPiece"}, "decoder"),
             ("model.dropout", 0.1, "dropout"),
             ("model.byte_fallback", True, "byte_fallback"),
             ("model.unk_token", "<unk>", "unk_token"),
             ("model.continuing_subword_prefix", "##", "continuing_subword_prefix")]
    for key, val, needle in cases:
        d = copy.deepcopy(base)
        if key.startswith("model."):
            d["model"][key[6:]] = val
        else:
            d[key] = val
        f = tmp_path / "t.json"
        f.write_text(json.dumps(d))
        with pytest.raises(KrikilError) as e:
            PebbleTokenizer.from_file(f)
        assert e.value.status == _lib.IO and needle in e.value.message, (key, e.value.message)
    d = copy.deepcopy(base)
    d["added_tokens"][0]["single_word"] = True
    (tmp_path / "t.json").write_text(json.dumps(d))
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(tmp_path / "t.json")
    assert "single_word" in e.value.message
    d = copy.deepcopy(base)
    d["model"]["merges"] = d["model"]["merges"] + [["zzq", "qqz"]]
    (tmp_path / "t.json").write_text(json.dumps(d))
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(tmp_path / "t.json")
    assert "merge token missing from vocab" in e.value.message
    # merges written as "a b" strings (the older file format) load and encode the same
    d = copy.deepcopy(base)
    d["model"]["merges"] = [" ".join(m) for m in d["model"]["merges"]]
    (tmp_path / "t.json").write_text(json.dumps(d))
    a = PebbleTokenizer.from_file(tmp_path / "t.json")
    b = PebbleTokenizer.from_file(os.path.join(GOLDEN, "tokenizer_small.json"))
    for text in ("the cat sat on the mat", "they're going home!", "Москва 1234"):
        assert a.encode(text) == b.encode(text)


@pytest.mark.parametrize("text", ['{"a": "x', '{"a": "\\q"}', '{"a": "\\ud800"}', '{"a": 1,}', '[1 2]',
                                  '{"a": tru}', '{} {}', '{"a": "\x01"}', '[' * 600 + ']' * 600, '-', '{"a": 1e}'])
def test_malformed_json_is_refused(tmp_path, text):
    """The tokenizer file reader rejects malformed JSON (and nesting beyond 512
    levels) with a positioned message instead of reading past it."""
    f = tmp_path / "t.json"
    f.write_text(text)
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.from_file(f)
    assert e.value.status == _lib.IO and "invalid JSON" in e.value.message and "at byte" in e.value.message


def test_resolve_path(tmp_path, monkeypatch):
    """src/tokenizer.rs:54-79: explicit path, the model's sibling, ./tokenizer.json."""
    model = tmp_path / "m" / "model.safetensors"
    model.parent.mkdir()
    monkeypatch.chdir(tmp_path)
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.resolve_path(model)
    assert e.value.message == (f"Could not find tokenizer.json. Looked at {model.parent}/tokenizer.json and "
                               "tokenizer.json. Use --tokenizer to specify its path.")
    (tmp_path / "tokenizer.json").write_text("{}")
    assert PebbleTokenizer.resolve_path(model) == "tokenizer.json"
    (model.parent / "tokenizer.json").write_text("{}")
    assert PebbleTokenizer.resolve_path(model) == f"{model.parent}/tokenizer.json"
    assert PebbleTokenizer.resolve_path("model.safetensors") == "tokenizer.json"
    with pytest.raises(KrikilError) as e:
        PebbleTokenizer.resolve_path(model, tmp_path / "nope.json")
    assert e.value.message == f"Explicit tokenizer path not found: {tmp_path}/nope.json"
    assert PebbleTokenizer.resolve_path(model, tmp_path / "tokenizer.json") == f"{tmp_path}/tokenizer.json"


def test_default_template_reference_tests():
    """src/template.rs:82-96."""
    e = ChatTemplateEngine.default_template()
    assert e.render_user_prompt("What is the capital of France?") == "user: What is the capital of France? assistant: "
    msgs = [ChatMessage.user("Hello"), ChatMessage.assistant("Hi there!"), ChatMessage.user("How are you?")]
    assert e.render(msgs, True) == "user: Hello assistant: Hi there! user: How are you? assistant: "
    assert e.render(msgs, False) == "user: Hello assistant: Hi there! user: How are you? "
    assert e.render([ChatMessage("system", "be brief")], False) == "system: be brief "
    assert DEFAULT_EOS_TOKEN_ID == 0 and "add_generation_prompt" in DEFAULT_CHAT_TEMPLATE


def test_template_cases_match_jinja():
    for c in _load("chat_template_cases.json")["cases"]:
        e = ChatTemplateEngine(c["template"])
        got = e.render([ChatMessage(r, t) for r, t in c["messages"]], c["add_generation_prompt"])
        assert got == c["expected"], c["template"]


def test_template_minijinja_printing_and_errors(tmp_path):
    assert ChatTemplateEngine("{{ 1 == 1 }} {{ none }} {{ x }} {{ 2.5 }} {{ 3.0 }}").render([], False) == \
        "true none  2.5 3.0"
    assert ChatTemplateEngine("a\n").render([], False) == "a"  # one trailing newline dropped
    for src in ("{% if x %}", "{{ 1 + }}", "{% for %}{% endfor %}", "{% frobnicate %}", "{{ 'a }}"):
        with pytest.raises(KrikilError) as e:
            ChatTemplateEngine(src).render([], False)
        assert e.value.message.startswith("Failed to parse Jinja chat template"), src
    for src in ("{{ raise_exception('no system role') }}", "{{ x.y }}", "{{ 1 + 'a' }}", "{{ 1 // 0 }}"):
        with pytest.raises(KrikilError) as e:
            ChatTemplateEngine(src).render([], False)
        assert e.value.message.startswith("Failed to render Jinja chat template"), src
    for src in ("{{ " + "(" * 5000 + "1" + ")" * 5000 + " }}", "{% if x %}" * 3000 + "{% endif %}" * 3000,
                "{{ " + "-" * 5000 + "1 }}", "{{ " + "not " * 5000 + "x }}", "{{ " + "[" * 5000 + "]" * 5000 + " }}"):
        with pytest.raises(KrikilError) as e:  # deep nesting is refused, not a stack overflow
            ChatTemplateEngine(src).render([], False)
        assert "nested too deeply" in e.value.message
    assert ChatTemplateEngine("{{ " + "(" * 50 + "1" + ")" * 50 + " }}").render([], False) == "1"
    with pytest.raises(KrikilError) as e:
        ChatTemplateEngine.from_file(tmp_path / "none.jinja")
    assert "Failed to read chat template from" in e.value.message


def test_text_header_symbols_exported():
    import re
    with open(os.path.join(os.path.dirname(GOLDEN), "..", "include", "krikil_text.h")) as f:
        names = sorted(set(re.findall(r"KRK_API\s+[\w\s\*]+?\b(krk_\w+)\s*\(", f.read())))
    assert len(names) == 10
    for n in names:
        assert hasattr(lib, n) and n in _lib.EXPORTED, n
