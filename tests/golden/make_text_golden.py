"""Golden vectors for the text front end (tokenizer and chat template).

The reference tokenizes with the `tokenizers` crate 0.21.4 (Cargo.lock:943-944;
src/tokenizer.rs) and renders chat templates with minijinja 2.x
(src/template.rs).  The Python binding of the same `tokenizers` crate is the
generator for the tokenizer cases; Jinja2 renders the template cases (only
constructs on which Jinja2 and minijinja agree).

Writes, next to this script:
  tokenizer_small.json        a byte-level BPE trained here on seeded
                              synthetic text (700 ids, the special token
                              "<|eos|>" and a non-special "<tool>" added
                              token with lstrip/rstrip)
  tokenizer_small_cases.json  its encode / decode results
  tokenizer_pebble_cases.json encode / decode results of the Pebble-25M
                              tokenizer.json (ids only; the test reads the
                              vocabulary from the path recorded here, or from
                              $KRIKIL_PEBBLE_TOKENIZER)
  chat_template_cases.json    templates, their inputs and rendered text

Run:  python tests/golden/make_text_golden.py /path/to/krikil-rs
"""
import json
import os
import random
import sys

from tokenizers import AddedToken, Tokenizer, decoders, models, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))

PIECES = list("abcdefghijklmnopqrstuvwxyzABCDEFXYZ0123456789 .,;:!?-'\"()[]{}<>|/\\\n\t") + [
    "'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'RE", "  ", "   ", " \n", "\r\n", "\n\n", "\t\t",
    "é", "ö", "ß", "Ω", "ж", "日本", "語", "한", "🙂", "👍🏽", "١٢٣", "²", "½", "Ⅻ", "́", " ", "　",
    " ", "\u0085", "\u001c", "\u0000", "​", "İ", "ǅ", "ﬁ", "<|eos|>", "<tool>", " <tool> ", "<|eos",
]
WORDS = ["the", "cat", "sat", "on", "mat", "they", "re", "going", "home", "I", "ll", "be", "there", "don", "t",
         "capital", "of", "France", "is", "Paris", "what", "user", "assistant", "hello", "world", "1234", "3.14",
         "Москва", "東京", "naïve", "café", "x", "y", "z"]


def corpus(rng, n):
    out = []
    for _ in range(n):
        w = [rng.choice(WORDS) for _ in range(rng.randint(3, 14))]
        s = " ".join(w)
        if rng.random() < 0.3:
            s = s.replace(" re", "'re").replace(" t ", "'t ").replace(" ll", "'ll")
        out.append(s + rng.choice([".", "?", "!", "", "\n"]))
    return out


def random_text(rng):
    n = rng.randint(0, 30)
    parts = [rng.choice(PIECES) if rng.random() < 0.6 else rng.choice(WORDS) for _ in range(n)]
    return "".join(parts) if rng.random() < 0.5 else " ".join(parts)


EDGE_TEXTS = ["", " ", "  ", "   ", "\n", "\n\n", " \n ", "a", " a", "  a", "a ", "a  ", "a  b", "a \n b",
              "'s", "'S", "x's", "x'sx", "''s", "!'s", "they're", "it'll've", "'", "' ", "123abc", "abc123",
              " 1 2 3", "½ ²", "<|eos|>", "<|eos|><|eos|>", "a<|eos|>b", " <|eos|> ", "<|eos", "<tool>",
              "x <tool> y", "x  <tool>  y", "<tool><tool>", " a", "　 a", "á", "🙂 ok",
              "user: What is the capital of France? assistant: "]


def tokenizer_cases(tok, rng, n_random, n_decode, vocab_n):
    enc = []
    for t in EDGE_TEXTS + [random_text(rng) for _ in range(n_random)]:
        enc.append({"text": t, "ids": tok.encode(t, add_special_tokens=False).ids})
    dec = []
    for _ in range(n_decode):
        ids = [rng.randrange(0, vocab_n + 40) for _ in range(rng.randint(0, 16))]
        if rng.random() < 0.3:
            ids.insert(rng.randint(0, len(ids)), 0)
        dec.append({"ids": ids, "skip": tok.decode(ids, skip_special_tokens=True),
                    "keep": tok.decode(ids, skip_special_tokens=False)})
    return enc, dec


def make_small(rng):
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=700, special_tokens=["<|eos|>"], show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(corpus(rng, 4000), trainer)
    tok.add_tokens([AddedToken("<tool>", lstrip=True, rstrip=True, special=False, normalized=False)])
    path = os.path.join(HERE, "tokenizer_small.json")
    tok.save(path, pretty=False)
    return Tokenizer.from_file(path)


TEMPLATE_CASES = [
    # (template, messages, add_generation_prompt)
    ("{% for m in messages %}<{{ m.role }}>{{ m['content'] | trim }}</{{ m.role }}>{% endfor %}"
     "{% if add_generation_prompt %}<assistant>{% endif %}", [["user", "  hi  "], ["assistant", "yo"]], True),
    ("{%- for m in messages -%}\n  {{- loop.index }}/{{ loop.length }}:{{ m.content -}}\n"
     "  {%- if not loop.last %}, {% endif -%}\n{%- endfor %}\n", [["user", "a"], ["user", "b"], ["user", "c"]],
     False),
    ("{% set sep = ' | ' %}{% for m in messages %}{% if loop.first %}[{% endif %}{{ m.role | upper }}{{ sep }}"
     "{{ m.content | length }}{% if loop.last %}]{% endif %}{% endfor %}", [["system", "rules"], ["user", "héllo"]],
     True),
    ("{% if messages | length == 0 %}empty{% elif messages[0].role == 'system' %}sys:{{ messages[0].content }}"
     "{% for m in messages[1:] %} {{ m.role }}={{ m.content }}{% endfor %}{% else %}nosys{% endif %}",
     [["system", "S"], ["user", "U"], ["assistant", "A"]], False),
    ("{% if messages | length == 0 %}empty{% else %}x{% endif %}", [], True),
    ("{{ 'a' ~ 1 ~ 'b' }} {{ 7 // 2 }} {{ 7 % 3 }} {{ -3 + 10 * 2 }} {{ 'yes' if add_generation_prompt else 'no' }}"
     " {% if 'ab' in 'cabd' %}in{% endif %}{% if 'z' not in messages[0].content %}out{% else %}notout{% endif %}",
     [["user", "zzz"]], True),
    ("{% for m in messages %}{{ m.role }}{% else %}none{% endfor %}", [], False),
    ("{# a comment #}{% for m in messages %}{{ m.content | default('d') }}{{ m.missing | default('D') }}"
     "{% if m.missing is defined %}1{% else %}0{% endif %}{% if m.content is string %}1{% endif %}"
     "{% if m.role is not none and not m.missing %}1{% endif %}{% endfor %}",
     [["user", "c"]], False),
    ("{% for m in messages %}{{ m.content[0] }}{{ m.content[-1] }}{{ m.content[1:3] }}{% endfor %}",
     [["user", "abcdef"]], False),
    ("{% for x in range(3) %}{{ x }}{% endfor %}{{ [1, 2, 3] | join('-') }}{{ messages | length }}",
     [["u", "v"]], False),
    ("{% for m in messages %}{% if m.role == 'user' %}user: {% elif m.role == 'assistant' %}assistant: {% else %}"
     "{{ m.role }}: {% endif %}{{ m.content }} {% endfor %}{% if add_generation_prompt %}assistant: {% endif %}",
     [["system", "be brief"], ["user", "Hi"], ["assistant", "Hello"], ["tool", "42"]], True),
]


def render_jinja2(src, msgs, agp):
    import jinja2
    env = jinja2.Environment(keep_trailing_newline=False)
    t = env.from_string(src)
    return t.render(messages=[{"role": r, "content": c} for r, c in msgs], add_generation_prompt=agp)


def main(ref_dir):
    rng = random.Random(20260)
    small = make_small(rng)
    enc, dec = tokenizer_cases(small, rng, 600, 300, small.get_vocab_size(with_added_tokens=True))
    dtok = [{"id": i, "text": small.decode([i], skip_special_tokens=False)}
            for i in range(small.get_vocab_size(with_added_tokens=True))]
    with open(os.path.join(HERE, "tokenizer_small_cases.json"), "w") as f:
        json.dump({"generator": "tokenizers (Python binding of the tokenizers crate)", "encode": enc, "decode": dec,
                   "decode_token": dtok, "eos_token_id": small.token_to_id("<|eos|>"),
                   "vocab_size": small.get_vocab_size(with_added_tokens=True)}, f, ensure_ascii=False)
    print("small:", len(enc), "encode,", len(dec), "decode cases")

    ref_tok = os.path.join(ref_dir, "tokenizer.json")
    if os.path.exists(ref_tok):
        peb = Tokenizer.from_file(ref_tok)
        enc, dec = tokenizer_cases(peb, rng, 400, 200, peb.get_vocab_size(with_added_tokens=True))
        with open(os.path.join(HERE, "tokenizer_pebble_cases.json"), "w") as f:
            json.dump({"generator": "tokenizers (Python binding of the tokenizers crate)",
                       "source_path": os.path.abspath(ref_tok), "encode": enc, "decode": dec,
                       "eos_token_id": peb.token_to_id("<|eos|>"),
                       "vocab_size": peb.get_vocab_size(with_added_tokens=True)}, f, ensure_ascii=False)
        print("pebble:", len(enc), "encode,", len(dec), "decode cases")

    cases = [{"template": s, "messages": m, "add_generation_prompt": a, "expected": render_jinja2(s, m, a)}
             for s, m, a in TEMPLATE_CASES]
    with open(os.path.join(HERE, "chat_template_cases.json"), "w") as f:
        json.dump({"generator": "jinja2", "cases": cases}, f, ensure_ascii=False, indent=1)
    print("templates:", len(cases))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <krikil-rs checkout>")
    main(sys.argv[1])
