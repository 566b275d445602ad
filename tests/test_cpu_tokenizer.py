"""The tokenizer (cuinf_tokenizer_*) against the reference's own
src/tokenizer.h: the committed fixtures hold the ids the reference tokenizer
gave for a list of strings on a small trained byte-level BPE
(tests/golden/make_tok_golden.py); when oracle/_ref/libreftok.so is built
here, seeded random strings are compared with it directly.  Decoding returns
the original bytes; on plain ASCII text the ids equal the `tokenizers`
library's own encoding of the same tokenizer.json."""
import ctypes
import json
import os
import random

import pytest

from cuda_inf_b200.tokenizer import Tokenizer, chat_prompt

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
TOK = os.path.join(HERE, "golden", "tok")
REF = os.path.join(ROOT, "oracle", "_ref", "libreftok.so")


@pytest.fixture(scope="module")
def tk():
    return Tokenizer(TOK)


def test_fixture_cases_match_reference(tk):
    cases = json.load(open(os.path.join(HERE, "golden", "tok_expected.json"), encoding="utf-8"))["cases"]
    assert len(cases) >= 10
    for c in cases:
        assert tk.encode(c["text"]) == c["ids"], c["text"]
        assert tk.decode(c["ids"]) == c["text"]


def test_special_tokens_and_skip(tk):
    ids = tk.encode("<|im_start|>user\nhi<|im_end|>")
    text = tk.decode(ids)
    assert text == "<|im_start|>user\nhi<|im_end|>"
    assert tk.decode(ids, skip_special=True) == "user\nhi"
    assert tk.encode("") == []
    assert tk.decode([10 ** 6, -1]) == ""  # unknown ids are skipped


def test_chat_prompt_template():
    assert chat_prompt("Hi there") == ("<|startoftext|><|im_start|>user\nHi there<|im_end|>\n"
                                       "<|im_start|>assistant\n")


@pytest.mark.skipif(not os.path.exists(REF), reason="reference tokenizer not built (make -C oracle ref)")
def test_random_strings_match_reference(tk):
    ref = ctypes.CDLL(REF)
    ref.reftok_load.restype = ctypes.c_void_p
    ref.reftok_load.argtypes = [ctypes.c_char_p]
    ref.reftok_encode.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    h = ref.reftok_load(TOK.encode())
    pool = (list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") + list(" \t\n\r'.,;:!?()[]{}+-*/#\"") +
            ["é", "ï", "ü", "東", "京", "п", "🙂", "λ", " ", "'s", "'ll", "<|im_end|>", "<|startoftext|>"])
    r = random.Random(12)
    for _ in range(400):
        s = "".join(r.choice(pool) for _ in range(r.randint(0, 40)))
        b = s.encode("utf-8")
        buf = (ctypes.c_int * 1024)()
        n = ref.reftok_encode(h, b, len(b), buf, 1024)
        assert tk.encode(s) == list(buf[:n]), repr(s)
        assert tk.decode(tk.encode(s)) == s


def test_ascii_matches_tokenizers_library(tk):
    tokenizers = pytest.importorskip("tokenizers")
    hf = tokenizers.Tokenizer.from_file(os.path.join(TOK, "tokenizer.json"))
    r = random.Random(3)
    words = ["the", "engine", "kernel", "cache", "Decode", "tensor", "x", "42", "2024", "it's", "a+b"]
    for _ in range(200):
        s = " ".join(r.choice(words) for _ in range(r.randint(1, 12)))
        assert tk.encode(s) == hf.encode(s).ids, s
