"""Tokenizer fixtures: a small byte-level BPE tokenizer trained here with the
`tokenizers` library on a seeded synthetic corpus (the checkpoint's
tokenizer.json is not available), exported to the reference's tsv files with
cuda_inf_b200.tokenizer.export_files, and the ids the REFERENCE tokenizer
(src/tokenizer.h, built unmodified into oracle/_ref/libreftok.so by
`make -C oracle ref`) gives for a list of test strings.

    python tests/golden/make_tok_golden.py     # writes tests/golden/tok/ and tok_expected.json
"""
import ctypes
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

SPECIALS = ["<|startoftext|>", "<|endoftext|>", "<|im_start|>", "<|im_end|>"]

WORDS = ("the of and to in is was for on that with as by at from it this be are or an have not "
         "engine kernel tensor memory token layer expert router cache group scale decode prefill "
         "weight value vector matrix shared thread warp block cluster stream graph launch").split()
EXTRA = ["café", "naïve", "Zürich", "Ångström", "東京", "数据", "привет", "🙂", "λx", "über"]


def corpus(n, seed=0):
    r = random.Random(seed)
    lines = []
    for _ in range(n):
        parts = []
        for _ in range(r.randint(3, 14)):
            k = r.random()
            if k < 0.7:
                w = r.choice(WORDS)
                parts.append(w.capitalize() if r.random() < 0.15 else w)
            elif k < 0.8:
                parts.append(str(r.randint(0, 99999)))
            elif k < 0.88:
                parts.append(r.choice(EXTRA))
            else:
                parts.append(r.choice(["(x)", "x*2", "a+b", "#", "--", "...", "it's", "we'll", "I'M", "don't"]))
        sep = r.choice([" ", " ", " ", "  ", "\t", "\n", " \n "])
        lines.append(sep.join(parts) + r.choice([".", "!", "?", ":", "", "\n"]))
    return lines


TESTS = [
    "<|startoftext|><|im_start|>user\nWhat is the capital of the cluster? Answer in one sentence.<|im_end|>\n"
    "<|im_start|>assistant\n",
    "The engine decodes 64 tokens per step.",
    "Hello, world! 123 numbers and  multiple   spaces.\nNew line.",
    "def foo(x): return x*2  # comment",
    "it's we'll I'M don't THEY'RE you've",
    "café naïve Zürich 東京 привет 🙂 λx",
    "   leading spaces and trailing   ",
    "tabs\tand\r\nwindows newlines\n\n\nmany",
    "1234567 12 3",
    "<|im_end|><|im_start|><|endoftext|>",
    "",
    "a",
    "((nested)) [brackets] {braces} <angle>",
    "x\n  y\n\n  z",
]


def main():
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers
    from cuda_inf_b200.tokenizer import export_files
    tok = Tokenizer(models.BPE(ignore_merges=True))
    # the split the reference's pre-tokenizer implements (tokenizer.h:104-152), then byte-level
    pattern = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"
               r"|\s*[\r\n]+|\s+(?!\S)|\s+")
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(pattern), behavior="isolated"),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=700, special_tokens=SPECIALS,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(corpus(4000), trainer=trainer)
    out = os.path.join(HERE, "tok")
    os.makedirs(out, exist_ok=True)
    tok.save(os.path.join(out, "tokenizer.json"))
    export_files(os.path.join(out, "tokenizer.json"), out)
    ref = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libreftok.so"))
    ref.reftok_load.restype = ctypes.c_void_p
    ref.reftok_load.argtypes = [ctypes.c_char_p]
    ref.reftok_encode.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int]
    h = ref.reftok_load(out.encode())
    assert h
    expected = []
    for t in TESTS:
        b = t.encode("utf-8")
        buf = (ctypes.c_int * 4096)()
        n = ref.reftok_encode(h, b, len(b), buf, 4096)
        expected.append({"text": t, "ids": list(buf[:n])})
    json.dump({"generator": "tests/golden/make_tok_golden.py", "cases": expected},
              open(os.path.join(HERE, "tok_expected.json"), "w"), indent=0, ensure_ascii=False)
    print("vocab", tok.get_vocab_size(), "cases", len(expected))


if __name__ == "__main__":
    main()
