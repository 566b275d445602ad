"""Tokenizer of the reference (src/tokenizer.h): byte-level BPE over the
files tools/export_tokenizer.py writes from tokenizer.json.  The work is in
libcuinf.so (cuinf_tokenizer_*); `export_files` writes those files from a
tokenizer.json."""
import ctypes
import json
import os

from ._lib import check, lib


def export_files(tokenizer_json, out_dir):
    """vocab.tsv (<id>\\t<token>), merges.tsv (<rank>\\t<left>\\t<right>) and
    special.tsv (<id>\\t<content> of the added tokens) from a tokenizer.json,
    the layout of the reference's tools/export_tokenizer.py."""
    T = json.load(open(tokenizer_json, encoding="utf-8"))
    os.makedirs(out_dir, exist_ok=True)
    vocab = T["model"]["vocab"]
    with open(os.path.join(out_dir, "vocab.tsv"), "w", encoding="utf-8", newline="\n") as f:
        for tok, i in sorted(vocab.items(), key=lambda kv: kv[1]):
            f.write(f"{i}\t{tok}\n")
    with open(os.path.join(out_dir, "merges.tsv"), "w", encoding="utf-8", newline="\n") as f:
        for r, m in enumerate(T["model"]["merges"]):
            a, b = m.split(" ", 1) if isinstance(m, str) else (m[0], m[1])
            f.write(f"{r}\t{a}\t{b}\n")
    with open(os.path.join(out_dir, "special.tsv"), "w", encoding="utf-8", newline="\n") as f:
        for a in T.get("added_tokens", []):
            f.write(f"{a['id']}\t{a['content']}\n")


class Tokenizer:
    def __init__(self, directory):
        h = ctypes.c_void_p()
        check(lib().cuinf_tokenizer_load(directory.encode(), ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().cuinf_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def vocab_size(self):
        return lib().cuinf_tokenizer_vocab_size(self._h)

    def encode(self, text):
        b = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        n = ctypes.c_int(0)
        check(lib().cuinf_tokenizer_encode(self._h, b, len(b), None, 0, ctypes.byref(n)))
        ids = (ctypes.c_int * max(1, n.value))()
        check(lib().cuinf_tokenizer_encode(self._h, b, len(b), ids, n.value, ctypes.byref(n)))
        return list(ids[:n.value])

    def decode_bytes(self, ids, skip_special=False):
        arr = (ctypes.c_int * max(1, len(ids)))(*ids)
        ln = ctypes.c_size_t(0)
        check(lib().cuinf_tokenizer_decode(self._h, arr, len(ids), int(skip_special), None, 0, ctypes.byref(ln)))
        buf = ctypes.create_string_buffer(max(1, ln.value))
        check(lib().cuinf_tokenizer_decode(self._h, arr, len(ids), int(skip_special), buf, ln.value,
                                           ctypes.byref(ln)))
        return buf.raw[:ln.value]

    def decode(self, ids, skip_special=False):
        return self.decode_bytes(ids, skip_special).decode("utf-8", errors="replace")


def chat_prompt(user):
    """The reference's single-turn chat template (engine.cu:697-699)."""
    b = user.encode("utf-8")
    ln = ctypes.c_size_t(0)
    check(lib().cuinf_chat_prompt(b, None, 0, ctypes.byref(ln)))
    buf = ctypes.create_string_buffer(ln.value)
    check(lib().cuinf_chat_prompt(b, buf, ln.value, ctypes.byref(ln)))
    return buf.raw[:ln.value].decode("utf-8")
