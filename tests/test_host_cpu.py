"""The C host (gemma4.c_b200/host/run.c): its tokenizer against the reference's
own tokenize() (gemma4.c:61-109) on a crafted tokenizer section, and the
command line's argument handling. No GPU needed."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gemma4.c_b200")

SECTION = 33429932
TEXT = 94
OFF_TEXTS = 12
OFF_SPECIALS = OFF_TEXTS + 262144 * TEXT
OFF_ENCODE = OFF_SPECIALS + 256 * 100
OFF_MERGES = OFF_ENCODE + 32768 * 16


def build_section(rng):
    """A tokenizer section with special tokens, a direct vocabulary of UTF-8
    pieces (ASCII letters, U+2581, a few multi-byte characters) and merges of
    random pairs, keys sorted as the exporter sorts them (bytewise)."""
    sec = np.zeros(SECTION, np.uint8)
    specials = [("<|turn>", 105), ("<turn|>", 106), ("<bos>", 2), ("<|tool>", 48)]
    pieces = [c.encode() for c in "abcdefghijklmnopqrstuvwxyzT?"] + ["▁".encode(), "é".encode(),
                                                                        "€".encode(), "😀".encode()]
    ids = {p: 1000 + i for i, p in enumerate(pieces)}
    enc = sorted((p.ljust(8, b"\0"), ids[p]) for p in pieces)
    base = sorted(set(ids.values())) + [238 + b for b in b"\n|<>"]
    merges, nxt = {}, 5000
    for _ in range(300):
        a, b = int(rng.choice(base)), int(rng.choice(base))
        key = np.array([a, b], np.int32).tobytes()
        if key not in merges:
            merges[key] = (nxt, int(rng.integers(0, 1000)))
            base.append(nxt)
            nxt += 1
    mer = sorted(merges.items())
    hdr = np.array([len(mer), len(enc), len(specials)], np.int32)
    sec[:12] = hdr.view(np.uint8)
    for i, (t, id_) in enumerate(specials):
        o = OFF_SPECIALS + i * 100
        sec[o:o + len(t)] = np.frombuffer(t.encode(), np.uint8)
        sec[o + 96:o + 100] = np.array([id_], np.int32).view(np.uint8)
    for i, (k, r) in enumerate(enc):
        o = OFF_ENCODE + i * 16
        sec[o:o + 8] = np.frombuffer(k, np.uint8)
        sec[o + 8:o + 16] = np.array([r, 0], np.int32).view(np.uint8)
    for i, (k, (r, rank)) in enumerate(mer):
        o = OFF_MERGES + i * 16
        sec[o:o + 8] = np.frombuffer(k, np.uint8)
        sec[o + 8:o + 16] = np.array([r, rank], np.int32).view(np.uint8)
    return sec


@pytest.fixture(scope="module")
def tok_lib():
    path = os.path.join(PKG, "libg4tok.so")
    if not os.path.exists(path):
        subprocess.run(["make", "-C", PKG, "libg4tok.so"], check=True, capture_output=True)
    L = C.CDLL(path)
    L.g4tok_encode.argtypes = [C.c_void_p, C.POINTER(C.c_char_p), np.ctypeslib.ndpointer(np.int32), C.c_int]
    L.g4tok_encode.restype = C.c_int
    return L


PROMPTS = [
    "Why is the sky blue?",
    "<|turn>user\nabc def<turn|>\n<|turn>model\n",
    "héllo wörld € 😀 <|tool> <unknown|> <<>> ||",
    "",
    " ",
    "aaaaaaaa bbbbbbbb zzzz TTTT ????",
    "\x01\x02\x7f binary-ish \xc3\xa9 " * 20,
]


def test_tokenizer_matches_reference(tok_lib, reference):
    rng = np.random.default_rng(5)
    sec = build_section(rng)
    ref = reference.lib
    ref.tokenize.argtypes = [C.c_void_p, C.POINTER(C.c_char_p), np.ctypeslib.ndpointer(np.int32), C.c_int]
    ref.tokenize.restype = C.c_int
    for prompt in PROMPTS:
        for segs in ((b"", prompt.encode(), b""), (b"<|turn>user\n", prompt.encode(), b"<turn|>\n<|turn>model\n")):
            arr = (C.c_char_p * 3)(*segs)
            a = np.zeros(4096, np.int32)
            b = np.zeros(4096, np.int32)
            na = tok_lib.g4tok_encode(sec.ctypes.data, arr, a, 4096)
            nb = ref.tokenize(sec.ctypes.data, arr, b, 4096)
            assert na == nb, (prompt, na, nb)
            assert np.array_equal(a[:na], b[:nb]), prompt
    # capacity limits: both refuse the same way
    arr = (C.c_char_p * 3)(b"", b"abcdefgh" * 4, b"")
    for cap in (1, 2, 5, 33, 34):
        a = np.zeros(64, np.int32)
        b = np.zeros(64, np.int32)
        assert tok_lib.g4tok_encode(sec.ctypes.data, arr, a, cap) == ref.tokenize(sec.ctypes.data, arr, b, cap)


def test_zeroed_section_gives_byte_tokens(tok_lib):
    """The synthetic model's section is all zeros: <bos> then one byte token per
    byte, a space spelled as U+2581 (three bytes)."""
    sec = np.zeros(SECTION, np.uint8)
    text = "Hi there é"
    arr = (C.c_char_p * 3)(b"", text.encode(), b"")
    out = np.zeros(64, np.int32)
    n = tok_lib.g4tok_encode(sec.ctypes.data, arr, out, 64)
    assert list(out[:n]) == [2] + [238 + b for b in text.replace(" ", "\u2581").encode()]


def test_run_rejects_missing_model():
    exe = os.path.join(PKG, "run")
    if not os.path.exists(exe):
        subprocess.run(["make", "-C", PKG, "run"], check=True, capture_output=True)
    r = subprocess.run([exe, "-m", os.path.join(ROOT, "no-such-model.bin"), "--bench", "8", "1"],
                       capture_output=True, text=True)
    assert r.returncode == 1 and "no-such-model.bin" in r.stderr
