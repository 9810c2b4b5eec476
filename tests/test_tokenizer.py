"""The host tokenizer (n550_tok_*) against the reference's own tokenizer.c,
compiled from the reference checkout into oracle/_ref/libref_tok.so, on the
reference's exported Qwen3 vocabulary (tok.bin, copied to oracle/_ref/):
identical token ids and decoded bytes on the reference's golden prompt
(main.c:118-119), on thousands of seeded random texts that mix the
pre-tokenizer's cases (letters, contractions, digits, symbol runs, spaces and
newlines, CJK, accented Latin, emoji, invalid UTF-8, special tokens), on the
chat template (main.c:124-131), and on the error cases. CPU only."""
import numpy as np
import pytest

import oracle
import n550_qwen3_bringup_handover_b200 as n5

pytestmark = pytest.mark.skipif(not oracle.tokenizer_available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def toks():
    return n5.Tokenizer(oracle.TOK_PATH), oracle.RefTokenizer()


WORDS = ["hello", "World", "the", "GPU", "tensor", "B200", "naïve", "café", "Ünïcödé", "straße",
         "Привет", "мир", "αβγ", "日本語", "中文", "分词器", "测试", "한국어", "العربية", "हिन्दी"]
PIECES = ["'s", "'T", "'re", "'VE", "'m", "'ll", "'D", "'x", "''", " ", "  ", "   ", "\t", "\n", "\r\n",
          "\n\n", " \n", " ", "　", " ", " ", "0", "42", "3.14", "１２３", "٣",
          "!", "?!", "...", " -- ", "(a)", "[]{}", "#", "@user", "$5", "100%", "😀", "🚀🚀", "→",
          "<|im_start|>", "<|im_end|>", "<|endoftext|>", "<think>", "</think>", "<|im_star",
          "，", "。", "、", "“quoted”"]
BAD = [b"\xff", b"\xc3", b"\xe4\xbd", b"\xf0\x9f\x98", b"\x80\x80", b"\xed\xa0\x80"]


def random_text(rng) -> bytes:
    parts = []
    for _ in range(int(rng.integers(1, 14))):
        r = rng.random()
        if r < 0.45:
            parts.append(WORDS[rng.integers(len(WORDS))].encode())
        elif r < 0.9:
            parts.append(PIECES[rng.integers(len(PIECES))].encode())
        elif r < 0.95:
            parts.append(BAD[rng.integers(len(BAD))])
        else:
            parts.append(bytes(rng.integers(0, 256, int(rng.integers(1, 6)), dtype=np.uint8)))
    return b"".join(parts)


def test_golden_prompt(toks):
    """The regression prompt of the reference's raw mode (main.c:118-119)."""
    t, r = toks
    text = "你好，请介绍一下你自己"
    assert list(t.encode(text)) == [108386, 37945, 109432, 107828]
    assert list(r.encode(text.encode())) == [108386, 37945, 109432, 107828]
    assert t.decode([108386, 37945, 109432, 107828]).decode() == text


def test_random_texts_match_reference(toks):
    t, r = toks
    rng = np.random.default_rng(2024)
    for i in range(3000):
        s = random_text(rng)
        got, want = t.encode(s), r.encode(s)
        assert np.array_equal(got, want), (i, s, list(got), list(want))
        assert t.decode(got) == s == r.decode(want)


def test_chat_template_matches_reference(toks):
    t, r = toks
    for prompt in ["你好", "Explain the B200's TMEM in one sentence.", "", " x\n\n y "]:
        full = ("<|im_start|>user\n" + prompt + "<|im_end|>\n<|im_start|>assistant\n"
                "<think>\n\n</think>\n\n").encode()
        assert np.array_equal(t.chat(prompt), r.encode(full))


def test_batch_encode_equals_single(toks):
    t, _ = toks
    rng = np.random.default_rng(7)
    texts = [random_text(rng) for _ in range(97)]
    for threads in (1, 4, 0):
        got = t.encode_batch(texts, threads=threads)
        assert all(np.array_equal(g, t.encode(s)) for g, s in zip(got, texts))


def test_overflow_and_errors_match_reference(toks):
    t, r = toks
    L = n5.lib()
    s = "hello world, this is a test".encode()
    n = len(t.encode(s))
    out = np.zeros(64, np.int32)
    ptr = out.ctypes.data_as(n5.C.c_void_p)
    assert L.n550_tok_encode(t.handle, s, len(s), ptr, n) == n
    assert L.n550_tok_encode(t.handle, s, len(s), ptr, n - 1) == n5.N550_TOK_ERR_OVERFLOW
    assert r.encode(s, max_out=n - 1) == n5.N550_TOK_ERR_OVERFLOW
    long_word = b"a" * 3000                      # one piece past the reference's 2048-byte limit
    assert L.n550_tok_encode(t.handle, long_word, len(long_word), ptr, 64) == n5.N550_TOK_ERR_OVERFLOW
    assert r.encode(long_word) == n5.N550_TOK_ERR_OVERFLOW
    buf = n5.C.create_string_buffer(4)
    ids = np.array([108386, 37945], np.int32)   # 6 bytes: no room
    assert L.n550_tok_decode(t.handle, ids.ctypes.data_as(n5.C.c_void_p), 2, buf, 4) == \
        n5.N550_TOK_ERR_OVERFLOW
    blob = bytearray(oracle.TOK_PATH.read_bytes())
    h = n5.C.c_void_p()
    for mutate, code in [(lambda b: b.__setitem__(0, ord("X")), n5.N550_TOK_ERR_MAGIC),
                         (lambda b: b.__setitem__(4, 2), n5.N550_TOK_ERR_VERSION),
                         (lambda b: b.__setitem__(56, b[56] ^ 1), n5.N550_TOK_ERR_SIZE)]:
        bad = bytearray(blob)
        mutate(bad)
        arr = np.frombuffer(bytes(bad), np.uint8)
        assert L.n550_tok_init(n5.C.byref(h), arr.ctypes.data_as(n5.C.c_void_p), arr.size) == code
        assert oracle.RefTokenizer(bytes(bad)).rc == code
    assert L.n550_tok_init(n5.C.byref(h), arr.ctypes.data_as(n5.C.c_void_p), 10) == n5.N550_TOK_ERR_SIZE
