"""Tokenizer (src/tokenizer.rs) and the text helpers of the generate loop
(src/generate.rs): the library's C++ implementation through the C ABI,
against the reference's own tests and against the Python restatement in
oracle/tokenizer.py on seeded random text.  Host code: no GPU."""

import ctypes as C
import random
import struct

import pytest

import furnace_b200 as fz
from furnace_b200 import synth
from oracle import tokenizer as ot


# ---- the reference's tests (src/tokenizer.rs:287-386, src/generate.rs:197-229) --
def tiny_parts():
    """src/tokenizer.rs:289-301: the 256 byte tokens, merges building "hell",
    one control token."""
    b2c, _ = ot.byte_unicode_map()
    return b2c + ["he", "ll", "hell", "<|test|>"], [1] * 259 + [3], ["h e", "l l", "he ll"]


@pytest.fixture(scope="module")
def tiny():
    return fz.Tokenizer.new(*tiny_parts())


@pytest.fixture(scope="module")
def tiny_ref():
    return ot.Tokenizer(*tiny_parts())


def test_merges_apply_by_rank(tiny, tiny_ref):
    assert tiny.encode("hello") == [258, 111] == tiny_ref.encode("hello")


@pytest.mark.parametrize("s", ["Hello, world! 123", "नमस्ते दुनिया",
                               "pizza \U0001F355 and \U0001F363", "  leading, trailing  ", "a   b\t\tc\n\nd"],
                         ids=["ascii", "hindi", "emoji", "whitespace", "whitespace2"])
def test_round_trip(tiny, tiny_ref, s):
    ids = tiny.encode(s)
    assert ids == tiny_ref.encode(s)
    assert tiny.decode(ids) == s


def test_special_token_is_not_split(tiny):
    ids = tiny.encode("a<|test|>b")
    assert ids == [ord("a"), 259, ord("b")]
    assert tiny.decode(ids) == "a<|test|>b"


def test_empty_string(tiny):
    assert tiny.encode("") == []
    assert tiny.decode([]) == ""


def test_byte_map_is_a_bijection(tiny):
    b2c, c2b = ot.byte_unicode_map()
    assert len(c2b) == 256 and b2c[0x20] == "Ġ" and b2c[0x0A] == "Ċ"
    # token b of the tiny vocabulary is byte b's code point: the library maps it back
    for b in range(256):
        assert tiny.token_bytes(b) == bytes([b])
    assert tiny.token_bytes(259) == b"<|test|>"
    with pytest.raises(fz.FurnaceError) as e:
        tiny.token_bytes(260)
    assert e.value.code == fz.FZ_EINVAL


def test_utf8_stream_holds_partial_characters():
    s = fz.Utf8Stream()
    assert s.push(bytes([0xE0, 0xA4])) == ""
    assert s.push(bytes([0xA8])) == "न"
    assert s.flush() == ""


def test_utf8_stream_mixed_ascii_and_partial():
    s = fz.Utf8Stream()
    assert s.push(b"ab\xc3") == "ab"
    assert s.push(b"\xa9!") == "é!"


def test_chat_template():
    want = ("<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n"
            "<|im_start|>user\nHi<|im_end|>\n<|im_start|>assistant\n")
    assert fz.chat_template("Hi") == want == ot.chat_template("Hi")


# ---- seeded random text against the restatement --------------------------------
POOL = (
    list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789")
    + list(" !\"#$%&'()*+,-./:;<=>?@[\\]^_`{|}~")
    + [" ", " ", "  ", "\t", "\n", "\r", "\r\n", "\n\n", " ", "　", " ", "\x0b", "\x0c", "\x85"]
    + ["'s", "'S", "'t", "'T", "'re", "'RE", "'Re", "'ve", "'VE", "'m", "'M", "'ll", "'LL", "'lL", "'d", "'D",
       "'ſ", "'x"]
    + ["é", "ß", "Ω", "Ж", "ж", "ǅ", "ʰ", "ا", "中", "文", "ア",
       "ก", "न", "म", "ह", "́", "्", "ि", "가"]
    + ["٣", "²", "½", "Ⅻ", "\U0001d7d9", "①"]
    + ["€", "©", "→", "\U0001f600", "\U0001f355", "‍", "️", "\U0001f1fa\U0001f1f8"]
    + ["hello", " world", "The", " the", "don't", "I'm", "123", "3.14", " x", "  ", "\t\t", "!!", "...", "<", ">"]
)


def rand_text(rng, n_max=40, pool=POOL):
    return "".join(rng.choice(pool) for _ in range(rng.randint(0, n_max)))


def test_pretokenize_matches_the_pattern():
    rng = random.Random(7)
    for _ in range(3000):
        s = rand_text(rng)
        got = fz.pretokenize(s)
        assert got == ot.pretokenize(s), repr(s)
        assert "".join(got) == s


def _train(corpus, n_merges):
    """A small BPE vocabulary: the most frequent adjacent pair of the corpus's
    pre-tokenized chunks, merged n_merges times."""
    b2c, _ = ot.byte_unicode_map()
    words = [[b2c[b] for b in chunk.encode()] for text in corpus for chunk in ot.pretokenize(text)]
    merges, tokens = [], list(b2c)
    for _ in range(n_merges):
        counts = {}
        for w in words:
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + 1
        if not counts:
            break
        (a, b), _ = max(counts.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append(f"{a} {b}")
        tokens.append(a + b)
        nw = []
        for w in words:
            o, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == a and w[i + 1] == b:
                    o.append(a + b)
                    i += 2
                else:
                    o.append(w[i])
                    i += 1
            nw.append(o)
        words = nw
    return tokens, merges


SPECIALS = [("<|endoftext|>", 3), ("<|im_start|>", 3), ("<|im_end|>", 3), ("<|im_start|>x", 4), ("<tool>", 4)]


@pytest.fixture(scope="module")
def trained():
    rng = random.Random(11)
    corpus = [rand_text(rng, 60) for _ in range(300)]
    tokens, merges = _train(corpus, 400)
    types = [1] * len(tokens)
    for lit, ty in SPECIALS:
        tokens.append(lit)
        types.append(ty)
    return tokens, types, merges


def test_encode_decode_match_the_restatement(trained):
    tokens, types, merges = trained
    t, r = fz.Tokenizer.new(tokens, types, merges), ot.Tokenizer(tokens, types, merges)
    assert len(t) == len(tokens)
    rng = random.Random(13)
    pool = POOL + [s for s, _ in SPECIALS] + ["<|im_start", "|>", "<tool"]
    for _ in range(1500):
        s = rand_text(rng, 50, pool)
        ids = t.encode(s)
        assert ids == r.encode(s), repr(s)
        assert t.decode(ids) == s
    # any id sequence, partial UTF-8 included: lossy like from_utf8_lossy
    for _ in range(1500):
        ids = [rng.randrange(len(tokens)) for _ in range(rng.randint(0, 12))]
        assert t.decode(ids) == r.decode(ids), ids


def test_lossy_decode_of_ill_formed_bytes(tiny, tiny_ref):
    """Ids 0-255 of the tiny vocabulary are single bytes, so decode of them
    is from_utf8_lossy of arbitrary bytes (maximal subparts -> U+FFFD)."""
    cases = [b"\xe0\xa4", b"\xed\xa0\x80", b"\xf0\x80\x80", b"\xf4\x90\x80\x80", b"\xc0\xaf", b"\xff", b"a\x80b",
             b"\xf0\x9f\x98", b"\xf0\x9f\x98\x80\xf0", b"\xe2\x82\xac\xe2\x82"]
    rng = random.Random(17)
    cases += [bytes(rng.randrange(256) for _ in range(rng.randint(1, 12))) for _ in range(2000)]
    for b in cases:
        assert tiny.decode(list(b)) == b.decode("utf-8", "replace") == tiny_ref.decode(list(b)), b


def test_utf8_stream_matches_the_restatement():
    rng = random.Random(19)
    for _ in range(300):
        data = "".join(rng.choice(POOL) for _ in range(20)).encode()
        if rng.random() < 0.3:
            i = rng.randrange(len(data) + 1)
            data = data[:i] + bytes([rng.randrange(256)]) + data[i:]
        s, r = fz.Utf8Stream(), ot.Utf8Stream()
        i = 0
        while i < len(data):
            k = rng.randint(1, 5)
            assert s.push(data[i:i + k]) == r.push(data[i:i + k])
            i += k
        assert s.flush() == r.flush()


def test_output_buffer_too_small_reports_the_size(tiny):
    L = fz.load_library()
    n = C.c_size_t()
    text = b"hello world"
    assert L.fz_tokenizer_encode(tiny._h, text, len(text), None, 0, C.byref(n)) == fz.FZ_ESPACE
    assert n.value == len(tiny.encode("hello world"))
    assert L.fz_chat_template(b"Hi", 2, None, 0, C.byref(n)) == fz.FZ_ESPACE and n.value == len(fz.chat_template("Hi"))
    s = fz.Utf8Stream()
    buf = C.create_string_buffer(1)
    assert L.fz_utf8_stream_push(s._h, b"abc", 3, buf, 1, C.byref(n)) == fz.FZ_ESPACE and n.value == 3
    assert s.push(b"d") == "d"  # the refused push left the stream as it was


def test_invalid_utf8_text_is_rejected(tiny):
    L = fz.load_library()
    n = C.c_size_t()
    ids = (C.c_uint32 * 8)()
    assert L.fz_tokenizer_encode(tiny._h, b"a\xffb", 3, ids, 8, C.byref(n)) == fz.FZ_EINVAL


# ---- Tokenizer::from_gguf (src/tokenizer.rs:67-90) ----------------------------
def _arr_str(k, vals):
    return synth._s(k) + struct.pack("<IIQ", 9, 8, len(vals)) + b"".join(synth._s(v) for v in vals)


def _arr_int(k, vals, tag=5):
    fmt = {0: "B", 5: "i", 11: "q"}[tag]
    return synth._s(k) + struct.pack("<IIQ", 9, tag, len(vals)) + struct.pack(f"<{len(vals)}{fmt}", *vals)


def _tok_gguf(path, tokens, types, merges, model="gpt2", pre="qwen2", type_tag=5, raw_token=None):
    meta = [synth._kv_str("tokenizer.ggml.model", model), synth._kv_str("tokenizer.ggml.pre", pre),
            _arr_str("tokenizer.ggml.tokens", tokens), _arr_int("tokenizer.ggml.token_type", types, type_tag),
            _arr_str("tokenizer.ggml.merges", merges)]
    if raw_token is not None:  # a string of arbitrary bytes
        meta.append(synth._s("bad") + struct.pack("<IQ", 8, len(raw_token)) + raw_token)
    head = b"GGUF" + struct.pack("<IQQ", 3, 0, len(meta)) + b"".join(meta)
    with open(path, "wb") as f:
        f.write(head + b"\0" * (-len(head) % 32))  # the data section starts aligned
    return path


def test_from_gguf_equals_new(tmp_path, trained):
    tokens, types, merges = trained
    f = fz.GgufFile.open(_tok_gguf(str(tmp_path / "t.gguf"), tokens, types, merges))
    a, b = fz.Tokenizer.from_gguf(f), fz.Tokenizer.new(tokens, types, merges)
    rng = random.Random(23)
    for _ in range(200):
        s = rand_text(rng, 30, POOL + ["<|im_end|>"])
        assert a.encode(s) == b.encode(s)
    # token types of any integer width (GgufValue::as_i64)
    f8 = fz.GgufFile.open(_tok_gguf(str(tmp_path / "u8.gguf"), tokens, types, merges, type_tag=0))
    assert fz.Tokenizer.from_gguf(f8).encode("<tool>x") == b.encode("<tool>x")


@pytest.mark.parametrize("kw,code", [({"model": "llama"}, fz.FZ_EFORMAT), ({"pre": "llama3"}, fz.FZ_EFORMAT)])
def test_from_gguf_rejects_other_tokenizers(tmp_path, kw, code):
    b2c, _ = ot.byte_unicode_map()
    f = fz.GgufFile.open(_tok_gguf(str(tmp_path / "t.gguf"), b2c, [1] * 256, [], **kw))
    with pytest.raises(fz.FurnaceError) as e:
        fz.Tokenizer.from_gguf(f)
    assert e.value.code == code


def test_token_type_count_must_match(tmp_path):
    b2c, _ = ot.byte_unicode_map()
    f = fz.GgufFile.open(_tok_gguf(str(tmp_path / "t.gguf"), b2c, [1] * 255, []))
    with pytest.raises(fz.FurnaceError) as e:
        fz.Tokenizer.from_gguf(f)
    assert e.value.code == fz.FZ_EINVAL
    with pytest.raises(fz.FurnaceError):
        fz.Tokenizer.new(b2c, [1] * 255, [])


def test_gguf_strings_must_be_utf8(tmp_path):
    """src/gguf.rs:71-75: a metadata string that is not UTF-8 fails the parse."""
    b2c, _ = ot.byte_unicode_map()
    with pytest.raises(fz.FurnaceError) as e:
        fz.GgufFile.open(_tok_gguf(str(tmp_path / "t.gguf"), b2c, [1] * 256, [], raw_token=b"ok\xff"))
    assert e.value.code == fz.FZ_EFORMAT


def test_synthetic_model_vocabulary(tmp_path):
    """The benchmark GGUFs carry placeholder token strings: the tokenizer
    loads, and text whose bytes are not in the vocabulary is an error."""
    f = fz.GgufFile.open(synth.write(synth.spec("tiny_q8"), str(tmp_path / "m.gguf")))
    t = fz.Tokenizer.from_gguf(f)
    assert len(t) == 2048
    assert t.token_bytes(5) == b"<t5>"
    with pytest.raises(fz.FurnaceError) as e:
        t.encode("abc")
    assert e.value.code == fz.FZ_EINVAL


def test_encode_matches_hf_tokenizers(trained):
    """A third implementation of the same published algorithm: HF
    `tokenizers` (0.22.2 here, Rust, Oniguruma regex) configured as Qwen2's
    tokenizer.json pre-tokenizer (Split on the same pattern, isolated, then
    ByteLevel without its own regex) over the same vocabulary, merges and
    special tokens, without Qwen's NFC normalizer (the reference applies
    none)."""
    tk = pytest.importorskip("tokenizers")
    tokens, types, merges = trained
    hf = tk.Tokenizer(tk.models.BPE(vocab={t: i for i, t in enumerate(tokens)},
                                    merges=[tuple(m.split(" ")) for m in merges]))
    hf.pre_tokenizer = tk.pre_tokenizers.Sequence([
        tk.pre_tokenizers.Split(tk.Regex(ot.QWEN2_SPLIT_PATTERN), behavior="isolated", invert=False),
        tk.pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    hf.add_special_tokens([tk.AddedToken(lit, special=True, normalized=False) for lit, _ in SPECIALS])
    ours = fz.Tokenizer.new(tokens, types, merges)
    rng = random.Random(29)
    pool = POOL + [s for s, _ in SPECIALS] + ["<|im_start", "|>", "<tool"]
    for _ in range(2000):
        s = rand_text(rng, 50, pool)
        assert ours.encode(s) == hf.encode(s, add_special_tokens=False).ids, repr(s)
