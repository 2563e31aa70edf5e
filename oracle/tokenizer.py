"""Python restatement of the reference tokenizer (TEST INFRASTRUCTURE ONLY).

Restates src/tokenizer.rs (byte-level BPE with the qwen2 pre-tokenizer) and
the text helpers of src/generate.rs (chat_template, Utf8Stream) as the
checker for the library's C++ tokenizer.  Only tests/ import it; the product
never does.

The pre-tokenizer compiles the reference's pattern (src/tokenizer.rs:16)
unchanged with the `regex` package, a backtracking engine with \\p{..}
classes, scoped case-insensitivity and lookahead, as fancy-regex (0.14.0,
over regex-syntax 0.8.11) provides them to the reference.  Lossy UTF-8
decoding uses Python's "replace" handler, which substitutes each maximal
ill-formed subsequence like Rust's String::from_utf8_lossy.

Pinned by tests/test_tokenizer.py against the reference's own tests
(src/tokenizer.rs:287-386, src/generate.rs:197-229).
"""

from __future__ import annotations

import regex

# src/tokenizer.rs:16
QWEN2_SPLIT_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*"
                       r"|\s*[\r\n]+|\s+(?!\S)|\s+")
_SPLIT = regex.compile(QWEN2_SPLIT_PATTERN)

TOKEN_TYPE_CONTROL, TOKEN_TYPE_USER_DEFINED = 3, 4  # src/tokenizer.rs:19-20


def byte_unicode_map():
    """src/tokenizer.rs:36-58: printable non-space Latin-1 bytes map to
    themselves, the other 68 to U+0100.. in byte order."""
    b2c = [None] * 256
    nxt = 256
    for b in range(256):
        if 0x21 <= b <= 0x7E or 0xA1 <= b <= 0xAC or 0xAE <= b <= 0xFF:
            b2c[b] = chr(b)
        else:
            b2c[b] = chr(nxt)
            nxt += 1
    return b2c, {c: b for b, c in enumerate(b2c)}


def pretokenize(text: str) -> list[str]:
    """The split of encode_ordinary (src/tokenizer.rs:215-232)."""
    out, last = [], 0
    for m in _SPLIT.finditer(text):
        if m.start() > last:
            out.append(text[last:m.start()])
        out.append(m.group())
        last = m.end()
    if last < len(text):
        out.append(text[last:])
    return out


class Tokenizer:
    """Tokenizer::new (src/tokenizer.rs:92-138)."""

    def __init__(self, tokens, token_types, merges):
        if len(tokens) != len(token_types):
            raise ValueError(f"{len(tokens)} tokens but {len(token_types)} token types")
        self.vocab = list(tokens)
        self.token_to_id = {t: i for i, t in enumerate(tokens)}
        self.merge_ranks = {m: r for r, m in enumerate(merges)}
        self.is_special = [t in (TOKEN_TYPE_CONTROL, TOKEN_TYPE_USER_DEFINED) for t in token_types]
        specials = [(t, i) for i, t in enumerate(tokens) if self.is_special[i]]
        # stable, longest (in UTF-8 bytes) first
        self.specials = sorted(specials, key=lambda s: -len(s[0].encode()))
        self.byte_to_char, self.char_to_byte = byte_unicode_map()

    def encode(self, text: str) -> list[int]:
        """src/tokenizer.rs:140-149 with split_specials (:183-213)."""
        ids = []
        pos = 0
        while pos < len(text):
            earliest = None
            for lit, i in self.specials:
                if not lit:
                    continue  # an empty literal never advances (the reference would loop)
                f = text.find(lit, pos)
                if f >= 0 and (earliest is None or f < earliest[0]):
                    earliest = (f, len(lit), i)
            if earliest is None:
                self._encode_ordinary(text[pos:], ids)
                break
            start, n, i = earliest
            if start > pos:
                self._encode_ordinary(text[pos:start], ids)
            ids.append(i)
            pos = start + n
        return ids

    def _encode_ordinary(self, text, ids):
        for chunk in pretokenize(text):
            self._bpe_chunk(chunk, ids)

    def _bpe_chunk(self, chunk, ids):
        """src/tokenizer.rs:234-285."""
        word = [self.byte_to_char[b] for b in chunk.encode()]
        while len(word) > 1:
            best = None
            for i in range(len(word) - 1):
                r = self.merge_ranks.get(word[i] + " " + word[i + 1])
                if r is not None and (best is None or r < best[0]):
                    best = (r, i)
            if best is None:
                break
            a, b = word[best[1]], word[best[1] + 1]
            nxt, i = [], 0
            while i < len(word):
                if i + 1 < len(word) and word[i] == a and word[i + 1] == b:
                    nxt.append(a + b)
                    i += 2
                else:
                    nxt.append(word[i])
                    i += 1
            word = nxt
        for sym in word:
            if sym not in self.token_to_id:
                raise KeyError(f"symbol {sym!r} not in vocab")
            ids.append(self.token_to_id[sym])

    def token_bytes(self, token_id: int) -> bytes:
        """src/tokenizer.rs:159-181."""
        tok = self.vocab[token_id]
        if self.is_special[token_id]:
            return tok.encode()
        out = bytearray()
        for c in tok:
            if c in self.char_to_byte:
                out.append(self.char_to_byte[c])
            else:
                out += c.encode()
        return bytes(out)

    def decode(self, ids) -> str:
        """src/tokenizer.rs:151-157."""
        return b"".join(self.token_bytes(i) for i in ids).decode("utf-8", "replace")


def chat_template(prompt: str) -> str:
    """src/generate.rs:13-21."""
    return ("<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n"
            f"<|im_start|>user\n{prompt}<|im_end|>\n<|im_start|>assistant\n")


class Utf8Stream:
    """src/generate.rs:24-66."""

    def __init__(self):
        self.buf = b""

    def push(self, data: bytes) -> str:
        self.buf += data
        try:
            out = self.buf.decode("utf-8")
            self.buf = b""
            return out
        except UnicodeDecodeError as e:
            # an error that runs to the end of the buffer is an incomplete
            # last character (Utf8Error::error_len() is None)
            if e.end == len(self.buf) and _incomplete_tail(self.buf[e.start:]):
                out = self.buf[:e.start].decode("utf-8")
                self.buf = self.buf[e.start:]
                return out
            out = self.buf.decode("utf-8", "replace")
            self.buf = b""
            return out

    def flush(self) -> str:
        out = self.buf.decode("utf-8", "replace")
        self.buf = b""
        return out


def _incomplete_tail(b: bytes) -> bool:
    """Whether b (the bytes from the first ill-formed point on) is a
    well-formed prefix of one UTF-8 character, cut short by the end."""
    lead = b[0]
    if 0xC2 <= lead <= 0xDF:
        n, lo, hi = 2, 0x80, 0xBF
    elif 0xE0 <= lead <= 0xEF:
        n, lo, hi = 3, 0xA0 if lead == 0xE0 else 0x80, 0x9F if lead == 0xED else 0xBF
    elif 0xF0 <= lead <= 0xF4:
        n, lo, hi = 4, 0x90 if lead == 0xF0 else 0x80, 0x8F if lead == 0xF4 else 0xBF
    else:
        return False
    if len(b) >= n:
        return False
    for k in range(1, len(b)):
        ok = lo <= b[k] <= hi if k == 1 else 0x80 <= b[k] <= 0xBF
        if not ok:
            return False
    return True
