// Byte-level BPE tokenizer (src/tokenizer.rs) and the text helpers of the
// generate loop (src/generate.rs:13-66), host side.
//
// Encode: literal special tokens are split out first (leftmost; the longest
// literal at equal starts), each span between them is cut into chunks by the
// qwen2 pre-tokenizer pattern (src/tokenizer.rs:16), and every chunk's bytes
// go through the GPT-2 byte alphabet and are merged by rank.  Decode: ids ->
// token strings -> bytes through the reverse alphabet -> UTF-8 with each
// maximal ill-formed subsequence replaced by U+FFFD (String::from_utf8_lossy).

#include <algorithm>
#include <string>
#include <unordered_map>
#include <vector>

#include "fz_internal.h"
#include "unicode_tables.h"

using namespace fz;

struct fz_tokenizer {
  std::vector<std::string> vocab;                       // id -> token in the mapped alphabet
  std::unordered_map<std::string, uint32_t> token_to_id;
  std::vector<std::pair<std::string, uint32_t>> specials; // longest literal first
  std::vector<bool> is_special;
  std::string byte_to_char[256];                        // UTF-8 of the mapped code point
  int16_t char_to_byte[324];                            // mapped code point -> byte, or -1
  // BPE over interned symbols: the merge rule "left right" of rank r is the
  // pair (left, right) -> (r, left + right).  Symbols never contain U+0020,
  // so a rule's key splits at its one space; rules without exactly one space
  // never match a pair.
  std::vector<std::string> sym_str;
  std::vector<int64_t> sym_vocab;  // vocabulary id of a symbol, or -1
  std::unordered_map<std::string, uint32_t> sym_index;
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> pair_merge;
  uint32_t byte_sym[256];
  uint32_t intern(const std::string& s) {
    auto it = sym_index.find(s);
    if (it != sym_index.end()) return it->second;
    const uint32_t id = (uint32_t)sym_str.size();
    sym_index.emplace(s, id);
    sym_str.push_back(s);
    auto v = token_to_id.find(s);
    sym_vocab.push_back(v == token_to_id.end() ? -1 : (int64_t)v->second);
    return id;
  }
};

struct fz_utf8_stream {
  std::string buf;
};

namespace {

// ---- code point classes (the pattern's \p{L}, \p{N}, \s) ----------------------
template <size_t N>
bool in_ranges(const uni::CpRange (&r)[N], uint32_t c) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (r[mid].hi < c)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo < N && r[lo].lo <= c;
}
bool is_letter(uint32_t c) { return c < 0x80 ? ((c | 0x20) - 'a') < 26u : in_ranges(uni::kLetter, c); }
bool is_number(uint32_t c) { return c < 0x80 ? (c - '0') < 10u : in_ranges(uni::kNumber, c); }
bool is_space(uint32_t c) { return c < 0x80 ? (c == ' ' || (c >= 9 && c <= 13)) : in_ranges(uni::kSpace, c); }
bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }

// The pattern's view of one code point, computed once per code point.
enum : uint8_t { C_LETTER = 1, C_NUMBER = 2, C_SPACE = 4, C_NL = 8 };
uint8_t classify(uint32_t c) {
  if (is_letter(c)) return C_LETTER;
  if (is_number(c)) return C_NUMBER;
  if (is_space(c)) return (uint8_t)(C_SPACE | (is_nl(c) ? C_NL : 0));
  return 0;  // other: not whitespace, letter or number
}
// the ASCII letter a contraction letter's case-insensitive match folds to, or 0
uint32_t fold(uint32_t c) {
  for (const auto& f : uni::kFold)
    if (f[0] == c) return f[1];
  return 0;
}

// Code points of well-formed UTF-8 and the byte offset of each (offs[n] = len).
void decode_utf8(const std::string& s, std::vector<uint32_t>* cps, std::vector<size_t>* offs) {
  cps->clear();
  offs->clear();
  const uint8_t* p = reinterpret_cast<const uint8_t*>(s.data());
  for (size_t i = 0; i < s.size();) {
    offs->push_back(i);
    const uint8_t b = p[i];
    uint32_t c;
    size_t len;
    if (b < 0x80) {
      c = b;
      len = 1;
    } else if (b < 0xE0) {
      c = b & 0x1F;
      len = 2;
    } else if (b < 0xF0) {
      c = b & 0x0F;
      len = 3;
    } else {
      c = b & 0x07;
      len = 4;
    }
    for (size_t k = 1; k < len; k++) c = (c << 6) | (p[i + k] & 0x3F);
    cps->push_back(c);
    i += len;
  }
  offs->push_back(s.size());
}

void append_utf8(std::string* out, uint32_t c) {
  if (c < 0x80) {
    out->push_back((char)c);
  } else if (c < 0x800) {
    out->push_back((char)(0xC0 | (c >> 6)));
    out->push_back((char)(0x80 | (c & 0x3F)));
  } else if (c < 0x10000) {
    out->push_back((char)(0xE0 | (c >> 12)));
    out->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (c & 0x3F)));
  } else {
    out->push_back((char)(0xF0 | (c >> 18)));
    out->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
    out->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
    out->push_back((char)(0x80 | (c & 0x3F)));
  }
}

// One step of a UTF-8 scan at p[i]: the length of the well-formed character
// there, or 0 with *sub = the length of the maximal ill-formed subpart (the
// lead byte and the continuation bytes that were still acceptable) and
// *at_end = whether the input ended inside an otherwise acceptable prefix.
size_t utf8_step(const uint8_t* p, size_t n, size_t i, size_t* sub, bool* at_end) {
  const uint8_t b = p[i];
  *at_end = false;
  if (b < 0x80) return 1;
  size_t len;
  uint8_t lo = 0x80, hi = 0xBF;
  if (b >= 0xC2 && b <= 0xDF) {
    len = 2;
  } else if (b >= 0xE0 && b <= 0xEF) {
    len = 3;
    if (b == 0xE0) lo = 0xA0;
    if (b == 0xED) hi = 0x9F;
  } else if (b >= 0xF0 && b <= 0xF4) {
    len = 4;
    if (b == 0xF0) lo = 0x90;
    if (b == 0xF4) hi = 0x8F;
  } else {
    *sub = 1;
    return 0;
  }
  size_t k = 1;
  for (; k < len; k++) {
    if (i + k >= n) {
      *sub = k;
      *at_end = true;
      return 0;
    }
    const uint8_t c = p[i + k];
    if (k == 1 ? (c < lo || c > hi) : (c < 0x80 || c > 0xBF)) break;
  }
  if (k == len) return len;
  *sub = k;
  return 0;
}

// String::from_utf8_lossy
std::string utf8_lossy(const std::string& s) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(s.data());
  const size_t n = s.size();
  std::string out;
  out.reserve(n);
  for (size_t i = 0; i < n;) {
    size_t sub = 0;
    bool at_end;
    const size_t len = utf8_step(p, n, i, &sub, &at_end);
    if (len) {
      out.append(s, i, len);
      i += len;
    } else {
      out += "\xEF\xBF\xBD";
      i += sub;
    }
  }
  return out;
}

// ---- the qwen2 pre-tokenizer ---------------------------------------------------
// End (code point index) of the pattern's match at i, alternatives in their
// order of preference:
//   (?i:'s|'t|'re|'ve|'m|'ll|'d) | [^\r\n\p{L}\p{N}]?\p{L}+ | \p{N} |
//   ' '?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n]+ | \s+(?!\S) | \s+
// Every code point starts some alternative, so the matches tile the text.
size_t match_at(const std::vector<uint32_t>& cp, const std::vector<uint8_t>& cl, size_t i) {
  const size_t n = cp.size();
  const uint32_t c0 = cp[i];
  const uint8_t k0 = cl[i];
  if (c0 == '\'' && i + 1 < n) {
    const uint32_t a = fold(cp[i + 1]);
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return i + 2;
    if (i + 2 < n) {
      const uint32_t b = fold(cp[i + 2]);
      if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return i + 3;
    }
  }
  {
    size_t j = i;
    if (!(k0 & (C_LETTER | C_NUMBER | C_NL)) && i + 1 < n && (cl[i + 1] & C_LETTER)) j = i + 1;
    if (cl[j] & C_LETTER) {
      while (j < n && (cl[j] & C_LETTER)) j++;
      return j;
    }
  }
  if (k0 & C_NUMBER) return i + 1;
  {
    size_t j = i;
    if (c0 == ' ' && i + 1 < n && cl[i + 1] == 0) j = i + 1;
    if (cl[j] == 0) {
      while (j < n && cl[j] == 0) j++;
      while (j < n && (cl[j] & C_NL)) j++;
      return j;
    }
  }
  size_t j = i;  // c0 is whitespace
  while (j < n && (cl[j] & C_SPACE)) j++;
  for (size_t k = j; k > i; k--)  // \s*[\r\n]+ ends after the run's last newline
    if (cl[k - 1] & C_NL) return k;
  if (j == n || j - i < 2) return j;  // \s+(?!\S) at the end of text, or \s+
  return j - 1;                       // \s+(?!\S): the last space stays for the next chunk
}

// Byte ranges of the chunks of `text` (well-formed UTF-8).
void pretokenize(const std::string& text, std::vector<std::pair<size_t, size_t>>* chunks) {
  std::vector<uint32_t> cp;
  std::vector<size_t> off;
  decode_utf8(text, &cp, &off);
  std::vector<uint8_t> cl(cp.size());
  for (size_t i = 0; i < cp.size(); i++) cl[i] = classify(cp[i]);
  chunks->clear();
  for (size_t i = 0; i < cp.size();) {
    const size_t j = match_at(cp, cl, i);
    chunks->push_back({off[i], off[j]});
    i = j;
  }
}

// ---- BPE (src/tokenizer.rs:234-285) ---------------------------------------------
// word / next: scratch reused across chunks
void bpe_chunk(const fz_tokenizer& t, const char* s, size_t len, std::vector<uint32_t>* ids,
               std::vector<uint32_t>& word, std::vector<uint32_t>& next) {
  word.resize(len);
  for (size_t i = 0; i < len; i++) word[i] = t.byte_sym[(uint8_t)s[i]];
  while (word.size() > 1) {
    // the adjacent pair of lowest rank (the first such pair on ties)
    uint32_t best = UINT32_MAX, merged = 0;
    size_t idx = 0;
    for (size_t i = 0; i + 1 < word.size(); i++) {
      auto it = t.pair_merge.find((uint64_t)word[i] << 32 | word[i + 1]);
      if (it != t.pair_merge.end() && it->second.first < best) {
        best = it->second.first;
        merged = it->second.second;
        idx = i;
      }
    }
    if (best == UINT32_MAX) break;
    const uint32_t a = word[idx], b = word[idx + 1];
    // every occurrence of the pair, left to right
    next.clear();
    for (size_t i = 0; i < word.size();) {
      if (i + 1 < word.size() && word[i] == a && word[i + 1] == b) {
        next.push_back(merged);
        i += 2;
      } else {
        next.push_back(word[i]);
        i += 1;
      }
    }
    word.swap(next);
  }
  for (uint32_t sym : word) {
    if (t.sym_vocab[sym] < 0) fail(FZ_EINVAL, "symbol \"%s\" not in vocab", t.sym_str[sym].c_str());
    ids->push_back((uint32_t)t.sym_vocab[sym]);
  }
}

void encode_ordinary(const fz_tokenizer& t, const std::string& text, std::vector<uint32_t>* ids) {
  std::vector<std::pair<size_t, size_t>> chunks;
  pretokenize(text, &chunks);
  std::vector<uint32_t> word, next;
  for (const auto& c : chunks) bpe_chunk(t, text.data() + c.first, c.second - c.first, ids, word, next);
}

std::vector<uint32_t> encode(const fz_tokenizer& t, const std::string& text) {
  std::vector<uint32_t> ids;
  // next occurrence of each special literal at or after the last search
  // position (npos: none left), searched again only once pos passes it
  std::vector<size_t> next(t.specials.size(), 0);
  std::vector<bool> searched(t.specials.size(), false);
  size_t pos = 0;
  while (pos < text.size()) {
    // leftmost special literal; the longest one at equal starts (specials are
    // sorted longest first and only a strictly earlier start replaces one)
    size_t start = std::string::npos, lit_len = 0;
    uint32_t id = 0;
    for (size_t k = 0; k < t.specials.size(); k++) {
      const auto& sp = t.specials[k];
      if (!searched[k] || (next[k] != std::string::npos && next[k] < pos)) {
        next[k] = text.find(sp.first, pos);
        searched[k] = true;
      }
      const size_t f = next[k];
      if (f != std::string::npos && (start == std::string::npos || f < start)) {
        start = f;
        lit_len = sp.first.size();
        id = sp.second;
      }
    }
    if (start == std::string::npos) {
      encode_ordinary(t, text.substr(pos), &ids);
      break;
    }
    if (start > pos) encode_ordinary(t, text.substr(pos, start - pos), &ids);
    ids.push_back(id);
    pos = start + lit_len;
  }
  return ids;
}

std::string token_bytes(const fz_tokenizer& t, uint32_t id) {
  if (id >= t.vocab.size()) fail(FZ_EINVAL, "token id %u out of range", id);
  const std::string& tok = t.vocab[id];
  if (t.is_special[id]) return tok;  // special tokens are literal text
  std::string out;
  std::vector<uint32_t> cp;
  std::vector<size_t> off;
  decode_utf8(tok, &cp, &off);
  for (uint32_t c : cp) {
    if (c < 324 && t.char_to_byte[c] >= 0)
      out.push_back((char)t.char_to_byte[c]);
    else
      append_utf8(&out, c);
  }
  return out;
}

// The GPT-2 byte <-> code point bijection (src/tokenizer.rs:36-58): printable
// non-space Latin-1 bytes map to themselves, the other 68 to 256, 257, ... in
// byte order.
void byte_alphabet(fz_tokenizer* t) {
  std::fill(std::begin(t->char_to_byte), std::end(t->char_to_byte), (int16_t)-1);
  uint32_t next = 256;
  for (uint32_t b = 0; b < 256; b++) {
    const bool self = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    const uint32_t c = self ? b : next++;
    t->byte_to_char[b].clear();
    append_utf8(&t->byte_to_char[b], c);
    t->char_to_byte[c] = (int16_t)b;
  }
}

// Tokenizer::new (src/tokenizer.rs:92-138)
std::unique_ptr<fz_tokenizer> make_tokenizer(std::vector<std::string> tokens, const std::vector<int64_t>& types,
                                             const std::vector<std::string>& merges) {
  if (types.size() != tokens.size())
    fail(FZ_EINVAL, "%zu tokens but %zu token types", tokens.size(), types.size());
  auto t = std::make_unique<fz_tokenizer>();
  t->token_to_id.reserve(tokens.size());
  for (size_t i = 0; i < tokens.size(); i++) t->token_to_id[tokens[i]] = (uint32_t)i;  // a later duplicate wins
  byte_alphabet(t.get());
  for (int b = 0; b < 256; b++) t->byte_sym[b] = t->intern(t->byte_to_char[b]);
  t->pair_merge.reserve(merges.size());
  for (size_t r = 0; r < merges.size(); r++) {
    const std::string& m = merges[r];
    const size_t sp = m.find(' ');
    if (sp == std::string::npos || m.find(' ', sp + 1) != std::string::npos) continue;
    const std::string a = m.substr(0, sp), b = m.substr(sp + 1);
    const uint32_t ia = t->intern(a), ib = t->intern(b), im = t->intern(a + b);
    t->pair_merge[(uint64_t)ia << 32 | ib] = {(uint32_t)r, im};  // a later duplicate rule wins
  }
  t->is_special.resize(tokens.size());
  for (size_t i = 0; i < tokens.size(); i++) {
    t->is_special[i] = types[i] == 3 || types[i] == 4;  // control, user-defined
    // an empty literal would match everywhere without advancing: never a split point
    if (t->is_special[i] && !tokens[i].empty()) t->specials.push_back({tokens[i], (uint32_t)i});
  }
  std::stable_sort(t->specials.begin(), t->specials.end(),
                   [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
  t->vocab = std::move(tokens);
  return t;
}

// Copy `s` into out[0, cap) and report its size; FZ_ESPACE when it does not fit.
void give(const std::string& s, char* out, size_t cap, size_t* len) {
  if (!len || (cap && !out)) fail(FZ_EINVAL, "null output pointer");
  *len = s.size();
  if (s.size() > cap) fail(FZ_ESPACE, "output needs %zu bytes, the buffer holds %zu", s.size(), cap);
  if (!s.empty()) memcpy(out, s.data(), s.size());
}

std::string text_arg(const char* text, size_t len) {
  if (!text && len) fail(FZ_EINVAL, "null text");
  std::string s(text ? text : "", len);
  if (!utf8_valid(reinterpret_cast<const uint8_t*>(s.data()), s.size())) fail(FZ_EINVAL, "text is not valid UTF-8");
  return s;
}

}  // namespace

// ---- C ABI ----------------------------------------------------------------------
extern "C" {

int fz_tokenizer_from_gguf(const fz_file* f, fz_tokenizer** out) {
  return guard([&] {
    if (!f || !out) fail(FZ_EINVAL, "null argument");
    const GgufFile& g = *f->g;
    const std::string& model = g.meta_str("tokenizer.ggml.model");
    if (model != "gpt2") fail(FZ_EFORMAT, "tokenizer model '%s' not supported (only gpt2 byte-level BPE)", model.c_str());
    const std::string& pre = g.meta_str("tokenizer.ggml.pre");
    if (pre != "qwen2") fail(FZ_EFORMAT, "pre-tokenizer '%s' not supported (only qwen2)", pre.c_str());
    auto tokens = g.meta_str_array("tokenizer.ggml.tokens");
    auto types = g.meta_int_array("tokenizer.ggml.token_type");
    auto merges = g.meta_str_array("tokenizer.ggml.merges");
    *out = make_tokenizer(std::move(tokens), types, merges).release();
  });
}

int fz_tokenizer_new(const char* const* tokens, const int64_t* token_types, size_t n, const char* const* merges,
                     size_t n_merges, fz_tokenizer** out) {
  return guard([&] {
    if (!out || (n && (!tokens || !token_types)) || (n_merges && !merges)) fail(FZ_EINVAL, "null argument");
    std::vector<std::string> tv(n), mv(n_merges);
    for (size_t i = 0; i < n; i++) tv[i] = text_arg(tokens[i], tokens[i] ? strlen(tokens[i]) : 0);
    for (size_t i = 0; i < n_merges; i++) mv[i] = text_arg(merges[i], merges[i] ? strlen(merges[i]) : 0);
    *out = make_tokenizer(std::move(tv), std::vector<int64_t>(token_types, token_types + n), mv).release();
  });
}

void fz_tokenizer_free(fz_tokenizer* t) { delete t; }

int fz_tokenizer_vocab_size(const fz_tokenizer* t, size_t* n) {
  return guard([&] {
    if (!t || !n) fail(FZ_EINVAL, "null argument");
    *n = t->vocab.size();
  });
}

int fz_tokenizer_encode(const fz_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap, size_t* n) {
  return guard([&] {
    if (!t || !n) fail(FZ_EINVAL, "null argument");
    const std::vector<uint32_t> v = encode(*t, text_arg(text, len));
    *n = v.size();
    if (v.size() > cap) fail(FZ_ESPACE, "%zu ids, the buffer holds %zu", v.size(), cap);
    if (!v.empty()) memcpy(ids, v.data(), v.size() * 4);
  });
}

int fz_tokenizer_decode(const fz_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t cap, size_t* len) {
  return guard([&] {
    if (!t || (n && !ids)) fail(FZ_EINVAL, "null argument");
    std::string bytes;
    for (size_t i = 0; i < n; i++) bytes += token_bytes(*t, ids[i]);
    give(utf8_lossy(bytes), out, cap, len);
  });
}

int fz_tokenizer_token_bytes(const fz_tokenizer* t, uint32_t id, char* out, size_t cap, size_t* len) {
  return guard([&] {
    if (!t) fail(FZ_EINVAL, "null argument");
    give(token_bytes(*t, id), out, cap, len);
  });
}

int fz_pretokenize(const char* text, size_t len, size_t* ends, size_t cap, size_t* n) {
  return guard([&] {
    if (!n) fail(FZ_EINVAL, "null argument");
    std::vector<std::pair<size_t, size_t>> chunks;
    pretokenize(text_arg(text, len), &chunks);
    *n = chunks.size();
    if (chunks.size() > cap) fail(FZ_ESPACE, "%zu chunks, the buffer holds %zu", chunks.size(), cap);
    for (size_t i = 0; i < chunks.size(); i++) ends[i] = chunks[i].second;
  });
}

int fz_chat_template(const char* prompt, size_t len, char* out, size_t cap, size_t* out_len) {
  return guard([&] {
    const std::string p = text_arg(prompt, len);
    give("<|im_start|>system\nYou are Qwen, created by Alibaba Cloud. You are a helpful assistant.<|im_end|>\n"
         "<|im_start|>user\n" + p + "<|im_end|>\n<|im_start|>assistant\n",
         out, cap, out_len);
  });
}

int fz_utf8_stream_new(fz_utf8_stream** out) {
  return guard([&] {
    if (!out) fail(FZ_EINVAL, "null argument");
    *out = new fz_utf8_stream();
  });
}

void fz_utf8_stream_free(fz_utf8_stream* s) { delete s; }

int fz_utf8_stream_push(fz_utf8_stream* s, const void* bytes, size_t n, char* out, size_t cap, size_t* len) {
  return guard([&] {
    if (!s || (n && !bytes)) fail(FZ_EINVAL, "null argument");
    std::string buf = s->buf;
    buf.append(static_cast<const char*>(bytes), n);
    // the first ill-formed point decides (std::str::from_utf8's error)
    const uint8_t* p = reinterpret_cast<const uint8_t*>(buf.data());
    size_t i = 0, sub = 0;
    bool at_end = false;
    while (i < buf.size()) {
      const size_t l = utf8_step(p, buf.size(), i, &sub, &at_end);
      if (!l) break;
      i += l;
    }
    std::string emit, keep;
    if (i == buf.size()) {
      emit = buf;  // all complete
    } else if (at_end) {
      emit = buf.substr(0, i);  // an incomplete last character waits for more bytes
      keep = buf.substr(i);
    } else {
      emit = utf8_lossy(buf);  // ill-formed: emit lossily and start over
    }
    give(emit, out, cap, len);
    s->buf.swap(keep);
  });
}

int fz_utf8_stream_flush(fz_utf8_stream* s, char* out, size_t cap, size_t* len) {
  return guard([&] {
    if (!s) fail(FZ_EINVAL, "null argument");
    give(utf8_lossy(s->buf), out, cap, len);
    s->buf.clear();
  });
}

}  // extern "C"
