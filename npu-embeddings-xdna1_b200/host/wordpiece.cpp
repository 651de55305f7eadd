// BERT WordPiece for the host tools -- see wordpiece.hpp.
#include "wordpiece.hpp"

#include <algorithm>
#include <fstream>
#include <sstream>
#include <stdexcept>

namespace nebw {
namespace {

struct CpRange {
  uint32_t lo, hi;
};
struct FoldEntry {
  uint32_t cp, off, len;
};

#include "bert_unicode.inc"

bool in_ranges(uint32_t cp, const CpRange *r, int n) {
  const CpRange *it =
      std::upper_bound(r, r + n, cp, [](uint32_t v, const CpRange &x) { return v < x.lo; });
  return it != r && cp <= (it - 1)->hi;
}

bool is_cjk(uint32_t cp) {  // the Han blocks of BasicTokenizer._is_chinese_char
  return (cp >= 0x4E00 && cp <= 0x9FFF) || (cp >= 0x3400 && cp <= 0x4DBF) ||
         (cp >= 0x20000 && cp <= 0x2A6DF) || (cp >= 0x2A700 && cp <= 0x2B73F) ||
         (cp >= 0x2B740 && cp <= 0x2B81F) || (cp >= 0x2B820 && cp <= 0x2CEAF) ||
         (cp >= 0xF900 && cp <= 0xFAFF) || (cp >= 0x2F800 && cp <= 0x2FA1F);
}

// lower(), NFD, Mn marks dropped -- appended to `out`
void fold(uint32_t cp, std::vector<uint32_t> &out) {
  if (cp >= 0xAC00 && cp <= 0xD7A3) {  // Hangul syllable: L V (T) jamo
    const uint32_t s = cp - 0xAC00;
    out.push_back(0x1100 + s / 588);
    out.push_back(0x1161 + (s % 588) / 28);
    if (s % 28) out.push_back(0x11A7 + s % 28);
    return;
  }
  const FoldEntry *it = std::lower_bound(
      kFold, kFold + kFold_n, cp, [](const FoldEntry &e, uint32_t v) { return e.cp < v; });
  if (it != kFold + kFold_n && it->cp == cp) {
    for (uint32_t k = 0; k < it->len; ++k) out.push_back(kFoldData[it->off + k]);
  } else {
    out.push_back(cp);
  }
}

// Lenient UTF-8: a byte that does not start a well-formed sequence decodes
// to U+FFFD on its own (the clean step then drops it).
std::vector<uint32_t> decode(const std::string &s) {
  std::vector<uint32_t> out;
  out.reserve(s.size());
  const size_t n = s.size();
  for (size_t i = 0; i < n;) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    int len;
    uint32_t cp;
    if (c < 0x80) len = 1, cp = c;
    else if ((c & 0xE0) == 0xC0) len = 2, cp = c & 0x1Fu;
    else if ((c & 0xF0) == 0xE0) len = 3, cp = c & 0x0Fu;
    else if ((c & 0xF8) == 0xF0) len = 4, cp = c & 0x07u;
    else len = 0, cp = 0;
    bool ok = len > 0 && i + len <= n;
    for (int k = 1; ok && k < len; ++k) {
      const unsigned char cc = static_cast<unsigned char>(s[i + k]);
      ok = (cc & 0xC0) == 0x80;
      cp = (cp << 6) | (cc & 0x3Fu);
    }
    if (!ok) {
      out.push_back(0xFFFD);
      ++i;
      continue;
    }
    out.push_back(cp);
    i += static_cast<size_t>(len);
  }
  return out;
}

void encode_utf8(uint32_t cp, std::string &s) {
  if (cp < 0x80) {
    s.push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    s.push_back(static_cast<char>(0xC0 | (cp >> 6)));
    s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    s.push_back(static_cast<char>(0xE0 | (cp >> 12)));
    s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    s.push_back(static_cast<char>(0xF0 | (cp >> 18)));
    s.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

constexpr size_t kMaxPieceChars = 100;

}  // namespace

WordPiece WordPiece::from_vocab_file(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("tokenizer: cannot open " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  WordPiece t;
  t.index(ss.str());
  return t;
}

WordPiece WordPiece::from_vocab_bytes(const char *data, size_t bytes) {
  WordPiece t;
  t.index(std::string(data, bytes));
  return t;
}

// One token per line, id = line number; a trailing '\r' is not part of it.
void WordPiece::index(const std::string &blob) {
  size_t at = 0;
  while (at < blob.size()) {
    size_t nl = blob.find('\n', at);
    if (nl == std::string::npos) nl = blob.size();
    std::string tok = blob.substr(at, nl - at);
    if (!tok.empty() && tok.back() == '\r') tok.pop_back();
    id_.emplace(tok, static_cast<int32_t>(tokens_.size()));
    tokens_.push_back(std::move(tok));
    at = nl + 1;
  }
  if (tokens_.empty()) throw std::runtime_error("tokenizer: empty vocabulary");
  auto need = [&](const char *t) {
    auto it = id_.find(t);
    if (it == id_.end()) throw std::runtime_error(std::string("tokenizer: vocabulary has no ") + t);
    return it->second;
  };
  cls_id = need("[CLS]");
  sep_id = need("[SEP]");
  pad_id = need("[PAD]");
  unk_id = need("[UNK]");
  for (const char *s : {"[CLS]", "[SEP]", "[PAD]", "[UNK]", "[MASK]"})
    if (id_.count(s)) specials_.emplace_back(s);
  std::stable_sort(specials_.begin(), specials_.end(),
                   [](const std::string &a, const std::string &b) { return a.size() > b.size(); });
}

int32_t WordPiece::id_of(const std::string &token) const {
  auto it = id_.find(token);
  return it == id_.end() ? unk_id : it->second;
}

// Special tokens in the raw text are kept whole: the text is cut at the
// earliest one (the longer one on a tie) and the parts around it tokenized.
std::vector<std::string> WordPiece::tokenize(const std::string &text) const {
  std::vector<std::string> out;
  size_t from = 0;
  while (true) {
    size_t best = std::string::npos;
    const std::string *which = nullptr;
    for (const auto &s : specials_) {
      const size_t p = text.find(s, from);
      if (p != std::string::npos && (best == std::string::npos || p < best)) {
        best = p;
        which = &s;
      }
    }
    if (!which) break;
    auto head = tokenize_text(text.substr(from, best - from));
    out.insert(out.end(), head.begin(), head.end());
    out.push_back(*which);
    from = best + which->size();
  }
  auto tail = tokenize_text(text.substr(from));
  out.insert(out.end(), tail.begin(), tail.end());
  return out;
}

void WordPiece::wordpiece(const std::vector<uint32_t> &piece,
                          std::vector<std::string> &out) const {
  if (piece.size() > kMaxPieceChars) {
    out.push_back("[UNK]");
    return;
  }
  std::string flat;
  std::vector<size_t> byte_at(piece.size() + 1);
  for (size_t i = 0; i < piece.size(); ++i) {
    byte_at[i] = flat.size();
    encode_utf8(piece[i], flat);
  }
  byte_at[piece.size()] = flat.size();
  std::vector<std::string> sub;
  for (size_t start = 0; start < piece.size();) {
    size_t end = piece.size();
    std::string hit;
    for (; end > start; --end) {
      std::string s = flat.substr(byte_at[start], byte_at[end] - byte_at[start]);
      if (start > 0) s.insert(0, "##");
      if (id_.count(s)) {
        hit = std::move(s);
        break;
      }
    }
    if (hit.empty()) {
      out.push_back("[UNK]");
      return;
    }
    sub.push_back(std::move(hit));
    start = end;
  }
  out.insert(out.end(), sub.begin(), sub.end());
}

std::vector<std::string> WordPiece::tokenize_text(const std::string &text) const {
  std::vector<uint32_t> clean;
  for (uint32_t cp : decode(text)) {
    if (cp == 0 || cp == 0xFFFD || in_ranges(cp, kControl, kControl_n)) continue;
    if (in_ranges(cp, kSpace, kSpace_n)) {
      clean.push_back(' ');
    } else if (is_cjk(cp)) {
      clean.push_back(' ');
      clean.push_back(cp);
      clean.push_back(' ');
    } else {
      clean.push_back(cp);
    }
  }
  std::vector<std::string> out;
  std::vector<uint32_t> word, folded, piece;
  auto flush = [&]() {
    if (word.empty()) return;
    folded.clear();
    for (uint32_t cp : word) fold(cp, folded);
    piece.clear();
    for (uint32_t cp : folded) {
      if (in_ranges(cp, kPunct, kPunct_n)) {
        if (!piece.empty()) wordpiece(piece, out);
        piece.assign(1, cp);
        wordpiece(piece, out);
        piece.clear();
      } else {
        piece.push_back(cp);
      }
    }
    if (!piece.empty()) wordpiece(piece, out);
    word.clear();
  };
  for (uint32_t cp : clean) {
    if (cp == ' ')
      flush();
    else
      word.push_back(cp);
  }
  flush();
  return out;
}

Tokens WordPiece::encode(const std::string &text, int max_len) const {
  if (max_len < 2) throw std::runtime_error("tokenizer: max_len below 2 cannot hold [CLS] [SEP]");
  const std::vector<std::string> toks = tokenize(text);
  const size_t take = std::min(toks.size(), static_cast<size_t>(max_len - 2));
  Tokens t;
  t.ids.reserve(static_cast<size_t>(max_len));
  t.ids.push_back(cls_id);
  for (size_t i = 0; i < take; ++i) t.ids.push_back(id_of(toks[i]));
  t.ids.push_back(sep_id);
  t.n_tokens = static_cast<int32_t>(t.ids.size());
  t.truncated = take < toks.size();
  t.mask.assign(t.ids.size(), 1);
  t.ids.resize(static_cast<size_t>(max_len), pad_id);
  t.mask.resize(static_cast<size_t>(max_len), 0);
  return t;
}

}  // namespace nebw
