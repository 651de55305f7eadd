// BERT WordPiece for the host tools: a pretokenizer over code points and a
// vocabulary trie (see wordpiece.hpp for the pipeline).
#include "wordpiece.hpp"

#include <algorithm>
#include <fstream>
#include <iterator>
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

// ---- Unicode classes (tables generated from unicodedata) -------------------

bool in_table(char32_t cp, const CpRange *table, int n) {
  int lo = 0, hi = n - 1;  // binary search over sorted, disjoint ranges
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    if (cp < table[mid].lo)
      hi = mid - 1;
    else if (cp > table[mid].hi)
      lo = mid + 1;
    else
      return true;
  }
  return false;
}

bool is_control(char32_t cp) { return in_table(cp, kControl, kControl_n); }
bool is_space(char32_t cp) { return in_table(cp, kSpace, kSpace_n); }
bool is_punct(char32_t cp) { return in_table(cp, kPunct, kPunct_n); }

// The CJK ideograph blocks HuggingFace's BasicTokenizer isolates
// (_is_chinese_char): the Unified Ideographs, Extensions A-E and the
// Compatibility Ideographs (and Supplement).  Kana and Hangul are not among
// them.
bool is_han(char32_t cp) {
  static constexpr CpRange kHan[] = {{0x3400, 0x4DBF},   {0x4E00, 0x9FFF},   {0xF900, 0xFAFF},
                                     {0x20000, 0x2A6DF}, {0x2A700, 0x2B73F}, {0x2B740, 0x2B81F},
                                     {0x2B820, 0x2CEAF}, {0x2F800, 0x2FA1F}};
  return in_table(cp, kHan, static_cast<int>(std::size(kHan)));
}

// Lower case, canonical decomposition and removal of nonspacing marks, one
// code point at a time, appended to `out`.
void fold_into(char32_t cp, std::u32string &out) {
  constexpr char32_t kSBase = 0xAC00, kLBase = 0x1100, kVBase = 0x1161, kTBase = 0x11A7;
  constexpr char32_t kVCount = 21, kTCount = 28, kSCount = 19 * kVCount * kTCount;
  if (cp >= kSBase && cp < kSBase + kSCount) {  // Hangul syllable -> L V (T) jamo
    const char32_t s = cp - kSBase;
    out += kLBase + s / (kVCount * kTCount);
    out += kVBase + (s % (kVCount * kTCount)) / kTCount;
    if (s % kTCount) out += kTBase + s % kTCount;
    return;
  }
  int lo = 0, hi = kFold_n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) / 2;
    if (cp < kFold[mid].cp) {
      hi = mid - 1;
    } else if (cp > kFold[mid].cp) {
      lo = mid + 1;
    } else {
      out.append(kFoldData + kFold[mid].off, kFoldData + kFold[mid].off + kFold[mid].len);
      return;
    }
  }
  out += cp;
}

// ---- UTF-8 ------------------------------------------------------------------

// Bytes of the sequence a lead byte starts (1-4), 0 for a byte that starts
// none (a continuation byte, or 0xF8-0xFF).
int lead_span(unsigned char b) {
  if (b < 0x80) return 1;
  if (b < 0xC0 || b >= 0xF8) return 0;
  return b < 0xE0 ? 2 : (b < 0xF0 ? 3 : 4);
}

// Lenient decoding: a byte that does not start a complete sequence of
// continuation bytes stands for U+FFFD on its own and decoding resumes at
// the next byte.  (Overlong forms and surrogates are decoded as written.)
std::u32string decode_utf8(const char *p, size_t n) {
  std::u32string out;
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const unsigned char b = static_cast<unsigned char>(p[i]);
    const int span = lead_span(b);
    bool whole = span > 0 && i + static_cast<size_t>(span) <= n;
    char32_t cp = span > 1 ? b & (0x7Fu >> span) : b;
    for (int k = 1; whole && k < span; ++k) {
      const unsigned char c = static_cast<unsigned char>(p[i + static_cast<size_t>(k)]);
      whole = (c >> 6) == 2;
      cp = (cp << 6) | (c & 0x3Fu);
    }
    if (whole) {
      out += cp;
      i += static_cast<size_t>(span);
    } else {
      out += char32_t{0xFFFD};
      i += 1;
    }
  }
  return out;
}

void append_utf8(char32_t cp, std::string &s) {
  if (cp < 0x80) {
    s += static_cast<char>(cp);
    return;
  }
  const int tail = cp < 0x800 ? 1 : (cp < 0x10000 ? 2 : 3);
  static constexpr unsigned char kLead[4] = {0, 0xC0, 0xE0, 0xF0};
  s += static_cast<char>(kLead[tail] | (cp >> (6 * tail)));
  for (int k = tail - 1; k >= 0; --k) s += static_cast<char>(0x80 | ((cp >> (6 * k)) & 0x3F));
}

// ---- pretokenizer -------------------------------------------------------------

constexpr size_t kMaxWordChars = 100;  // longer words are [UNK] whole

// Code points in, words out: `emit` receives each folded, punctuation-split
// word in order.
template <typename Emit>
void pretokenize(const std::u32string &text, Emit emit) {
  std::u32string raw, folded, piece;
  auto finish_raw = [&]() {
    if (raw.empty()) return;
    folded.clear();
    for (char32_t cp : raw) fold_into(cp, folded);
    raw.clear();
    piece.clear();
    for (char32_t cp : folded) {
      if (!is_punct(cp)) {
        piece += cp;
        continue;
      }
      if (!piece.empty()) emit(piece);
      piece.assign(1, cp);
      emit(piece);
      piece.clear();
    }
    if (!piece.empty()) emit(piece);
  };
  for (char32_t cp : text) {
    if (cp == 0 || cp == 0xFFFD || is_control(cp)) continue;
    if (is_space(cp)) {
      finish_raw();
    } else if (is_han(cp)) {
      finish_raw();
      raw.assign(1, cp);
      finish_raw();
    } else {
      raw += cp;
    }
  }
  finish_raw();
}

}  // namespace

// ---- vocabulary --------------------------------------------------------------

WordPiece WordPiece::from_vocab_file(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("WordPiece vocabulary file could not be opened: " + path);
  std::string blob((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return WordPiece(blob);
}

WordPiece WordPiece::from_vocab_bytes(const char *data, size_t bytes) {
  return WordPiece(std::string(data, bytes));
}

int32_t WordPiece::child(int32_t node, char32_t cp) const {
  const auto it = edges_.find((static_cast<uint64_t>(node) << 21) | cp);
  return it == edges_.end() ? -1 : it->second;
}

int32_t WordPiece::add_child(int32_t node, char32_t cp) {
  const uint64_t key = (static_cast<uint64_t>(node) << 21) | cp;
  const auto it = edges_.find(key);
  if (it != edges_.end()) return it->second;
  const int32_t n = static_cast<int32_t>(node_token_.size());
  node_token_.push_back(-1);
  edges_.emplace(key, n);
  return n;
}

// The blob holds one entry per '\n'-terminated line (a final line without
// '\n' counts; one trailing '\r' is not part of an entry); entry k has id k,
// and a repeated entry keeps its first id.
WordPiece::WordPiece(const std::string &blob) {
  for (size_t at = 0; at < blob.size();) {
    size_t end = blob.find('\n', at);
    if (end == std::string::npos) end = blob.size();
    size_t stop = end;
    if (stop > at && blob[stop - 1] == '\r') --stop;
    vocab_.emplace_back(blob, at, stop - at);
    ids_.emplace(vocab_.back(), static_cast<int32_t>(vocab_.size() - 1));
    at = end + 1;
  }
  if (vocab_.empty()) throw std::runtime_error("WordPiece vocabulary is empty");
  auto special = [&](const char *name) {
    const auto it = ids_.find(name);
    if (it == ids_.end())
      throw std::runtime_error(std::string("WordPiece vocabulary lacks the special token ") + name);
    return it->second;
  };
  cls_id = special("[CLS]");
  sep_id = special("[SEP]");
  pad_id = special("[PAD]");
  unk_id = special("[UNK]");
  for (const char *name : {"[MASK]", "[CLS]", "[SEP]", "[PAD]", "[UNK]"}) {  // longest first
    const auto it = ids_.find(name);
    if (it != ids_.end()) specials_.emplace_back(name, it->second);
  }

  // The tries.  A word's pieces are canonical UTF-8 of their code points, so
  // an entry whose bytes are not the canonical encoding of what they decode
  // to can never match one and is left out.
  node_token_ = {-1, -1};
  auto insert = [&](int32_t root, const char *p, size_t n, int32_t id) {
    const std::u32string cps = decode_utf8(p, n);
    std::string back;
    for (char32_t cp : cps) append_utf8(cp, back);
    if (back.size() != n || back.compare(0, n, p, n) != 0) return;
    int32_t node = root;
    for (char32_t cp : cps) node = add_child(node, cp);
    if (node_token_[static_cast<size_t>(node)] < 0) node_token_[static_cast<size_t>(node)] = id;
  };
  for (size_t id = 0; id < vocab_.size(); ++id) {
    const std::string &e = vocab_[id];
    insert(0, e.data(), e.size(), static_cast<int32_t>(id));
    if (e.size() >= 2 && e[0] == '#' && e[1] == '#')
      insert(1, e.data() + 2, e.size() - 2, static_cast<int32_t>(id));
  }
}

int32_t WordPiece::id_of(const std::string &token) const {
  const auto it = ids_.find(token);
  return it == ids_.end() ? unk_id : it->second;
}

// ---- tokenization ---------------------------------------------------------------

// Greedy longest match: from each position the longest entry of the trie
// (whole entries at the word's start, "##" continuations after it); a word
// with a position where nothing matches is one [UNK].
void WordPiece::word_ids(const std::u32string &word, std::vector<int32_t> &out) const {
  if (word.size() > kMaxWordChars) {
    out.push_back(unk_id);
    return;
  }
  const size_t mark = out.size();
  for (size_t start = 0; start < word.size();) {
    int32_t node = start == 0 ? 0 : 1, hit = -1;
    size_t hit_end = start;
    for (size_t k = start; k < word.size(); ++k) {
      node = child(node, word[k]);
      if (node < 0) break;
      if (node_token_[static_cast<size_t>(node)] >= 0) {
        hit = node_token_[static_cast<size_t>(node)];
        hit_end = k + 1;
      }
    }
    if (hit < 0) {
      out.resize(mark);
      out.push_back(unk_id);
      return;
    }
    out.push_back(hit);
    start = hit_end;
  }
}

// Special tokens written in the text stay whole: at each byte position the
// longest special that starts there is taken, and the text between specials
// is pretokenized.
void WordPiece::piece_ids(const std::string &text, std::vector<int32_t> &out) const {
  auto plain = [&](size_t from, size_t to) {
    if (to <= from) return;
    pretokenize(decode_utf8(text.data() + from, to - from),
                [&](const std::u32string &w) { word_ids(w, out); });
  };
  size_t from = 0;
  for (size_t i = 0; i < text.size(); ++i) {
    if (text[i] != '[') continue;  // every special token starts with '['
    for (const auto &s : specials_) {
      if (text.compare(i, s.first.size(), s.first) != 0) continue;
      plain(from, i);
      out.push_back(s.second);
      from = i + s.first.size();
      i = from - 1;
      break;
    }
  }
  plain(from, text.size());
}

std::vector<std::string> WordPiece::tokenize(const std::string &text) const {
  std::vector<int32_t> ids;
  piece_ids(text, ids);
  std::vector<std::string> out;
  out.reserve(ids.size());
  for (int32_t id : ids) out.push_back(vocab_[static_cast<size_t>(id)]);
  return out;
}

Tokens WordPiece::encode(const std::string &text, int max_len) const {
  if (max_len < 2)
    throw std::runtime_error("WordPiece: a sequence length below 2 cannot hold [CLS] and [SEP]");
  std::vector<int32_t> pieces;
  piece_ids(text, pieces);
  const size_t room = static_cast<size_t>(max_len) - 2, kept = std::min(pieces.size(), room);
  Tokens t;
  t.truncated = pieces.size() > room;
  t.n_tokens = static_cast<int32_t>(kept + 2);
  t.ids.assign(static_cast<size_t>(max_len), pad_id);
  t.mask.assign(static_cast<size_t>(max_len), 0);
  t.ids[0] = cls_id;
  std::copy(pieces.begin(), pieces.begin() + static_cast<std::ptrdiff_t>(kept), t.ids.begin() + 1);
  t.ids[kept + 1] = sep_id;
  std::fill(t.mask.begin(), t.mask.begin() + static_cast<std::ptrdiff_t>(kept + 2), 1);
  return t;
}

}  // namespace nebw
