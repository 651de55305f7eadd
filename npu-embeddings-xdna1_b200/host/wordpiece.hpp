// BERT WordPiece tokenizer for the host tools: text -> [CLS] ids [SEP] + pad,
// the attention mask, as the runtime's tokenizer produces them for the
// embedding models (npue::WordPiece, runtime/include/tokenizers/wordpiece.hpp,
// runtime/src/tokenizers/wordpiece.cpp).  Same pipeline, in HuggingFace
// BasicTokenizer order:
//
//   clean      drop U+0000, U+FFFD and control characters; whitespace -> ' '
//   CJK        Han ideographs padded with spaces (one token each); Hiragana,
//              Katakana and Hangul are not "CJK" in this sense
//   split      on spaces
//   fold       per code point: lower(), NFD, drop Mn marks (one table lookup;
//              Hangul syllables decomposed arithmetically)
//   punct      every punctuation code point its own token
//   wordpiece  greedy longest match first, "##" continuations, a piece with
//              no match (or longer than 100 code points) becomes [UNK]
//   specials   [CLS] [SEP] [PAD] [UNK] [MASK] in the raw text stay single
//              tokens
//
// encode(): [CLS] + the first max_len - 2 tokens + [SEP], then [PAD] up to
// max_len; mask 1 on the real positions.  Invalid UTF-8 bytes decode to
// U+FFFD and are dropped.  The Unicode tables (bert_unicode.inc) are
// generated from Python's unicodedata by gen_unicode_tables.py.
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace nebw {

struct Tokens {
  std::vector<int32_t> ids, mask;  // [max_len]
  int32_t n_tokens = 0;            // real positions, [CLS] and [SEP] included
  bool truncated = false;
};

class WordPiece {
 public:
  static WordPiece from_vocab_file(const std::string &path);
  static WordPiece from_vocab_bytes(const char *data, size_t bytes);

  std::vector<std::string> tokenize(const std::string &text) const;
  Tokens encode(const std::string &text, int max_len) const;
  int32_t id_of(const std::string &token) const;
  size_t vocab_size() const { return tokens_.size(); }

  int32_t cls_id = -1, sep_id = -1, pad_id = -1, unk_id = -1;

 private:
  void index(const std::string &blob);
  std::vector<std::string> tokenize_text(const std::string &text) const;
  void wordpiece(const std::vector<uint32_t> &piece, std::vector<std::string> &out) const;

  std::vector<std::string> tokens_;
  std::unordered_map<std::string, int32_t> id_;
  std::vector<std::string> specials_;  // longest first
};

}  // namespace nebw
