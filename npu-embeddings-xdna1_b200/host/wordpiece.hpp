// BERT WordPiece tokenizer for the host tools: text -> [CLS] ids [SEP] + pad
// and the attention mask, with the output contract of the runtime's tokenizer
// for the embedding models (npue::WordPiece, runtime/include/tokenizers/
// wordpiece.hpp).  The algorithm is HuggingFace's BertTokenizer
// (BasicTokenizer with do_lower_case and tokenize_chinese_chars, then
// WordpieceTokenizer with max_input_chars_per_word = 100), written here as
// two stages:
//
//   Pretokenizer  UTF-8 -> code points -> words: U+0000, U+FFFD and control
//                 characters dropped, whitespace separates words, each Han
//                 ideograph is a word of its own, each code point of a word
//                 is folded (lower case, canonical decomposition, nonspacing
//                 marks removed; one table lookup, Hangul syllables
//                 decomposed arithmetically), and every punctuation code
//                 point splits off as a word of its own.
//   PieceTrie     the vocabulary as two code-point tries -- whole entries,
//                 and the "##" continuation entries without their prefix --
//                 walked for the longest entry at each position of a word;
//                 a word with a position nothing matches, or longer than 100
//                 code points, becomes [UNK].
//
// Special tokens ([CLS] [SEP] [PAD] [UNK] [MASK], those the vocabulary has)
// written in the raw text are kept whole.  The Unicode tables
// (bert_unicode.inc) are generated from Python's unicodedata by
// gen_unicode_tables.py.
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

  // The pieces of `text` (no [CLS] / [SEP]), as vocabulary strings.
  std::vector<std::string> tokenize(const std::string &text) const;
  // [CLS] + the first max_len - 2 pieces + [SEP], then [PAD] up to max_len.
  Tokens encode(const std::string &text, int max_len) const;
  int32_t id_of(const std::string &token) const;
  size_t vocab_size() const { return vocab_.size(); }

  int32_t cls_id = -1, sep_id = -1, pad_id = -1, unk_id = -1;

 private:
  explicit WordPiece(const std::string &blob);
  void piece_ids(const std::string &text, std::vector<int32_t> &out) const;
  void word_ids(const std::u32string &word, std::vector<int32_t> &out) const;
  int32_t child(int32_t node, char32_t cp) const;
  int32_t add_child(int32_t node, char32_t cp);

  std::vector<std::string> vocab_;                // id -> entry
  std::unordered_map<std::string, int32_t> ids_;  // entry -> first id
  // trie over code points: node 0 roots whole entries, node 1 the "##"
  // continuations; edges keyed by (node << 21) | code point
  std::unordered_map<uint64_t, int32_t> edges_;
  std::vector<int32_t> node_token_;           // entry id ending at a node, or -1
  std::vector<std::pair<std::string, int32_t>> specials_;  // longest first
};

}  // namespace nebw
