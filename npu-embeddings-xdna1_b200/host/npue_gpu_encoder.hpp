// GpuNpueEncoder -- libnebw behind the reference runtime's own encoder
// interface, npue::Encoder (runtime/include/runtime/encoder.hpp:19-27):
// texts in, pooled + L2-normalised [batch][hidden] fp32 out.
//
// This header is compiled inside the reference runtime: its include path
// holds the reference's runtime/include (for runtime/encoder.hpp and
// runtime/types.hpp) and this repo's include/ and host/ directories.  The
// tokenizer stays the runtime's own -- any type with
//   npue::Encoded encode(const std::string &text, int max_len) const
// (app::AnyTokenizer, tokenizer_facade.hpp:84) -- as does the truncation
// policy: the callback gets what app::check_truncation
// (common/app_state.hpp:73-87) takes, and by default refuses a cut input the
// way that function does without --allow-truncation.
//
// encode() does what EmbedService::chunk does around BertEncoder::run
// (runtime/src/server/embed_service.cpp:29-64): prefix + text through the
// tokenizer at the runtime's sequence length, the truncation check per row,
// the token count summed into *tokens; then one GPU pass over the batch
// (GpuBertEncoder: the embedding gather, the encoder, pooling and L2 on the
// device) instead of the host embedding build, run() and pool_rows().
#pragma once

#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

#include "gpu_bert_encoder.hpp"
#include "runtime/encoder.hpp"
#include "runtime/types.hpp"

namespace nebw {

template <class Tokenizer>
class GpuNpueEncoder final : public npue::Encoder {
 public:
  // (truncated, tokens before the cut, the input's index, the limit)
  using TruncationCheck = std::function<void(bool, int32_t, size_t, int64_t)>;

  // `seq`: the runtime's sequence length (g_seq), at most the container's
  // max_seq_len.  `tok` must outlive the encoder.
  GpuNpueEncoder(const std::string &npue_path, const Tokenizer &tok, int64_t seq, int device = 0,
                 TruncationCheck check = {})
      : gpu_(npue_path, device), tok_(tok), seq_(seq), check_(std::move(check)) {
    if (seq_ <= 1 || seq_ > gpu_.max_seq())
      throw std::runtime_error("nebw: sequence length " + std::to_string(seq_) +
                               " is outside [2, the container's max_seq_len " +
                               std::to_string(gpu_.max_seq()) + "]");
    if (!check_)
      check_ = [](bool truncated, int32_t full, size_t index, int64_t limit) {
        if (truncated)
          throw std::runtime_error("input " + std::to_string(index) + " is " +
                                   std::to_string(full) + " tokens; the limit is " +
                                   std::to_string(limit));
      };
  }

  std::vector<float> encode(const std::vector<std::string> &texts, const std::string &prefix,
                            int64_t *tokens) override {
    const int64_t n = static_cast<int64_t>(texts.size());
    std::vector<int32_t> ids(static_cast<size_t>(n * seq_)), mask(ids.size());
    int64_t ntok = 0;
    for (int64_t b = 0; b < n; ++b) {
      const npue::Encoded en = tok_.encode(prefix.empty() ? texts[b] : prefix + texts[b],
                                           static_cast<int>(seq_));
      check_(en.truncated, en.n_tokens_full, static_cast<size_t>(b), seq_);
      if (static_cast<int64_t>(en.input_ids.size()) != seq_ ||
          en.attention_mask.size() != en.input_ids.size())
        throw std::runtime_error("nebw: the tokenizer did not pad input " + std::to_string(b) +
                                 " to the sequence length");
      std::copy(en.input_ids.begin(), en.input_ids.end(), ids.begin() + b * seq_);
      std::copy(en.attention_mask.begin(), en.attention_mask.end(), mask.begin() + b * seq_);
      ntok += en.n_tokens;
    }
    std::vector<float> out = gpu_.encode(ids, mask, n, seq_);
    if (tokens) *tokens += ntok;
    return out;
  }

  int64_t hidden() const override { return gpu_.hidden(); }
  int64_t seq() const override { return seq_; }

  GpuBertEncoder &gpu() { return gpu_; }

 private:
  GpuBertEncoder gpu_;
  const Tokenizer &tok_;
  int64_t seq_;
  TruncationCheck check_;
};

}  // namespace nebw
