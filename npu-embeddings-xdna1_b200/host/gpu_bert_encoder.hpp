// GpuBertEncoder -- the reference runtime's encoder interface over libnebw.
//
// Header-only C++17 host side of the drop-in.  It mirrors the shape of the
// reference's encoder and the call EmbedService::chunk makes on it
// (runtime/src/server/embed_service.cpp:29-64: token ids and the 1/0
// attention mask as the tokenizer emits them, padded to the sequence length;
// pooled, L2-normalised [batch, hidden] fp32 out), and the reference's error
// convention: every failure is a std::runtime_error whose text names the
// cause (nebw_last_error()).
//
// Behaviour matched to the reference beyond the arithmetic:
//   * a row whose mask is all zero is the reference's "empty sequence":
//     mean pooling returns the zero vector (pool_rows divides a zero sum by
//     max(0, 1e-9) and L2-normalises with the 1e-24 floor), CLS pooling
//     throws "CLS pooling on a sequence whose first token is masked"
//     (runtime/include/common/app_state.hpp:345-347);
//   * a mask that is not a prefix of ones cannot come from the reference's
//     tokenizers (wordpiece.cpp:354-378) and is refused rather than answered
//     for a different input.
//
// Link with -lnebw (libnebw.so) and include this header with include/ on
// the include path.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "nebw.h"

namespace nebw {

inline void check(int rc) {
  if (rc != NEBW_OK) throw std::runtime_error(std::string("nebw: ") + nebw_last_error());
}

class GpuBertEncoder {
 public:
  // Open GPU `device` and stage every tensor of the `.npue` container at
  // `npue_path` (the reference's npue::File + set_model_shape + stage_all).
  GpuBertEncoder(const std::string &npue_path, int device = 0)
      : GpuBertEncoder(npue_path, std::vector<int>{device}) {}

  // The same over several GPUs of this process: one weight replica per GPU,
  // each batch split by the library's length-balanced plan and gathered back
  // in request order over NCCL (nebw_comm_init_all + nebw_encode_multi), one
  // host thread per GPU -- the reference's --pipeline lanes
  // (embed_service.cpp:66-108) over GPUs.  `timeout_s` bounds every
  // collective wait.
  GpuBertEncoder(const std::string &npue_path, const std::vector<int> &devices,
                 double timeout_s = 60.0) {
    if (devices.empty()) throw std::runtime_error("nebw: no GPU given");
    try {
      for (int d : devices) {
        nebw_dev *dev = nullptr;
        check(nebw_open(d, &dev));
        devs_.push_back(dev);
        nebw_model *m = nullptr;
        check(nebw_model_load_npue(dev, npue_path.c_str(), &m));
        models_.push_back(m);
      }
      if (devs_.size() > 1) {
        comms_.assign(devs_.size(), nullptr);
        check(nebw_comm_init_all(static_cast<int32_t>(devs_.size()), devs_.data(), timeout_s,
                                 comms_.data()));
      }
      check(nebw_model_get_config(models_[0], &cfg_));
    } catch (...) {
      release();
      throw;
    }
    dev_ = devs_[0];
    model_ = models_[0];
  }
  ~GpuBertEncoder() { release(); }
  GpuBertEncoder(const GpuBertEncoder &) = delete;
  GpuBertEncoder &operator=(const GpuBertEncoder &) = delete;

  int64_t hidden() const { return cfg_.hidden; }
  int64_t max_seq() const { return cfg_.max_seq_len; }
  bool cls_pooling() const { return cfg_.pooling == NEBW_POOL_CLS; }

  // ids, attention_mask: [batch, seq] row-major.  Returns [batch, hidden].
  std::vector<float> encode(const std::vector<int32_t> &ids,
                            const std::vector<int32_t> &attention_mask, int64_t batch,
                            int64_t seq) {
    if (batch < 0 || seq <= 0 || ids.size() != static_cast<size_t>(batch * seq) ||
        attention_mask.size() != ids.size())
      throw std::runtime_error("nebw: ids/mask must both hold batch * seq values");
    std::vector<float> out(static_cast<size_t>(batch) * cfg_.hidden, 0.f);
    if (batch == 0) return out;
    // Lengths from the mask; all-zero rows are set aside (see the header).
    std::vector<int32_t> lens, keep_ids;
    std::vector<int64_t> keep;
    for (int64_t b = 0; b < batch; ++b) {
      int32_t len = 0;
      while (len < seq && attention_mask[b * seq + len] != 0) ++len;
      for (int64_t s = len; s < seq; ++s)
        if (attention_mask[b * seq + s] != 0)
          throw std::runtime_error("nebw: attention mask of row " + std::to_string(b) +
                                   " is not a prefix of ones");
      if (len == 0) {
        if (cls_pooling())
          throw std::runtime_error("CLS pooling on a sequence whose first token is masked");
        continue;  // mean pooling of an empty row: the zero vector
      }
      keep.push_back(b);
      lens.push_back(len);
      keep_ids.insert(keep_ids.end(), ids.begin() + b * seq, ids.begin() + (b + 1) * seq);
    }
    if (keep.empty()) return out;
    std::vector<float> got(keep.size() * cfg_.hidden);
    if (comms_.empty())
      check(nebw_encode(model_, keep_ids.data(), lens.data(), static_cast<int32_t>(keep.size()),
                        static_cast<int32_t>(seq), got.data()));
    else
      check(nebw_encode_multi(static_cast<int32_t>(models_.size()), models_.data(), comms_.data(),
                              keep_ids.data(), lens.data(), static_cast<int32_t>(keep.size()),
                              static_cast<int32_t>(seq), got.data()));
    for (size_t i = 0; i < keep.size(); ++i)
      std::copy(got.begin() + i * cfg_.hidden, got.begin() + (i + 1) * cfg_.hidden,
                out.begin() + keep[i] * cfg_.hidden);
    return out;
  }

  // Replay each (batch, seq) shape's pass as a CUDA graph (nebw_model_set_graphs):
  // the same embeddings bit for bit, one launch per request instead of ~7 per
  // layer (measured: one bge-large sequence 2.45 -> 2.11 ms, one bge-small
  // sequence 0.78 -> 0.61 ms).  Worth it when requests come in a few batch
  // shapes, as a server's do; each new shape is captured once (up to 16 kept).
  // Single-GPU encoders only.
  void use_graphs(bool on) {
    if (!comms_.empty()) throw std::runtime_error("nebw: graphs are for the single-GPU encoder");
    check(nebw_model_set_graphs(model_, on ? 1 : 0));
  }

  nebw_model *model() { return model_; }
  nebw_dev *device() { return dev_; }
  size_t gpus() const { return devs_.size(); }

 private:
  void release() {
    for (nebw_comm *c : comms_) nebw_comm_destroy(c);
    for (nebw_model *m : models_) nebw_model_destroy(m);
    for (nebw_dev *d : devs_) nebw_close(d);
    comms_.clear();
    models_.clear();
    devs_.clear();
  }

  std::vector<nebw_dev *> devs_;
  std::vector<nebw_model *> models_;
  std::vector<nebw_comm *> comms_;  // empty on one GPU
  nebw_dev *dev_ = nullptr;
  nebw_model *model_ = nullptr;
  nebw_config cfg_{};
};

}  // namespace nebw
