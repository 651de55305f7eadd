// The weight packer in C++: a Hugging Face BERT checkpoint directory ->
// a `.npue` container, in this library's tma_bf16 layout (bf16 [N, K]
// GEMM operands, uploaded with no re-tiling) or the reference packer's host
// layout (F32 [K, N]).  Replaces the BERT branch of the reference's packer
// (tools/pack/pack_npue.py:2620-2835; its C++ counterpart
// runtime/src/common/npue_pack.cpp is the runtime's --prepare-model).
#pragma once

#include <cstdint>
#include <string>

namespace nebw {

struct PackOptions {
  std::string layout = "tma_bf16";  // "tma_bf16" or "host"
  int64_t max_seq = 256;            // position-table rows kept
  bool fold_scale = true;           // 1/sqrt(head_dim) into the Q columns and bias
};

// Writes the container; returns its size in bytes.  Throws
// std::runtime_error naming the cause.
uint64_t pack_checkpoint(const std::string &model_dir, const std::string &out_path,
                         const PackOptions &opt);

// SHA-256 (FIPS 180-4) of a byte string, lower-case hex.
std::string sha256_hex(const void *data, size_t n);

}  // namespace nebw
