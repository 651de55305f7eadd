// nebw_embed -- the embedding CLI path of the reference (`npuembeddings embed`,
// runtime/include/runtime/run_execute.hpp:150-258, embed_service.cpp:29-64)
// with the encoder on a B200, through the C++ host side of the library.
//
//   nebw_embed <model.npue> <ids.i32> <mask.i32> <seq> <out.f32> [devices]
//       token ids and the 1/0 attention mask as raw little-endian int32
//       [n, seq] (as a tokenizer emits them, padded to seq) -> raw fp32
//       [n, hidden] pooled embeddings
//   nebw_embed --text <model.npue> <texts.txt> <seq> <out.f32> [devices] [--vocab v.txt]
//       one text per line, WordPiece-tokenized on the host (wordpiece.hpp)
//       with the vocabulary the container carries (tokenizer.vocab) or
//       --vocab, then encoded on the GPU
//   nebw_embed --tokenize <model.npue|vocab.txt> <texts.txt> <seq> <ids.i32> <mask.i32>
//       the tokenizer alone (no GPU): the ids and mask files of the first form
//   nebw_embed --prepare-model <checkpoint_dir> <out.npue> [tma_bf16|host] [max_seq]
//       the packer (no GPU): a Hugging Face BERT checkpoint -> a container
//       (the runtime's --prepare-model, runtime/src/cli/cli.cpp:60)
//
// `devices` is one GPU index or a comma-separated list ("0,1,2,3"): with
// several, the batch is sharded over them and gathered back in request
// order (one weight replica per GPU).
//
// Exit status 0 on success, 1 with the cause on stderr otherwise.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../csrc/npue_file.h"
#include "gpu_bert_encoder.hpp"
#include "wordpiece.hpp"

namespace {
std::vector<int32_t> read_i32(const std::string &path) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) throw std::runtime_error("cannot open " + path);
  const std::streamsize n = f.tellg();
  if (n % 4) throw std::runtime_error(path + " is not a whole number of int32");
  std::vector<int32_t> v(static_cast<size_t>(n / 4));
  f.seekg(0);
  f.read(reinterpret_cast<char *>(v.data()), n);
  return v;
}

template <typename T>
void write_raw(const std::string &path, const std::vector<T> &v) {
  std::ofstream o(path, std::ios::binary);
  o.write(reinterpret_cast<const char *>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
  if (!o) throw std::runtime_error("cannot write " + path);
}

std::vector<std::string> read_lines(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::vector<std::string> out;
  std::string line;
  while (std::getline(f, line)) {
    if (!line.empty() && line.back() == '\r') line.pop_back();
    out.push_back(line);
  }
  return out;
}

bool ends_with(const std::string &s, const char *suffix) {
  const size_t n = std::strlen(suffix);
  return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

// The vocabulary a container carries (the packer's tokenizer.vocab), or a
// vocab.txt file.
nebw::WordPiece load_vocab(const std::string &path) {
  if (!ends_with(path, ".npue")) return nebw::WordPiece::from_vocab_file(path);
  nebw::NpueFile f(path);
  if (!f.has("tokenizer.vocab"))
    throw std::runtime_error(path + " carries no tokenizer.vocab; pass --vocab vocab.txt");
  const auto &t = f.tensor("tokenizer.vocab");
  return nebw::WordPiece::from_vocab_bytes(reinterpret_cast<const char *>(t.data), t.nbytes);
}

void tokenize_all(const nebw::WordPiece &wp, const std::vector<std::string> &texts, int seq,
                  std::vector<int32_t> &ids, std::vector<int32_t> &mask) {
  ids.clear();
  mask.clear();
  for (const auto &t : texts) {
    const nebw::Tokens e = wp.encode(t, seq);
    ids.insert(ids.end(), e.ids.begin(), e.ids.end());
    mask.insert(mask.end(), e.mask.begin(), e.mask.end());
  }
}

// "0" or "0,1,3" -> GPU indices
std::vector<int> parse_devices(const std::string &s) {
  std::vector<int> v;
  size_t at = 0;
  while (at <= s.size()) {
    const size_t c = s.find(',', at);
    const std::string part = s.substr(at, c == std::string::npos ? std::string::npos : c - at);
    if (part.empty() || part.find_first_not_of("0123456789") != std::string::npos)
      throw std::runtime_error("bad device list '" + s + "'");
    v.push_back(std::atoi(part.c_str()));
    if (c == std::string::npos) break;
    at = c + 1;
  }
  return v;
}

int usage(const char *argv0) {
  std::fprintf(stderr,
               "usage: %s <model.npue> <ids.i32> <mask.i32> <seq> <out.f32> [devices]\n"
               "       %s --text <model.npue> <texts.txt> <seq> <out.f32> [devices] [--vocab v.txt]\n"
               "       %s --tokenize <model.npue|vocab.txt> <texts.txt> <seq> <ids.i32> <mask.i32>\n"
               "       %s --prepare-model <checkpoint_dir> <out.npue> [tma_bf16|host] [max_seq]\n",
               argv0, argv0, argv0, argv0);
  return 2;
}
}  // namespace

int main(int argc, char **argv) {
  try {
    if (argc >= 2 && std::strcmp(argv[1], "--prepare-model") == 0) {
      if (argc < 4 || argc > 6) return usage(argv[0]);
      const char *layout = argc > 4 ? argv[4] : "tma_bf16";
      const int max_seq = argc > 5 ? std::atoi(argv[5]) : 0;
      uint64_t bytes = 0;
      nebw::check(nebw_pack_checkpoint(argv[2], argv[3], layout, max_seq, 1, &bytes));
      std::printf("%s: %llu bytes, layout %s\n", argv[3], static_cast<unsigned long long>(bytes),
                  layout);
      return 0;
    }
    if (argc >= 2 && std::strcmp(argv[1], "--tokenize") == 0) {
      if (argc != 7) return usage(argv[0]);
      const nebw::WordPiece wp = load_vocab(argv[2]);
      std::vector<int32_t> ids, mask;
      tokenize_all(wp, read_lines(argv[3]), std::atoi(argv[4]), ids, mask);
      write_raw(argv[5], ids);
      write_raw(argv[6], mask);
      return 0;
    }
    if (argc >= 2 && std::strcmp(argv[1], "--text") == 0) {
      if (argc < 6) return usage(argv[0]);
      std::string vocab = argv[2];
      std::vector<int> devices{0};
      for (int i = 6; i < argc; ++i) {
        if (std::strcmp(argv[i], "--vocab") == 0 && i + 1 < argc) vocab = argv[++i];
        else devices = parse_devices(argv[i]);
      }
      const int seq = std::atoi(argv[4]);
      const nebw::WordPiece wp = load_vocab(vocab);
      const std::vector<std::string> texts = read_lines(argv[3]);
      std::vector<int32_t> ids, mask;
      tokenize_all(wp, texts, seq, ids, mask);
      nebw::GpuBertEncoder enc(argv[2], devices);
      const std::vector<float> out =
          enc.encode(ids, mask, static_cast<int64_t>(texts.size()), seq);
      write_raw(argv[5], out);
      std::printf("%zu texts -> %zu embeddings of %lld dims -> %s\n", texts.size(), texts.size(),
                  static_cast<long long>(enc.hidden()), argv[5]);
      return 0;
    }
    if (argc < 6) return usage(argv[0]);
    const int64_t seq = std::atoll(argv[4]);
    const std::vector<int> devices = argc > 6 ? parse_devices(argv[6]) : std::vector<int>{0};
    const std::vector<int32_t> ids = read_i32(argv[2]), mask = read_i32(argv[3]);
    if (seq <= 0 || ids.size() % seq || mask.size() != ids.size())
      throw std::runtime_error("ids/mask sizes do not match seq");
    const int64_t n = static_cast<int64_t>(ids.size()) / seq;
    nebw::GpuBertEncoder enc(argv[1], devices);
    const std::vector<float> out = enc.encode(ids, mask, n, seq);
    write_raw(argv[5], out);
    std::printf("%lld embeddings of %lld dims -> %s\n", static_cast<long long>(n),
                static_cast<long long>(enc.hidden()), argv[5]);
    return 0;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "nebw_embed: %s\n", e.what());
    return 1;
  }
}
