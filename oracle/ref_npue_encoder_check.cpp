// TEST INFRASTRUCTURE ONLY -- the serving drop-in compiled against the
// reference's own headers and tokenizer.
//
//   npue_encoder_check <model.npue> <texts.txt> <seq> <out.f32> <ids.i32> <mask.i32> [reps]
//
// Opens the container with the reference's npue::File, takes the reference's
// own tokenizer from it (app::load_tokenizer, tokenizer_facade.hpp:129), wraps
// libnebw in nebw::GpuNpueEncoder (host/npue_gpu_encoder.hpp) and uses it ONLY
// through the reference's interface, npue::Encoder &, the way the runtime's
// encode path holds its encoder.  Writes the embeddings and the tokenizer's
// ids / mask (so the test can run the CPU oracle on the very same tokens),
// and prints one line: texts, tokens, seconds for `reps` timed encode calls
// after one untimed call.  Built by oracle/Makefile `encoder_check` from the
// reference tree where it lies, linked with libnebw.so.
#include <chrono>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "npue_gpu_encoder.hpp"
#include "runtime/model.hpp"
#include "tokenizers/tokenizer_facade.hpp"

namespace {

std::vector<std::string> read_lines(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::vector<std::string> v;
  for (std::string s; std::getline(f, s);) v.push_back(s);
  return v;
}

template <class T>
void write_all(const std::string &path, const std::vector<T> &v) {
  std::ofstream f(path, std::ios::binary);
  f.write(reinterpret_cast<const char *>(v.data()), static_cast<std::streamsize>(v.size() * sizeof(T)));
  if (!f) throw std::runtime_error("cannot write " + path);
}

}  // namespace

int main(int argc, char **argv) {
  if (argc < 7) {
    std::fprintf(stderr, "usage: %s model.npue texts.txt seq out.f32 ids.i32 mask.i32 [reps]\n",
                 argv[0]);
    return 2;
  }
  try {
    const std::string model = argv[1];
    const std::vector<std::string> texts = read_lines(argv[2]);
    const int64_t seq = std::stoll(argv[3]);
    const int reps = argc > 7 ? std::stoi(argv[7]) : 0;
    npue::File file(model);
    const app::AnyTokenizer tok = app::load_tokenizer(file, model);
    nebw::GpuNpueEncoder<app::AnyTokenizer> gpu(model, tok, seq, 0);
    npue::Encoder &enc = gpu;  // the reference's interface, nothing else
    int64_t ntok = 0;
    const std::vector<float> out = enc.encode(texts, "", &ntok);
    if (static_cast<int64_t>(out.size()) != static_cast<int64_t>(texts.size()) * enc.hidden())
      throw std::runtime_error("encode returned the wrong shape");
    std::vector<int32_t> ids, mask;
    for (const auto &t : texts) {
      const npue::Encoded e = tok.encode(t, static_cast<int>(seq));
      ids.insert(ids.end(), e.input_ids.begin(), e.input_ids.end());
      mask.insert(mask.end(), e.attention_mask.begin(), e.attention_mask.end());
    }
    write_all(argv[4], out);
    write_all(argv[5], ids);
    write_all(argv[6], mask);
    double secs = 0.0;
    if (reps > 0) {
      const auto t0 = std::chrono::steady_clock::now();
      for (int r = 0; r < reps; ++r) enc.encode(texts, "", nullptr);
      secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    }
    std::printf("texts %zu tokens %lld reps %d seconds %.6f hidden %lld seq %lld\n", texts.size(),
                static_cast<long long>(ntok), reps, secs, static_cast<long long>(enc.hidden()),
                static_cast<long long>(enc.seq()));
    return 0;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
}
