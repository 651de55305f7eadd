// nebw_embed -- file in, file out, through the C++ host side of the library.
//
//   nebw_embed <model.npue> <ids.i32> <mask.i32> <seq> <out.f32> [device]
//
// ids.i32 / mask.i32: raw little-endian int32 [n, seq] (token ids and the 1/0
// attention mask as a tokenizer emits them, padded to seq); out.f32: raw
// fp32 [n, hidden] pooled embeddings.  The batch path of the reference's
// `npuembeddings embed` after tokenisation (runtime/include/runtime/
// run_execute.hpp:150-258, embed_service.cpp:29-64), with the encoder on a
// B200.  Exit status 0 on success, 1 with the cause on stderr otherwise.
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "gpu_bert_encoder.hpp"

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
}  // namespace

int main(int argc, char **argv) {
  if (argc < 6) {
    std::fprintf(stderr, "usage: %s <model.npue> <ids.i32> <mask.i32> <seq> <out.f32> [device]\n",
                 argv[0]);
    return 2;
  }
  try {
    const int64_t seq = std::atoll(argv[4]);
    const int device = argc > 6 ? std::atoi(argv[6]) : 0;
    const std::vector<int32_t> ids = read_i32(argv[2]), mask = read_i32(argv[3]);
    if (seq <= 0 || ids.size() % seq || mask.size() != ids.size())
      throw std::runtime_error("ids/mask sizes do not match seq");
    const int64_t n = static_cast<int64_t>(ids.size()) / seq;
    nebw::GpuBertEncoder enc(argv[1], device);
    const std::vector<float> out = enc.encode(ids, mask, n, seq);
    std::ofstream o(argv[5], std::ios::binary);
    o.write(reinterpret_cast<const char *>(out.data()),
            static_cast<std::streamsize>(out.size() * sizeof(float)));
    if (!o) throw std::runtime_error(std::string("cannot write ") + argv[5]);
    std::printf("%lld embeddings of %lld dims -> %s\n", static_cast<long long>(n),
                static_cast<long long>(enc.hidden()), argv[5]);
    return 0;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "nebw_embed: %s\n", e.what());
    return 1;
  }
}
