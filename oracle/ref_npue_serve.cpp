// TEST INFRASTRUCTURE ONLY -- `npuembeddings serve` with the encoder on the
// GPU, built from the reference's own serving code.
//
//   npue_serve_gpu <model.npue> <port> [seq]
//
// The reference's HTTP server and /v1/embeddings handler (app::serve_http,
// runtime/src/server/embed_backend.cpp, compiled from the reference tree by
// oracle/Makefile `serve_check`), its container reader and its own
// tokenizer (app::load_tokenizer), with nebw::GpuNpueEncoder
// (host/npue_gpu_encoder.hpp) as the app::EmbedBackend's embed function and
// the runtime's own truncation policy (app::check_truncation: an input over
// the sequence length is npue::InputTooLong, HTTP 400), each request shape's
// pass replayed as a CUDA graph.  This is the wiring
// a maintainer adds to the runtime's `serve` subcommand
// (runtime/src/cli/subcommand.cpp:202-274) in place of make_service's
// BertEncoder lanes.  Serves on 127.0.0.1 until SIGINT / SIGTERM.
#include <cstdio>
#include <string>
#include <vector>

#include "common/app_state.hpp"
#include "npue_gpu_encoder.hpp"
#include "runtime/model.hpp"
#include "server/embed_backend.hpp"
#include "tokenizers/tokenizer_facade.hpp"

int main(int argc, char **argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: %s model.npue port [seq]\n", argv[0]);
    return 2;
  }
  try {
    const std::string model = argv[1];
    const int port = std::stoi(argv[2]);
    npue::File file(model);
    const int64_t seq = argc > 3 ? std::stoll(argv[3]) : file.config_int("max_seq_len");
    const app::AnyTokenizer tok = app::load_tokenizer(file, model);
    nebw::GpuNpueEncoder<app::AnyTokenizer> gpu(model, tok, seq, 0, app::check_truncation);
    gpu.gpu().use_graphs(true);  // a server's requests come in a few batch shapes
    app::EmbedBackend be;
    be.vocab_size = tok.vocab_size();
    be.hidden = gpu.hidden();
    be.seq = gpu.seq();
    be.embed = [&gpu](const std::vector<std::string> &texts, const std::string &prefix,
                      int64_t *tokens) { return gpu.encode(texts, prefix, tokens); };
    return app::serve_http(be, "nebw-gpu", port, "127.0.0.1");
  } catch (const std::exception &e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
}
