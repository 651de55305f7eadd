// The weight packer in C++ (see npue_pack.h).
//
// Input: a checkpoint directory with config.json, 1_Pooling/config.json (the
// pooling mode), optionally CHECKPOINT.json (repo_id) and vocab.txt, and the
// weights as model.safetensors (or pytorch_model.safetensors): an 8-byte
// little-endian header length, a JSON header {name: {dtype, shape,
// data_offsets}}, raw little-endian data.  F32, F16, BF16 and F64 tensors
// are read (widened or rounded to fp32).
//
// The transformation is the reference packer's BERT branch
// (tools/pack/pack_npue.py:2703-2790) -- Q, K and V fused along N, every
// nn.Linear weight [out, in] transposed to [K = in, N = out],
// 1/sqrt(head_dim) folded into the Q columns and the Q bias in fp32, the
// position table cut to max_seq_len, the tensor names, config keys and
// tensor order that packer writes -- so the `host` layout is the reference
// packer's --dtype f32 container.  `tma_bf16` stores each GEMM operand as
// bf16 (round to nearest even) [N, K], with the layout descriptor and hash
// the library's loader checks.  The container, including its JSON directory,
// is byte-identical to the one nebw/pack.py writes for the same checkpoint
// (tests/test_pack.py).
#include "npue_pack.h"

#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <vector>

#include "npue_file.h"

namespace nebw {
namespace {

// ---- SHA-256 -------------------------------------------------------------
// The round constants and initial state are the first 32 fractional bits of
// the cube roots (resp. square roots) of the first primes, computed here
// exactly with integer roots.

using u128 = unsigned __int128;

uint64_t iroot(u128 v, int k) {  // floor(v^(1/k)), k = 2 or 3
  uint64_t lo = 0, hi = 1ull << 43;
  while (lo < hi) {
    const uint64_t mid = lo + (hi - lo + 1) / 2;
    u128 p = mid;
    for (int i = 1; i < k; ++i) p *= mid;
    if (p <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

struct ShaTables {
  uint32_t k[64], h0[8];
  ShaTables() {
    int n = 0;
    for (uint32_t p = 2; n < 64; ++p) {
      bool prime = true;
      for (uint32_t d = 2; d * d <= p; ++d)
        if (p % d == 0) prime = false;
      if (!prime) continue;
      k[n] = static_cast<uint32_t>(iroot(static_cast<u128>(p) << 96, 3));
      if (n < 8) h0[n] = static_cast<uint32_t>(iroot(static_cast<u128>(p) << 64, 2));
      ++n;
    }
  }
};

uint32_t rotr(uint32_t x, int r) { return (x >> r) | (x << (32 - r)); }

}  // namespace

std::string sha256_hex(const void *data, size_t n) {
  static const ShaTables t;
  uint32_t h[8];
  std::memcpy(h, t.h0, sizeof h);
  const uint8_t *p = static_cast<const uint8_t *>(data);
  auto block = [&](const uint8_t *b) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t{b[4 * i]} << 24) | (uint32_t{b[4 * i + 1]} << 16) |
             (uint32_t{b[4 * i + 2]} << 8) | uint32_t{b[4 * i + 3]};
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b2 = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + t.k[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b2) ^ (a & c) ^ (b2 & c);
      const uint32_t t2 = S0 + mj;
      hh = g; g = f; f = e; e = d + t1; d = c; c = b2; b2 = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b2; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
  };
  size_t i = 0;
  for (; i + 64 <= n; i += 64) block(p + i);
  uint8_t tail[128] = {};
  const size_t rem = n - i;
  std::memcpy(tail, p + i, rem);
  tail[rem] = 0x80;
  const size_t tl = rem + 1 + 8 <= 64 ? 64 : 128;
  const uint64_t bits = static_cast<uint64_t>(n) * 8;
  for (int k = 0; k < 8; ++k) tail[tl - 1 - k] = static_cast<uint8_t>(bits >> (8 * k));
  block(tail);
  if (tl == 128) block(tail + 64);
  static const char *hex = "0123456789abcdef";
  std::string out(64, '0');
  for (int k = 0; k < 8; ++k)
    for (int j = 0; j < 8; ++j) out[k * 8 + j] = hex[(h[k] >> (28 - 4 * j)) & 15];
  return out;
}

namespace {

// ---- JSON text as Python's json.dumps(separators=(",", ":")) writes it ----

void put_string(std::string &o, const std::string &s) {  // ensure_ascii
  o += '"';
  size_t i = 0;
  while (i < s.size()) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    uint32_t cp = c;
    int len = 1;
    if (c >= 0x80) {  // well-formed UTF-8 (the inputs are JSON text or ASCII names)
      len = c >= 0xF0 ? 4 : (c >= 0xE0 ? 3 : 2);
      cp = c & (0x3F >> (len - 1));
      for (int k = 1; k < len && i + k < s.size(); ++k)
        cp = (cp << 6) | (static_cast<unsigned char>(s[i + k]) & 0x3F);
    }
    i += static_cast<size_t>(len);
    char buf[16];
    switch (cp) {
      case '"': o += "\\\""; continue;
      case '\\': o += "\\\\"; continue;
      case '\n': o += "\\n"; continue;
      case '\r': o += "\\r"; continue;
      case '\t': o += "\\t"; continue;
      case '\b': o += "\\b"; continue;
      case '\f': o += "\\f"; continue;
      default: break;
    }
    if (cp >= 0x20 && cp < 0x7F) {
      o += static_cast<char>(cp);
    } else if (cp < 0x10000) {
      std::snprintf(buf, sizeof buf, "\\u%04x", cp);
      o += buf;
    } else {  // a surrogate pair
      const uint32_t v = cp - 0x10000;
      std::snprintf(buf, sizeof buf, "\\u%04x", 0xD800 + (v >> 10));
      o += buf;
      std::snprintf(buf, sizeof buf, "\\u%04x", 0xDC00 + (v & 0x3FF));
      o += buf;
    }
  }
  o += '"';
}

// repr(float): the shortest digits that round-trip, fixed notation for
// decimal exponents -4..15 (with ".0" on integral values), else d[.ddd]e+XX.
std::string py_float(double x) {
  if (std::isnan(x)) return "NaN";
  if (std::isinf(x)) return x > 0 ? "Infinity" : "-Infinity";
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof buf, x, std::chars_format::scientific);
  std::string sci(buf, r.ptr);
  const size_t epos = sci.find('e');
  std::string mant = sci.substr(0, epos);
  const int exp10 = std::stoi(sci.substr(epos + 1));
  std::string sign;
  if (mant[0] == '-') {
    sign = "-";
    mant.erase(0, 1);
  }
  std::string digits;
  for (char c : mant)
    if (c != '.') digits += c;
  if (exp10 >= -4 && exp10 < 16) {
    std::string s;
    if (exp10 < 0) {
      s = "0." + std::string(static_cast<size_t>(-exp10 - 1), '0') + digits;
    } else if (static_cast<int>(digits.size()) <= exp10 + 1) {
      s = digits + std::string(static_cast<size_t>(exp10 + 1 - static_cast<int>(digits.size())), '0') + ".0";
    } else {
      s = digits.substr(0, static_cast<size_t>(exp10 + 1)) + "." +
          digits.substr(static_cast<size_t>(exp10 + 1));
    }
    return sign + s;
  }
  std::string s = digits.substr(0, 1);
  if (digits.size() > 1) s += "." + digits.substr(1);
  char e[16];
  std::snprintf(e, sizeof e, "e%c%02d", exp10 < 0 ? '-' : '+', std::abs(exp10));
  return sign + s + e;
}

// A JSON number from a parsed config: Python keeps integers integers.
std::string py_number(const Json &v) {
  if (v.kind != Json::Number) throw std::runtime_error("expected a number");
  const bool is_int = v.str.find_first_of(".eE") == std::string::npos;
  return is_int ? v.str : py_float(v.num);
}

// ---- input -----------------------------------------------------------------

std::string read_file(const std::string &path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::ostringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

bool exists(const std::string &path) { return std::ifstream(path).good(); }

struct Tensor {
  std::vector<int64_t> shape;
  std::vector<float> v;
};

float half_to_float(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  float f;
  if (e == 0) f = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) f = m ? NAN : INFINITY;
  else f = std::ldexp(static_cast<float>(m | 1024), static_cast<int>(e) - 25);
  return sign ? -f : f;
}

std::map<std::string, Tensor> read_safetensors(const std::string &raw, const std::string &path) {
  if (raw.size() < 8) throw std::runtime_error(path + ": too short for a safetensors file");
  uint64_t n = 0;
  std::memcpy(&n, raw.data(), 8);
  if (8 + n > raw.size()) throw std::runtime_error(path + ": header length past the file");
  const Json header = Json::parse(raw.substr(8, n));
  const size_t base = 8 + n;
  std::map<std::string, Tensor> out;
  for (const auto &kv : header.obj) {
    if (kv.first == "__metadata__") continue;
    const Json &e = kv.second;
    const std::string dt = e.find("dtype")->str;
    const Json *offs = e.find("data_offsets");
    const uint64_t b0 = static_cast<uint64_t>(offs->arr.at(0).num),
                   b1 = static_cast<uint64_t>(offs->arr.at(1).num);
    if (base + b1 > raw.size() || b1 < b0)
      throw std::runtime_error(path + ": tensor " + kv.first + " lies past the file");
    Tensor t;
    int64_t count = 1;
    for (const Json &d : e.find("shape")->arr) {
      t.shape.push_back(static_cast<int64_t>(d.num));
      count *= t.shape.back();
    }
    const char *p = raw.data() + base + b0;
    const size_t esz = dt == "F32" ? 4 : dt == "F64" ? 8 : (dt == "F16" || dt == "BF16") ? 2 : 0;
    if (!esz)
      throw std::runtime_error(path + ": tensor " + kv.first + " has dtype " + dt +
                               "; F32, F16, BF16 or F64 expected");
    if (static_cast<uint64_t>(count) * esz != b1 - b0)
      throw std::runtime_error(path + ": tensor " + kv.first + " size does not match its shape");
    t.v.resize(static_cast<size_t>(count));
    for (int64_t i = 0; i < count; ++i) {
      if (dt == "F32") {
        std::memcpy(&t.v[i], p + 4 * i, 4);
      } else if (dt == "F64") {
        double d;
        std::memcpy(&d, p + 8 * i, 8);
        t.v[i] = static_cast<float>(d);
      } else {
        uint16_t h;
        std::memcpy(&h, p + 2 * i, 2);
        if (dt == "BF16") {
          const uint32_t u = uint32_t{h} << 16;
          std::memcpy(&t.v[i], &u, 4);
        } else {
          t.v[i] = half_to_float(h);
        }
      }
    }
    out.emplace(kv.first, std::move(t));
  }
  return out;
}

// BertModel names tensors embeddings.* / encoder.*; BertFor* and
// sentence-transformers exports prefix them with `bert.` or `0.auto_model.`.
std::map<std::string, Tensor> strip_prefix(std::map<std::string, Tensor> src) {
  for (const char *pre : {"0.auto_model.", "bert.", "model."}) {
    const std::string pfx(pre);
    bool hit = false;
    for (const auto &kv : src)
      if (kv.first.compare(0, pfx.size() + 11, pfx + "embeddings.") == 0) hit = true;
    if (!hit) continue;
    std::map<std::string, Tensor> out;
    for (auto &kv : src)
      if (kv.first.compare(0, pfx.size(), pfx) == 0) out.emplace(kv.first.substr(pfx.size()), std::move(kv.second));
    return out;
  }
  return src;
}

std::string read_pooling(const std::string &dir) {
  const std::string p = dir + "/1_Pooling/config.json";
  if (!exists(p)) throw std::runtime_error(p + " not found -- cannot determine the pooling mode");
  const Json c = Json::parse(read_file(p));
  std::vector<std::string> modes;
  for (const auto &kv : c.obj)
    if (kv.first.compare(0, 13, "pooling_mode_") == 0 && kv.second.kind == Json::Bool &&
        kv.second.b)
      modes.push_back(kv.first);
  if (modes.size() == 1 && modes[0] == "pooling_mode_cls_token") return "cls";
  if (modes.size() == 1 && modes[0] == "pooling_mode_mean_tokens") return "mean";
  throw std::runtime_error(p + ": cls and mean pooling are implemented; the checkpoint asks for "
                           "something else");
}

uint16_t bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// ---- output -----------------------------------------------------------------

constexpr uint64_t kAlign = 4096;
uint64_t pad_to(uint64_t n) { return (kAlign - n % kAlign) % kAlign; }

struct Writer {
  std::vector<std::string> entries;  // JSON text of each directory entry
  std::vector<std::vector<uint8_t>> blobs;
  uint64_t cursor = 0;

  void add(const std::string &name, std::vector<uint8_t> bytes, const std::string &dtype,
           const std::string &role, const std::vector<int64_t> &shape,
           const std::string &layout_json = "", const std::string &layout_hash = "") {
    std::string e = "{\"name\":";
    put_string(e, name);
    e += ",\"role\":";
    put_string(e, role);
    e += ",\"dtype\":";
    put_string(e, dtype);
    std::string sh = "[";
    for (size_t i = 0; i < shape.size(); ++i) sh += (i ? "," : "") + std::to_string(shape[i]);
    sh += "]";
    e += ",\"logical_shape\":" + sh + ",\"padded_shape\":" + sh;
    e += ",\"offset\":" + std::to_string(cursor) + ",\"nbytes\":" + std::to_string(bytes.size());
    if (!layout_json.empty()) {
      e += ",\"layout\":" + layout_json + ",\"layout_hash\":";
      put_string(e, layout_hash);
    }
    e += "}";
    entries.push_back(std::move(e));
    cursor += bytes.size() + pad_to(bytes.size());
    blobs.push_back(std::move(bytes));
  }

  uint64_t write(const std::string &path, const std::string &config_json) {
    std::string dir = "{\"config\":" + config_json + ",\"tensors\":[";
    for (size_t i = 0; i < entries.size(); ++i) dir += (i ? "," : "") + entries[i];
    dir += "]}";
    const uint64_t json_offset = 64, json_length = dir.size();
    uint64_t data_offset = json_offset + json_length;
    data_offset += pad_to(data_offset);
    uint8_t head[64] = {};
    std::memcpy(head, "NPUE", 4);
    const uint32_t version = 1, arch = 0, flags = 1;  // BERT; the writer's fixed flags word
    std::memcpy(head + 4, &version, 4);
    std::memcpy(head + 8, &arch, 4);
    std::memcpy(head + 12, &flags, 4);
    std::memcpy(head + 16, &json_offset, 8);
    std::memcpy(head + 24, &json_length, 8);
    std::memcpy(head + 32, &data_offset, 8);
    std::memcpy(head + 40, &cursor, 8);
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot create " + path);
    f.write(reinterpret_cast<const char *>(head), 64);
    f.write(dir.data(), static_cast<std::streamsize>(dir.size()));
    const std::string zeros(kAlign, '\0');
    f.write(zeros.data(), static_cast<std::streamsize>(data_offset - json_offset - json_length));
    for (const auto &b : blobs) {
      f.write(reinterpret_cast<const char *>(b.data()), static_cast<std::streamsize>(b.size()));
      f.write(zeros.data(), static_cast<std::streamsize>(pad_to(b.size())));
    }
    if (!f) throw std::runtime_error("write failed: " + path);
    return data_offset + cursor;
  }
};

std::vector<uint8_t> f32_bytes(const float *p, size_t n) {
  std::vector<uint8_t> b(n * 4);
  std::memcpy(b.data(), p, n * 4);
  return b;
}

}  // namespace

uint64_t pack_checkpoint(const std::string &model_dir, const std::string &out_path,
                         const PackOptions &opt) {
  if (opt.layout != "tma_bf16" && opt.layout != "host")
    throw std::runtime_error("layout " + opt.layout + ": tma_bf16 or host");
  if (opt.max_seq <= 0) throw std::runtime_error("max_seq must be positive");
  const bool host = opt.layout == "host";
  const Json cfg = Json::parse(read_file(model_dir + "/config.json"));
  if (const Json *mt = cfg.find("model_type"))
    if (mt->str != "bert")
      throw std::runtime_error("model_type " + mt->str +
                               ": this packer handles BERT encoders (arch bert_abs_gelu_postln)");
  auto num = [&](const char *key) -> const Json & {
    const Json *v = cfg.find(key);
    if (!v || v->kind != Json::Number)
      throw std::runtime_error(std::string("config.json lacks the number ") + key);
    return *v;
  };
  std::string wpath;
  for (const char *n : {"model.safetensors", "pytorch_model.safetensors"})
    if (wpath.empty() && exists(model_dir + "/" + n)) wpath = model_dir + "/" + n;
  if (wpath.empty()) throw std::runtime_error("no model.safetensors in " + model_dir);
  const std::string raw = read_file(wpath);
  const std::string source_sha = sha256_hex(raw.data(), raw.size());
  std::map<std::string, Tensor> src = strip_prefix(read_safetensors(raw, wpath));
  auto T = [&](const std::string &name) -> const Tensor & {
    const auto it = src.find(name);
    if (it == src.end()) throw std::runtime_error(wpath + " lacks tensor " + name);
    return it->second;
  };

  const int64_t L = static_cast<int64_t>(num("num_hidden_layers").num);
  const int64_t heads = static_cast<int64_t>(num("num_attention_heads").num);
  const int64_t H = static_cast<int64_t>(num("hidden_size").num);
  const int64_t F = static_cast<int64_t>(num("intermediate_size").num);
  const int64_t V = static_cast<int64_t>(num("vocab_size").num);
  const int64_t TV = static_cast<int64_t>(num("type_vocab_size").num);
  if (L <= 0 || heads <= 0 || H <= 0 || H % heads || F <= 0 || V <= 0 || TV <= 0)
    throw std::runtime_error("config.json geometry refused");
  const int64_t hd = H / heads;
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
  std::string repo_id = "unknown";
  if (exists(model_dir + "/CHECKPOINT.json"))
    repo_id = Json::parse(read_file(model_dir + "/CHECKPOINT.json")).find("repo_id")->str;

  std::string c = "{\"arch\":\"bert_abs_gelu_postln\",\"source_repo\":";
  put_string(c, repo_id);
  c += ",\"source_sha256\":";
  put_string(c, source_sha);
  c += ",\"num_layers\":" + py_number(num("num_hidden_layers")) +
       ",\"num_heads\":" + py_number(num("num_attention_heads")) +
       ",\"hidden\":" + py_number(num("hidden_size")) + ",\"head_dim\":" + std::to_string(hd) +
       ",\"intermediate\":" + py_number(num("intermediate_size")) +
       ",\"layer_norm_eps\":" + py_number(num("layer_norm_eps")) +
       ",\"vocab_size\":" + py_number(num("vocab_size")) +
       ",\"max_seq_len\":" + std::to_string(opt.max_seq) + ",\"pooling\":";
  put_string(c, read_pooling(model_dir));
  c += std::string(",\"l2_normalize\":true,\"activation\":\"gelu_erf_exact\",\"gemm_layout\":") +
       (host ? "\"host\"" : "\"tma_bf16\"") + ",\"a_dtype\":" + (host ? "\"f32\"" : "\"bf16\"") +
       ",\"fusions\":{\"qkv_fused\":true,\"transposed_to_kn\":true,\"qk_scale_folded_into_q\":" +
       (opt.fold_scale ? "true" : "false") + ",\"gemm_operands_bf16\":" + (host ? "false" : "true") +
       ",\"biases_and_layernorm_fp32\":true,\"position_embeddings_presliced_to\":" +
       std::to_string(opt.max_seq) +
       "},\"not_implemented\":[\"pooler.dense (unused by sentence-transformers)\"]";
  if (!host) c += ",\"tma\":{\"operand_order\":\"NK\",\"k_box\":64,\"swizzle_bytes\":128}";
  c += "}";

  // the layout descriptor of a tma_bf16 operand and its hash (sha256 of the
  // descriptor's canonical JSON: sorted keys, no spaces)
  const std::string layout_json = "{\"kind\":\"dense\",\"order\":\"n,k\",\"dtype\":\"BF16\"}";
  const std::string canonical = "{\"dtype\":\"BF16\",\"kind\":\"dense\",\"order\":\"n,k\"}";
  const std::string layout_hash = sha256_hex(canonical.data(), canonical.size());

  Writer w;
  auto vec = [&](const std::string &name, const Tensor &t, const std::string &role,
                 std::vector<int64_t> shape) {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    if (static_cast<int64_t>(t.v.size()) != n)
      throw std::runtime_error("tensor for " + name + " has " + std::to_string(t.v.size()) +
                               " values, " + std::to_string(n) + " expected");
    w.add(name, f32_bytes(t.v.data(), t.v.size()), "F32", role, shape);
  };
  // GEMM operand from row-major kn [K, N]
  auto gemm = [&](const std::string &name, const std::vector<float> &kn, int64_t K, int64_t N) {
    if (host) {
      w.add(name, f32_bytes(kn.data(), kn.size()), "F32", "gemm_b_host", {K, N});
      return;
    }
    std::vector<uint8_t> b(static_cast<size_t>(N * K) * 2);
    for (int64_t n = 0; n < N; ++n)
      for (int64_t k = 0; k < K; ++k) {
        const uint16_t v = bf16_rne(kn[static_cast<size_t>(k * N + n)]);
        std::memcpy(&b[static_cast<size_t>(n * K + k) * 2], &v, 2);
      }
    w.add(name, std::move(b), "BF16", "gemm_b_tma", {N, K}, layout_json, layout_hash);
  };
  // nn.Linear weight [out, in] -> kn [in, out]
  auto transpose = [](const Tensor &t, int64_t out, int64_t in) {
    if (static_cast<int64_t>(t.v.size()) != out * in)
      throw std::runtime_error("a linear weight has the wrong size");
    std::vector<float> kn(static_cast<size_t>(out * in));
    for (int64_t o = 0; o < out; ++o)
      for (int64_t i = 0; i < in; ++i) kn[static_cast<size_t>(i * out + o)] = t.v[static_cast<size_t>(o * in + i)];
    return kn;
  };

  vec("embeddings.word", T("embeddings.word_embeddings.weight"), "embedding", {V, H});
  {
    const Tensor &pos = T("embeddings.position_embeddings.weight");
    if (static_cast<int64_t>(pos.v.size()) < opt.max_seq * H)
      throw std::runtime_error("the position table has fewer than max_seq rows");
    w.add("embeddings.position", f32_bytes(pos.v.data(), static_cast<size_t>(opt.max_seq * H)),
          "F32", "embedding", {opt.max_seq, H});
  }
  vec("embeddings.token_type", T("embeddings.token_type_embeddings.weight"), "embedding", {TV, H});
  vec("embeddings.ln.weight", T("embeddings.LayerNorm.weight"), "layernorm", {H});
  if (exists(model_dir + "/vocab.txt")) {
    const std::string vb = read_file(model_dir + "/vocab.txt");
    w.add("tokenizer.vocab", std::vector<uint8_t>(vb.begin(), vb.end()), "U8", "tokenizer",
          {static_cast<int64_t>(vb.size())});
  }
  vec("embeddings.ln.bias", T("embeddings.LayerNorm.bias"), "layernorm", {H});
  for (int64_t i = 0; i < L; ++i) {
    const std::string p = "encoder.layer." + std::to_string(i) + ".", o = "layer." + std::to_string(i) + ".";
    const std::string sa = p + "attention.self.";
    // Q | K | V stacked along N, transposed to [H, 3H]
    std::vector<float> qkv(static_cast<size_t>(H * 3 * H)), qkv_b(static_cast<size_t>(3 * H));
    const char *parts[3] = {"query", "key", "value"};
    for (int part = 0; part < 3; ++part) {
      const Tensor &wt = T(sa + parts[part] + ".weight"), &bt = T(sa + parts[part] + ".bias");
      if (static_cast<int64_t>(wt.v.size()) != H * H || static_cast<int64_t>(bt.v.size()) != H)
        throw std::runtime_error(sa + parts[part] + " has the wrong size");
      for (int64_t r = 0; r < H; ++r) {
        for (int64_t k = 0; k < H; ++k)
          qkv[static_cast<size_t>(k * 3 * H + part * H + r)] = wt.v[static_cast<size_t>(r * H + k)];
        qkv_b[static_cast<size_t>(part * H + r)] = bt.v[static_cast<size_t>(r)];
      }
    }
    if (opt.fold_scale) {
      for (int64_t k = 0; k < H; ++k)
        for (int64_t n = 0; n < H; ++n) qkv[static_cast<size_t>(k * 3 * H + n)] *= scale;
      for (int64_t n = 0; n < H; ++n) qkv_b[static_cast<size_t>(n)] *= scale;
    }
    gemm(o + "qkv", qkv, H, 3 * H);
    w.add(o + "qkv.bias", f32_bytes(qkv_b.data(), qkv_b.size()), "F32", "bias", {3 * H});
    const std::string ao = p + "attention.output.";
    gemm(o + "attn_out", transpose(T(ao + "dense.weight"), H, H), H, H);
    vec(o + "attn_out.bias", T(ao + "dense.bias"), "bias", {H});
    vec(o + "ln1.weight", T(ao + "LayerNorm.weight"), "layernorm", {H});
    vec(o + "ln1.bias", T(ao + "LayerNorm.bias"), "layernorm", {H});
    gemm(o + "ffn_up", transpose(T(p + "intermediate.dense.weight"), F, H), H, F);
    vec(o + "ffn_up.bias", T(p + "intermediate.dense.bias"), "bias", {F});
    gemm(o + "ffn_down", transpose(T(p + "output.dense.weight"), H, F), F, H);
    vec(o + "ffn_down.bias", T(p + "output.dense.bias"), "bias", {H});
    vec(o + "ln2.weight", T(p + "output.LayerNorm.weight"), "layernorm", {H});
    vec(o + "ln2.bias", T(p + "output.LayerNorm.bias"), "layernorm", {H});
  }
  return w.write(out_path, c);
}

}  // namespace nebw
