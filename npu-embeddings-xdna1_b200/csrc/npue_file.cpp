// Host-side `.npue` reader; see npue_file.h for the format and provenance.
#include "npue_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace nebw {

namespace {

struct Parser {
  const std::string &s;
  size_t i = 0;

  [[noreturn]] void fail(const char *what) const {
    throw std::runtime_error(std::string("container JSON: ") + what + " at byte " +
                             std::to_string(i));
  }
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool lit(const char *w) {
    const size_t n = std::strlen(w);
    if (s.compare(i, n, w) == 0) {
      i += n;
      return true;
    }
    return false;
  }
  std::string string_body() {
    // at the opening quote
    ++i;
    std::string out;
    while (i < s.size() && s[i] != '"') {
      char c = s[i++];
      if (c == '\\') {
        if (i >= s.size()) fail("unterminated escape");
        const char e = s[i++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            if (i + 4 > s.size()) fail("short \\u escape");
            const unsigned cp = static_cast<unsigned>(std::stoul(s.substr(i, 4), nullptr, 16));
            i += 4;
            // UTF-8 encode the BMP code point (surrogates are kept as-is)
            if (cp < 0x80) {
              out += static_cast<char>(cp);
            } else if (cp < 0x800) {
              out += static_cast<char>(0xC0 | (cp >> 6));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            } else {
              out += static_cast<char>(0xE0 | (cp >> 12));
              out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
              out += static_cast<char>(0x80 | (cp & 0x3F));
            }
            break;
          }
          default: fail("bad escape");
        }
      } else {
        out += c;
      }
    }
    if (i >= s.size()) fail("unterminated string");
    ++i;
    return out;
  }
  Json value(int depth) {
    if (depth > 64) fail("nesting too deep");
    ws();
    if (i >= s.size()) fail("unexpected end");
    Json v;
    const char c = s[i];
    if (c == '{') {
      v.kind = Json::Object;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') {
        ++i;
        return v;
      }
      while (true) {
        ws();
        if (i >= s.size() || s[i] != '"') fail("expected key");
        std::string k = string_body();
        ws();
        if (i >= s.size() || s[i] != ':') fail("expected ':'");
        ++i;
        v.obj.emplace_back(std::move(k), value(depth + 1));
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          ++i;
          return v;
        }
        fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v.kind = Json::Array;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') {
        ++i;
        return v;
      }
      while (true) {
        v.arr.push_back(value(depth + 1));
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          ++i;
          return v;
        }
        fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::String;
      v.str = string_body();
      return v;
    }
    if (lit("true")) {
      v.kind = Json::Bool;
      v.b = true;
      return v;
    }
    if (lit("false")) {
      v.kind = Json::Bool;
      return v;
    }
    if (lit("null")) return v;
    // number
    const size_t start = i;
    while (i < s.size() && (std::strchr("+-0123456789.eE", s[i]) != nullptr)) ++i;
    if (start == i) fail("unexpected character");
    v.kind = Json::Number;
    v.str = s.substr(start, i - start);
    v.num = std::stod(v.str);
    return v;
  }
};

}  // namespace

const Json *Json::find(const std::string &key) const {
  if (kind != Object) return nullptr;
  for (const auto &kv : obj)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

Json Json::parse(const std::string &text) {
  Parser p{text};
  Json v = p.value(0);
  p.ws();
  if (p.i != text.size()) p.fail("trailing bytes");
  return v;
}

NpueFile::NpueFile(const std::string &path) : path_(path) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) throw std::runtime_error("cannot open " + path);
  struct stat st {};
  if (::fstat(fd, &st) < 0) {
    ::close(fd);
    throw std::runtime_error("cannot stat " + path);
  }
  size_ = static_cast<size_t>(st.st_size);
  if (size_ < 64) {
    ::close(fd);
    throw std::runtime_error(path + ": truncated (no 64-byte header)");
  }
  void *m = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) throw std::runtime_error("cannot mmap " + path);
  base_ = static_cast<const uint8_t *>(m);

  auto u32 = [&](size_t off) {
    uint32_t v;
    std::memcpy(&v, base_ + off, 4);
    return v;
  };
  auto u64 = [&](size_t off) {
    uint64_t v;
    std::memcpy(&v, base_ + off, 8);
    return v;
  };
  try {
    if (std::memcmp(base_, "NPUE", 4) != 0) throw std::runtime_error(path + ": not a .npue file");
    if (u32(4) != 1)
      throw std::runtime_error(path + ": version " + std::to_string(u32(4)) + ", expected 1");
    arch_ = u32(8);
    const uint64_t json_off = u64(16), json_len = u64(24), data_off = u64(32), data_len = u64(40);
    if (data_off % 4096 != 0) throw std::runtime_error(path + ": data_offset is not 4096-aligned");
    if (json_off + json_len > size_ || data_off + data_len != size_)
      throw std::runtime_error(path + ": header sizes do not match the file size");
    const Json dir =
        Json::parse(std::string(reinterpret_cast<const char *>(base_ + json_off), json_len));
    const Json *cfg = dir.find("config");
    const Json *tens = dir.find("tensors");
    if (!cfg || cfg->kind != Json::Object || !tens || tens->kind != Json::Array)
      throw std::runtime_error(path + ": directory lacks config/tensors");
    config_ = *cfg;
    for (const Json &e : tens->arr) {
      NpueTensor t;
      const Json *n = e.find("name"), *r = e.find("role"), *d = e.find("dtype"),
                 *sh = e.find("logical_shape"), *o = e.find("offset"), *nb = e.find("nbytes");
      if (!n || !d || !sh || !o || !nb) throw std::runtime_error(path + ": malformed tensor entry");
      t.name = n->str;
      t.role = r ? r->str : "";
      t.dtype = d->str;
      const Json *lh = e.find("layout_hash");
      if (lh) {
        if (lh->kind != Json::String)
          throw std::runtime_error(path + ": tensor " + t.name + " has a non-string layout_hash");
        t.layout_hash = lh->str;
      }
      if (const Json *lj = e.find("layout"); lj && lj->kind == Json::Object) {
        auto str = [&](const char *k) {
          const Json *v = lj->find(k);
          return v && v->kind == Json::String ? v->str : std::string();
        };
        auto num = [&](const char *k) {
          const Json *v = lj->find(k);
          return v && v->kind == Json::Number ? static_cast<int64_t>(v->num) : int64_t{0};
        };
        t.layout_kind = str("kind");
        t.layout_order = str("order");
        t.layout_inner = str("inner");
        t.layout_dtype = str("dtype");
        t.tile_k = num("tile_k");
        t.tile_n = num("tile_n");
        t.mac_s = num("mac_s");
        t.mac_t = num("mac_t");
      }
      if (const Json *ps = e.find("padded_shape"); ps && ps->kind == Json::Array)
        for (const Json &x : ps->arr) t.padded_shape.push_back(static_cast<int64_t>(x.num));
      for (const Json &x : sh->arr) t.shape.push_back(static_cast<int64_t>(x.num));
      t.offset = static_cast<uint64_t>(o->num);
      t.nbytes = static_cast<uint64_t>(nb->num);
      if (t.offset + t.nbytes > data_len)
        throw std::runtime_error(path + ": tensor " + t.name + " runs past the data block");
      t.data = base_ + data_off + t.offset;
      tensors_[t.name] = t;
    }
  } catch (...) {
    ::munmap(const_cast<uint8_t *>(base_), size_);
    base_ = nullptr;
    throw;
  }
}

NpueFile::~NpueFile() {
  if (base_) ::munmap(const_cast<uint8_t *>(base_), size_);
}

const NpueTensor &NpueFile::tensor(const std::string &name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw std::runtime_error(path_ + ": no tensor named " + name);
  return it->second;
}

std::string NpueFile::config_string(const std::string &key) const {
  const Json *v = config_.find(key);
  if (!v) throw std::runtime_error(path_ + ": config key '" + key + "' is missing");
  switch (v->kind) {
    case Json::String:
    case Json::Number: return v->str;
    case Json::Bool: return v->b ? "true" : "false";
    default: throw std::runtime_error(path_ + ": config key '" + key + "' is not a scalar");
  }
}

int64_t NpueFile::config_int(const std::string &key) const {
  return std::stoll(config_string(key));
}

double NpueFile::config_double(const std::string &key) const {
  return std::stod(config_string(key));
}

}  // namespace nebw
