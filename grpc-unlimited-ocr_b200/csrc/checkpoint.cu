// Safetensors shards and the shard index, memory-mapped read-only (host code).
//
// The checks and their order are the reference's readers':
//   parse_safetensors_header (src/weights/safetensors.cpp:69-124) — a JSON
//     object header, "__metadata__" skipped, each entry with a known dtype,
//     non-negative integer dims, two unsigned data offsets inside the data
//     section and a byte count equal to shape x dtype size, entries checked in
//     name order, then the extents sorted by start must tile the data section;
//   SafetensorsFile (:126-163) — at least 8 bytes, a little-endian header
//     length of at most 100 MiB that fits the file;
//   ShardedWeights::open (src/weights/sharded_weights.cpp:12-61) — a
//     weight_map object of plain file names, every indexed tensor in the shard
//     the index names, no shard holding a tensor the index does not list.
// The JSON reader below is a small strict RFC 8259 parser of our own (objects
// keep the last of duplicate keys and iterate in key order).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "checkpoint.h"
#include "moe_kernels.h"

using namespace uocr_b200;

namespace {

constexpr uint64_t kMaxHeaderBytes = 100ull * 1024 * 1024;
constexpr int kMaxJsonDepth = 128;

// ---- JSON ----------------------------------------------------------------
struct Json {
  enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
  bool boolean = false;
  bool is_uint = false;  // an integer literal >= 0 that fits uint64
  bool is_int = false;   // an integer literal that fits int64
  uint64_t u = 0;
  int64_t i = 0;
  std::string text;  // the string, or a number's literal
  std::vector<Json> items;
  std::map<std::string, Json> fields;
};

class JsonParser {
 public:
  JsonParser(const char* p, size_t n) : p_(p), end_(p + n) {}

  bool parse(Json& out) {
    skip_ws();
    if (!value(out, 0)) return false;
    skip_ws();
    return p_ == end_;
  }

 private:
  void skip_ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool literal(const char* word) {
    const size_t n = std::strlen(word);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void put_utf8(std::string& s, uint32_t c) {
    if (c < 0x80) {
      s += static_cast<char>(c);
    } else if (c < 0x800) {
      s += static_cast<char>(0xC0 | (c >> 6));
      s += static_cast<char>(0x80 | (c & 0x3F));
    } else if (c < 0x10000) {
      s += static_cast<char>(0xE0 | (c >> 12));
      s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      s += static_cast<char>(0x80 | (c & 0x3F));
    } else {
      s += static_cast<char>(0xF0 | (c >> 18));
      s += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
      s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
      s += static_cast<char>(0x80 | (c & 0x3F));
    }
  }
  bool hex4(uint32_t& v) {
    if (end_ - p_ < 4) return false;
    v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool string(std::string& s) {
    if (p_ >= end_ || *p_ != '"') return false;
    ++p_;
    while (p_ < end_) {
      const unsigned char c = static_cast<unsigned char>(*p_++);
      if (c == '"') return true;
      if (c < 0x20) return false;
      if (c != '\\') {
        s += static_cast<char>(c);
        continue;
      }
      if (p_ >= end_) return false;
      const char e = *p_++;
      switch (e) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          uint32_t c1 = 0;
          if (!hex4(c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // high surrogate: a low one must follow
            uint32_t c2 = 0;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return false;
            p_ += 2;
            if (!hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000) return false;
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          } else if (c1 >= 0xDC00 && c1 < 0xE000) {
            return false;
          }
          put_utf8(s, c1);
          break;
        }
        default:
          return false;
      }
    }
    return false;
  }
  bool number(Json& out) {
    const char* start = p_;
    bool neg = false, integral = true;
    if (p_ < end_ && *p_ == '-') {
      neg = true;
      ++p_;
    }
    if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
    if (*p_ == '0') {
      ++p_;
    } else {
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    const char* int_end = p_;
    if (p_ < end_ && *p_ == '.') {
      integral = false;
      ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
      integral = false;
      ++p_;
      if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
      if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
      while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
    }
    out.kind = Json::kNumber;
    out.text.assign(start, p_);
    if (integral) {
      uint64_t mag = 0;
      bool fits = true;
      for (const char* q = start + (neg ? 1 : 0); q < int_end; ++q) {
        const uint64_t d = static_cast<uint64_t>(*q - '0');
        if (mag > (UINT64_MAX - d) / 10) {
          fits = false;
          break;
        }
        mag = mag * 10 + d;
      }
      if (fits && !neg) {
        out.is_uint = true;
        out.u = mag;
        if (mag <= static_cast<uint64_t>(INT64_MAX)) {
          out.is_int = true;
          out.i = static_cast<int64_t>(mag);
        }
      } else if (fits && neg && mag <= static_cast<uint64_t>(INT64_MAX) + 1) {
        out.is_int = true;
        out.i = mag == static_cast<uint64_t>(INT64_MAX) + 1 ? INT64_MIN : -static_cast<int64_t>(mag);
      }
    }
    return true;
  }
  bool value(Json& out, int depth) {
    if (depth > kMaxJsonDepth || p_ >= end_) return false;
    const char c = *p_;
    if (c == '{') {
      ++p_;
      out.kind = Json::kObject;
      skip_ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        skip_ws();
        std::string key;
        if (!string(key)) return false;
        skip_ws();
        if (p_ >= end_ || *p_ != ':') return false;
        ++p_;
        skip_ws();
        Json v;
        if (!value(v, depth + 1)) return false;
        out.fields[key] = std::move(v);
        skip_ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++p_;
      out.kind = Json::kArray;
      skip_ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        skip_ws();
        Json v;
        if (!value(v, depth + 1)) return false;
        out.items.push_back(std::move(v));
        skip_ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return false;
      }
    }
    if (c == '"') {
      out.kind = Json::kString;
      return string(out.text);
    }
    if (c == 't' || c == 'f') {
      out.kind = Json::kBool;
      out.boolean = c == 't';
      return literal(c == 't' ? "true" : "false");
    }
    if (c == 'n') {
      out.kind = Json::kNull;
      return literal("null");
    }
    return number(out);
  }

  const char* p_;
  const char* end_;
};

std::string dump(const Json& v) {
  switch (v.kind) {
    case Json::kNull: return "null";
    case Json::kBool: return v.boolean ? "true" : "false";
    case Json::kNumber: return v.text;
    case Json::kString: return "\"" + v.text + "\"";
    case Json::kArray: return "[...]";
    default: return "{...}";
  }
}

// ---- dtypes ----------------------------------------------------------------
struct DtypeRow {
  const char* name;
  int dtype;
  uint64_t size;
};
constexpr DtypeRow kDtypes[] = {{"BF16", UOCR_DTYPE_BF16, 2}, {"F16", UOCR_DTYPE_F16, 2}, {"F32", UOCR_DTYPE_F32, 4},
                                {"I64", UOCR_DTYPE_I64, 8},   {"I32", UOCR_DTYPE_I32, 4}, {"U8", UOCR_DTYPE_U8, 1}};

const DtypeRow* find_dtype(const std::string& name) {
  for (const auto& r : kDtypes)
    if (name == r.name) return &r;
  return nullptr;
}

std::string str(uint64_t v) { return std::to_string(v); }

// ---- one shard ---------------------------------------------------------------
struct Shard {
  std::string path;
  const uint8_t* map = nullptr;
  size_t size = 0;
  std::map<std::string, CkTensor> tensors;
  ~Shard() {
    if (map != nullptr) munmap(const_cast<uint8_t*>(map), size);
  }
};

// The header's tensors against a data section of data_size bytes at data;
// empty string on success, else the first problem.
std::string parse_header(const char* text, size_t len, const uint8_t* data, uint64_t data_size,
                         std::map<std::string, CkTensor>& out) {
  Json header;
  if (!JsonParser(text, len).parse(header) || header.kind != Json::kObject) return "header is not a JSON object";
  struct Extent {
    uint64_t begin, end;
    const std::string* name;
  };
  std::vector<Extent> extents;
  for (const auto& [name, entry] : header.fields) {
    if (name == "__metadata__") continue;
    if (entry.kind != Json::kObject || !entry.fields.count("dtype") || !entry.fields.count("shape") ||
        !entry.fields.count("data_offsets"))
      return "tensor " + name + ": entry lacks dtype, shape or data_offsets";
    const Json& dt = entry.fields.at("dtype");
    const DtypeRow* row = dt.kind == Json::kString ? find_dtype(dt.text) : nullptr;
    if (row == nullptr) return "tensor " + name + ": unsupported dtype " + dump(dt);
    const Json& sh = entry.fields.at("shape");
    if (sh.kind != Json::kArray) return "tensor " + name + ": shape is not an array";
    std::vector<int64_t> shape;
    for (const Json& d : sh.items) {
      if (!d.is_int || d.i < 0) return "tensor " + name + ": shape holds a non-integer or negative dim";
      shape.push_back(d.i);
    }
    const Json& off = entry.fields.at("data_offsets");
    if (off.kind != Json::kArray || off.items.size() != 2 || !off.items[0].is_uint || !off.items[1].is_uint)
      return "tensor " + name + ": data_offsets is not two unsigned integers";
    const uint64_t begin = off.items[0].u, end = off.items[1].u;
    if (begin > end || end > data_size)
      return "tensor " + name + ": data_offsets [" + str(begin) + ", " + str(end) + ") outside a " + str(data_size) +
             "-byte data section";
    uint64_t need = row->size;
    for (const int64_t d : shape) {
      const uint64_t ud = static_cast<uint64_t>(d);
      if (ud != 0 && need > UINT64_MAX / ud) return "tensor " + name + ": shape overflows";
      need *= ud;
    }
    if (end - begin != need)
      return "tensor " + name + ": " + str(end - begin) + " bytes stored, shape and dtype need " + str(need);
    auto it = out.emplace(name, CkTensor{row->dtype, std::move(shape), data + begin, end - begin}).first;
    extents.push_back({begin, end, &it->first});
  }
  std::sort(extents.begin(), extents.end(), [](const Extent& a, const Extent& b) { return a.begin < b.begin; });
  uint64_t cursor = 0;
  for (const auto& e : extents) {
    if (e.begin != cursor)
      return "tensor " + *e.name + ": starts at " + str(e.begin) + " but the previous tensor ends at " + str(cursor);
    cursor = e.end;
  }
  if (cursor != data_size) return "tensors end at " + str(cursor) + " but the data section is " + str(data_size) + " bytes";
  return {};
}

int open_shard(const std::string& path, std::unique_ptr<Shard>& out) {
  auto bad = [&](const std::string& what) { return set_last_error(UOCR_ERR_INVALID_ARGUMENT, path + ": " + what); };
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return bad(std::string("cannot open: ") + std::strerror(errno));
  struct stat st {};
  if (::fstat(fd, &st) != 0) {
    const int e = errno;
    ::close(fd);
    return bad(std::string("cannot stat: ") + std::strerror(e));
  }
  const size_t size = static_cast<size_t>(st.st_size);
  if (size < 8) {
    ::close(fd);
    return bad(str(size) + " bytes is too short for a safetensors file");
  }
  void* m = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  const int map_err = errno;
  ::close(fd);
  if (m == MAP_FAILED) return bad(std::string("mmap failed: ") + std::strerror(map_err));
  auto s = std::make_unique<Shard>();
  s->path = path;
  s->map = static_cast<const uint8_t*>(m);
  s->size = size;
  uint64_t hlen = 0;
  std::memcpy(&hlen, s->map, 8);  // little-endian on every target
  if (hlen > kMaxHeaderBytes || hlen > size - 8) return bad("header length " + str(hlen) + " does not fit the file");
  const std::string err = parse_header(reinterpret_cast<const char*>(s->map + 8), static_cast<size_t>(hlen),
                                       s->map + 8 + hlen, size - 8 - hlen, s->tensors);
  if (!err.empty()) return bad(err);
  out = std::move(s);
  return UOCR_OK;
}

bool ends_with(const std::string& s, const char* suffix) {
  const size_t n = std::strlen(suffix);
  return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

}  // namespace

struct uocr_checkpoint {
  std::vector<std::unique_ptr<Shard>> shards;
  std::map<std::string, const CkTensor*> where;
};

namespace uocr_b200 {

const CkTensor* checkpoint_find(const uocr_checkpoint* c, const std::string& name) {
  const auto it = c->where.find(name);
  return it == c->where.end() ? nullptr : it->second;
}

const char* dtype_name(int dtype) {
  for (const auto& r : kDtypes)
    if (r.dtype == dtype) return r.name;
  return "?";
}

}  // namespace uocr_b200

namespace {

int open_index(const std::string& index_path, uocr_checkpoint& ck) {
  auto bad = [&](const std::string& what) {
    return set_last_error(UOCR_ERR_INVALID_ARGUMENT, index_path + ": " + what);
  };
  std::ifstream in(index_path, std::ios::binary);
  if (!in) return bad("cannot open the shard index");
  const std::string text((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  Json index;
  const bool parsed = JsonParser(text.data(), text.size()).parse(index);
  if (!parsed || index.kind != Json::kObject || !index.fields.count("weight_map") ||
      index.fields.at("weight_map").kind != Json::kObject)
    return bad("not a shard index (no weight_map object)");
  const size_t slash = index_path.find_last_of('/');
  const std::string dir = slash == std::string::npos ? std::string() : index_path.substr(0, slash + 1);
  std::map<std::string, size_t> slot;  // shard file -> index into ck.shards
  std::map<std::string, std::string> expected;
  for (const auto& [name, shard] : index.fields.at("weight_map").fields) {
    if (shard.kind != Json::kString) return bad("weight_map[" + name + "] is not a file name");
    const std::string& file = shard.text;
    if (file.find('/') != std::string::npos || file == ".." || file.empty())
      return bad("shard name " + file + " is not a plain file name");
    expected.emplace(name, file);
    if (!slot.count(file)) {
      std::unique_ptr<Shard> s;
      const int rc = open_shard(dir + file, s);
      if (rc != UOCR_OK) return rc;
      slot.emplace(file, ck.shards.size());
      ck.shards.push_back(std::move(s));
    }
  }
  for (const auto& [file, k] : slot) {
    for (const auto& [name, t] : ck.shards[k]->tensors) {
      const auto e = expected.find(name);
      if (e == expected.end())
        return set_last_error(UOCR_ERR_INVALID_ARGUMENT, file + ": holds " + name + ", which the index does not list");
      if (e->second != file)
        return set_last_error(UOCR_ERR_INVALID_ARGUMENT,
                              file + ": holds " + name + ", which the index places in " + e->second);
      ck.where.emplace(name, &t);
    }
  }
  for (const auto& [name, file] : expected)
    if (!ck.where.count(name))
      return set_last_error(UOCR_ERR_INVALID_ARGUMENT,
                            file + ": the index places " + name + " here but the shard lacks it");
  return UOCR_OK;
}

}  // namespace

int uocr_checkpoint_open(const char* path, uocr_checkpoint** out) {
  if (path == nullptr || out == nullptr) return set_last_error(UOCR_ERR_INVALID_ARGUMENT, "checkpoint_open: null argument");
  *out = nullptr;
  auto ck = std::make_unique<uocr_checkpoint>();
  const std::string p(path);
  int rc;
  if (ends_with(p, ".safetensors")) {
    std::unique_ptr<Shard> s;
    rc = open_shard(p, s);
    if (rc == UOCR_OK) {
      for (const auto& [name, t] : s->tensors) ck->where.emplace(name, &t);
      ck->shards.push_back(std::move(s));
    }
  } else {
    rc = open_index(p, *ck);
  }
  if (rc != UOCR_OK) return rc;
  *out = ck.release();
  return UOCR_OK;
}

int uocr_checkpoint_close(uocr_checkpoint* ckpt) {
  delete ckpt;
  return UOCR_OK;
}

int uocr_checkpoint_count(const uocr_checkpoint* ckpt, int64_t* tensors) {
  if (ckpt == nullptr || tensors == nullptr)
    return set_last_error(UOCR_ERR_INVALID_ARGUMENT, "checkpoint_count: null argument");
  *tensors = static_cast<int64_t>(ckpt->where.size());
  return UOCR_OK;
}

int uocr_checkpoint_tensor(const uocr_checkpoint* ckpt, const char* name, uocr_tensor_view* out) {
  if (ckpt == nullptr || name == nullptr || out == nullptr)
    return set_last_error(UOCR_ERR_INVALID_ARGUMENT, "checkpoint_tensor: null argument");
  const CkTensor* t = checkpoint_find(ckpt, name);
  if (t == nullptr) return set_last_error(UOCR_ERR_INVALID_ARGUMENT, std::string("no tensor named ") + name);
  if (t->shape.size() > UOCR_MAX_TENSOR_RANK)
    return set_last_error(UOCR_ERR_UNSUPPORTED, std::string("checkpoint_tensor: ") + name + " has rank above 8");
  *out = uocr_tensor_view{};
  out->dtype = t->dtype;
  out->rank = static_cast<int32_t>(t->shape.size());
  for (size_t k = 0; k < t->shape.size(); ++k) out->shape[k] = t->shape[k];
  out->data = t->data;
  out->bytes = static_cast<int64_t>(t->bytes);
  return UOCR_OK;
}
