#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace rkt_rt {

namespace {

// Minimal JSON value for the safetensors header: objects, arrays, strings,
// integers (and the literals, which the header never needs but may contain in
// __metadata__ values written by other tools -- they are rejected there, since
// metadata values must be strings).
struct JVal {
  enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
  bool b = false;
  double num = 0;
  int64_t inum = 0;
  bool is_int = false;
  std::string str;
  std::vector<JVal> arr;
  std::vector<std::pair<std::string, JVal>> obj;
};

class Parser {
 public:
  Parser(const char* p, size_t n) : p_(p), end_(p + n) {}

  JVal parse() {
    JVal v = value();
    ws();
    if (p_ != end_) fail("trailing bytes after the header object");
    return v;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void fail(const char* what) { throw std::runtime_error(std::string("safetensors header: ") + what); }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  char peek() {
    ws();
    if (p_ >= end_) fail("unexpected end");
    return *p_;
  }
  void expect(char c) {
    if (peek() != c) fail("unexpected character");
    ++p_;
  }
  static void put_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (end_ - p_ < 4) fail("short \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  std::string string() {
    expect('"');
    std::string s;
    while (true) {
      if (p_ >= end_) fail("unterminated string");
      const char c = *p_++;
      if (c == '"') break;
      if (c != '\\') {
        s += c;
        continue;
      }
      if (p_ >= end_) fail("bad escape");
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
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
            if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') fail("lone surrogate");
            p_ += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(s, cp);
          break;
        }
        default: fail("bad escape");
      }
    }
    return s;
  }
  JVal number() {
    JVal v;
    v.kind = JVal::Num;
    const char* s = p_;
    bool is_int = true;
    if (p_ < end_ && *p_ == '-') ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '+' ||
                         *p_ == '-')) {
      if (*p_ == '.' || *p_ == 'e' || *p_ == 'E') is_int = false;
      ++p_;
    }
    std::string tok(s, p_);
    if (tok.empty() || tok == "-") fail("bad number");
    v.is_int = is_int;
    if (is_int) {
      errno = 0;
      char* e = nullptr;
      v.inum = strtoll(tok.c_str(), &e, 10);
      if (errno || *e) fail("integer out of range");
      v.num = (double)v.inum;
    } else {
      v.num = strtod(tok.c_str(), nullptr);
    }
    return v;
  }
  JVal value() {
    const char c = peek();
    JVal v;
    if (c == '{') {
      ++p_;
      v.kind = JVal::Obj;
      if (peek() == '}') {
        ++p_;
        return v;
      }
      while (true) {
        std::string k = string();
        expect(':');
        v.obj.emplace_back(std::move(k), value());
        const char d = peek();
        ++p_;
        if (d == '}') break;
        if (d != ',') fail("expected , or }");
      }
    } else if (c == '[') {
      ++p_;
      v.kind = JVal::Arr;
      if (peek() == ']') {
        ++p_;
        return v;
      }
      while (true) {
        v.arr.push_back(value());
        const char d = peek();
        ++p_;
        if (d == ']') break;
        if (d != ',') fail("expected , or ]");
      }
    } else if (c == '"') {
      v.kind = JVal::Str;
      v.str = string();
    } else if (c == 't' || c == 'f' || c == 'n') {
      const char* lit = c == 't' ? "true" : (c == 'f' ? "false" : "null");
      const size_t n = strlen(lit);
      if ((size_t)(end_ - p_) < n || strncmp(p_, lit, n)) fail("bad literal");
      p_ += n;
      v.kind = c == 'n' ? JVal::Null : JVal::Bool;
      v.b = c == 't';
    } else {
      v = number();
    }
    return v;
  }
};

const JVal* field(const JVal& o, const char* k) {
  for (auto& kv : o.obj)
    if (kv.first == k) return &kv.second;
  return nullptr;
}

}  // namespace

int dtype_itemsize(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "F8_E4M3" || d == "F8_E5M2" || d == "I8" || d == "U8" || d == "BOOL") return 1;
  return 0;
}

SafetensorsFile::SafetensorsFile(const std::string& path) : path_(path) {
  fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd_ < 0) throw std::runtime_error("safetensors: cannot open " + path);
  struct stat st {};
  if (fstat(fd_, &st) != 0) {
    ::close(fd_);
    throw std::runtime_error("safetensors: cannot stat " + path);
  }
  size_ = (uint64_t)st.st_size;
  auto bail = [&](const std::string& why) {
    if (map_) munmap(map_, size_);
    ::close(fd_);
    map_ = nullptr;
    fd_ = -1;
    throw std::runtime_error("safetensors: " + path + ": " + why);
  };
  if (size_ < 8) bail("file shorter than the 8-byte header length");
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (m == MAP_FAILED) bail("mmap failed");
  map_ = static_cast<uint8_t*>(m);
  uint64_t n = 0;
  for (int i = 7; i >= 0; --i) n = (n << 8) | map_[i];  // little-endian
  if (n > size_ - 8 || n > (100u << 20)) bail("header length out of range");
  data_off_ = 8 + n;
  JVal root;
  try {
    root = Parser(reinterpret_cast<const char*>(map_ + 8), n).parse();
  } catch (const std::exception& e) {
    bail(e.what());
  }
  if (root.kind != JVal::Obj) bail("header is not an object");
  const uint64_t data_size = size_ - data_off_;
  std::vector<std::pair<uint64_t, uint64_t>> ranges;
  for (auto& kv : root.obj) {
    if (kv.first == "__metadata__") {
      if (kv.second.kind != JVal::Obj) bail("__metadata__ is not an object");
      for (auto& m2 : kv.second.obj) {
        if (m2.second.kind != JVal::Str) bail("__metadata__ values must be strings");
        meta_[m2.first] = m2.second.str;
      }
      continue;
    }
    const JVal& t = kv.second;
    if (t.kind != JVal::Obj) bail("entry " + kv.first + " is not an object");
    const JVal* dt = field(t, "dtype");
    const JVal* sh = field(t, "shape");
    const JVal* off = field(t, "data_offsets");
    if (!dt || dt->kind != JVal::Str || !sh || sh->kind != JVal::Arr || !off || off->kind != JVal::Arr ||
        off->arr.size() != 2)
      bail("entry " + kv.first + " lacks dtype/shape/data_offsets");
    TensorInfo ti;
    ti.dtype = dt->str;
    const int isz = dtype_itemsize(ti.dtype);
    if (!isz) bail("entry " + kv.first + " has unknown dtype " + ti.dtype);
    uint64_t numel = 1;
    for (auto& d : sh->arr) {
      if (d.kind != JVal::Num || !d.is_int || d.inum < 0) bail("entry " + kv.first + " has a bad shape");
      ti.shape.push_back(d.inum);
      numel *= (uint64_t)d.inum;
    }
    for (auto& o : off->arr)
      if (o.kind != JVal::Num || !o.is_int || o.inum < 0) bail("entry " + kv.first + " has bad offsets");
    ti.begin = (uint64_t)off->arr[0].inum;
    ti.end = (uint64_t)off->arr[1].inum;
    if (ti.end < ti.begin || ti.end > data_size) bail("entry " + kv.first + " lies outside the file");
    if (ti.end - ti.begin != numel * (uint64_t)isz) bail("entry " + kv.first + " size != prod(shape) * itemsize");
    if (tensors_.count(kv.first)) bail("duplicate entry " + kv.first);
    if (ti.end > ti.begin) ranges.emplace_back(ti.begin, ti.end);
    tensors_[kv.first] = std::move(ti);
  }
  std::sort(ranges.begin(), ranges.end());
  for (size_t i = 1; i < ranges.size(); ++i)
    if (ranges[i].first < ranges[i - 1].second) bail("tensor byte ranges overlap");
}

SafetensorsFile::~SafetensorsFile() {
  if (map_) munmap(map_, size_);
  if (fd_ >= 0) ::close(fd_);
}

std::vector<std::string> SafetensorsFile::keys() const {
  std::vector<std::string> k;
  k.reserve(tensors_.size());
  for (auto& kv : tensors_) k.push_back(kv.first);
  return k;
}

const TensorInfo& SafetensorsFile::info(const std::string& name) const {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) throw std::out_of_range("safetensors: no tensor " + name + " in " + path_);
  return it->second;
}

const uint8_t* SafetensorsFile::data(const std::string& name) const {
  const TensorInfo& t = info(name);
  return map_ + data_off_ + t.begin;
}

}  // namespace rkt_rt
