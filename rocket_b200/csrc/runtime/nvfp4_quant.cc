#include "nvfp4_quant.h"

#include <sys/stat.h>

#include <algorithm>
#include <cfenv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <thread>

#include "prefix_store.h"
#include "safetensors.h"

namespace rkt_rt {

// ------------------------------------------------------------------ scalar codes
uint8_t e4m3_from_float(float v) {
  // e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa bits; no infinities, max 448 (0x7e).
  // Subnormals m * 2^-9 (m = 0..7) and the first normal 2^-6 (0x08) are contiguous
  // in the bit pattern, so both ranges round with one nearbyint.
  uint8_t sign = std::signbit(v) ? 0x80 : 0;
  float a = std::fabs(v);
  if (!(a == a)) return 0x7f;  // NaN
  if (a >= 448.f) return sign | 0x7e;
  if (a < 0.015625f) return sign | (uint8_t)std::nearbyint(a * 512.f);
  int e;
  std::frexp(a, &e);            // a = m * 2^e, m in [0.5, 1)
  const int E = e - 1;          // a in [2^E, 2^(E+1)), E in [-6, 8]
  const float mant = std::ldexp(a, -E) - 1.f;  // exact
  const int q = (int)std::nearbyint(mant * 8.f);  // 0..8; 8 carries into the exponent
  return sign | (uint8_t)(((E + 7) << 3) + q);
}

float e4m3_to_float(uint8_t b) {
  const int ex = (b >> 3) & 15, m = b & 7;
  float v;
  if ((b & 0x7f) == 0x7f) return NAN;
  if (ex == 0) v = std::ldexp((float)m, -9);
  else v = std::ldexp(1.f + m / 8.f, ex - 7);
  return (b & 0x80) ? -v : v;
}

uint8_t e2m1_code(float q) {
  // magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6; at a midpoint the even code wins
  const float a = std::fabs(q);
  uint8_t c = 0;
  if (a > 0.25f) c = 1;
  if (a >= 0.75f) c = 2;
  if (a > 1.25f) c = 3;
  if (a >= 1.75f) c = 4;
  if (a > 2.5f) c = 5;
  if (a >= 3.5f) c = 6;
  if (a > 5.f) c = 7;
  if (q < 0 && c) c |= 8;
  return c;
}

float e2m1_value(uint8_t code) {
  static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = mag[code & 7];
  return (code & 8) ? -v : v;
}

float to_float(const void* src, SrcType t, size_t i) {
  switch (t) {
    case SrcType::F32: return static_cast<const float*>(src)[i];
    case SrcType::BF16: {
      uint32_t u = (uint32_t)static_cast<const uint16_t*>(src)[i] << 16;
      float f;
      memcpy(&f, &u, 4);
      return f;
    }
    case SrcType::F16: {
      const uint16_t h = static_cast<const uint16_t*>(src)[i];
      const int ex = (h >> 10) & 31, m = h & 1023;
      float v;
      if (ex == 0) v = std::ldexp((float)m, -24);
      else if (ex == 31) v = m ? NAN : INFINITY;
      else v = std::ldexp(1.f + m / 1024.f, ex - 15);
      return (h & 0x8000) ? -v : v;
    }
  }
  return 0.f;
}

namespace {

template <class F>
void parallel_rows(int64_t rows, int threads, F&& f) {
  if (threads <= 0) threads = (int)std::max(1u, std::thread::hardware_concurrency());
  threads = (int)std::min<int64_t>(threads, std::max<int64_t>(1, rows));
  if (threads == 1) {
    f(0, rows);
    return;
  }
  std::vector<std::thread> th;
  const int64_t per = (rows + threads - 1) / threads;
  for (int i = 0; i < threads; ++i) {
    const int64_t a = i * per, b = std::min(rows, a + per);
    if (a >= b) break;
    th.emplace_back([&f, a, b] { f(a, b); });
  }
  for (auto& x : th) x.join();
}

struct RoundNearest {  // nearbyint must round half to even
  int old;
  RoundNearest() : old(std::fegetround()) { std::fesetround(FE_TONEAREST); }
  ~RoundNearest() { std::fesetround(old); }
};

}  // namespace

float tensor_amax(const void* src, SrcType t, size_t n, int threads) {
  std::vector<float> part(std::max(1, threads <= 0 ? (int)std::thread::hardware_concurrency() : threads) + 1, 0.f);
  const int64_t nt = (int64_t)part.size() - 1;
  std::vector<std::thread> th;
  const int64_t per = ((int64_t)n + nt - 1) / nt;
  for (int64_t i = 0; i < nt; ++i) {
    th.emplace_back([&, i] {
      const int64_t a = i * per, b = std::min<int64_t>((int64_t)n, a + per);
      float m = 0.f;
      for (int64_t j = a; j < b; ++j) m = std::max(m, std::fabs(to_float(src, t, (size_t)j)));
      part[i] = m;
    });
  }
  for (auto& x : th) x.join();
  return *std::max_element(part.begin(), part.end());
}

float quantize_nvfp4(const void* src, SrcType t, int64_t rows, int64_t cols, float g, uint8_t* packed,
                     uint8_t* sf, int threads) {
  if (cols % 16) throw std::invalid_argument("quantize_nvfp4: cols must be a multiple of 16");
  if (!(g > 0.f)) {
    const float amax = tensor_amax(src, t, (size_t)(rows * cols), threads);
    g = amax > 0.f ? (float)((double)amax / (448.0 * 6.0)) : 1.f;
  }
  const int64_t nb = cols / 16;
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    RoundNearest rn;
    float x[16];
    for (int64_t r = r0; r < r1; ++r) {
      for (int64_t b = 0; b < nb; ++b) {
        const size_t base = (size_t)(r * cols + b * 16);
        float bamax = 0.f;
        for (int i = 0; i < 16; ++i) {
          x[i] = to_float(src, t, base + i);
          bamax = std::max(bamax, std::fabs(x[i]));
        }
        const float s_req = bamax / 6.0f / g;
        const uint8_t sb = e4m3_from_float(std::min(s_req, 448.f));
        sf[r * nb + b] = sb;
        const float denom = e4m3_to_float(sb) * g;
        uint8_t* out = packed + (size_t)(r * cols / 2 + b * 8);
        for (int i = 0; i < 16; i += 2) {
          const uint8_t lo = denom > 0.f ? e2m1_code(x[i] / denom) : 0;
          const uint8_t hi = denom > 0.f ? e2m1_code(x[i + 1] / denom) : 0;
          out[i / 2] = (uint8_t)(lo | (hi << 4));
        }
      }
    }
  });
  return g;
}

void quantize_fp8_rows(const void* src, SrcType t, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                       int threads) {
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    RoundNearest rn;
    for (int64_t r = r0; r < r1; ++r) {
      float amax = 0.f;
      for (int64_t c = 0; c < cols; ++c) amax = std::max(amax, std::fabs(to_float(src, t, (size_t)(r * cols + c))));
      const float s = amax > 0.f ? amax / 448.0f : 1.f;
      scale[r] = s;
      for (int64_t c = 0; c < cols; ++c) {
        const float v = to_float(src, t, (size_t)(r * cols + c)) / s;
        q[r * cols + c] = e4m3_from_float(std::max(-448.f, std::min(448.f, v)));
      }
    }
  });
}

size_t sf_swizzled_bytes(int64_t rows, int64_t k_sf) {
  return (size_t)((rows + 127) / 128) * (size_t)((k_sf + 3) / 4) * 512;
}

void swizzle_sf(const uint8_t* sf_linear, int64_t rows, int64_t k_sf, uint8_t* out) {
  const int64_t k_tiles = (k_sf + 3) / 4;
  memset(out, 0, sf_swizzled_bytes(rows, k_sf));
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t rr = r % 128;
    for (int64_t s = 0; s < k_sf; ++s) {
      const int64_t atom = (r / 128) * k_tiles + s / 4;
      out[atom * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (s % 4)] = sf_linear[r * k_sf + s];
    }
  }
}

// ------------------------------------------------------------------ writer
namespace {

std::string json_str(const std::string& s) {
  std::string o = "\"";
  for (unsigned char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += (char)c;
    } else if (c < 0x20) {
      char b[8];
      snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else {
      o += (char)c;
    }
  }
  return o + "\"";
}

std::string hex(const Digest256& d) {
  char b[65];
  for (int i = 0; i < 4; ++i) snprintf(b + 16 * i, 17, "%016llx", (unsigned long long)d.w[i]);
  return std::string(b, 64);
}

}  // namespace

void write_safetensors(const std::string& path, std::vector<OutTensor> ts,
                       const std::map<std::string, std::string>& meta) {
  std::sort(ts.begin(), ts.end(), [](const OutTensor& a, const OutTensor& b) { return a.name < b.name; });
  std::string h = "{";
  bool first = true;
  if (!meta.empty()) {
    h += "\"__metadata__\":{";
    bool f2 = true;
    for (auto& kv : meta) {
      if (!f2) h += ",";
      h += json_str(kv.first) + ":" + json_str(kv.second);
      f2 = false;
    }
    h += "}";
    first = false;
  }
  uint64_t off = 0;
  for (auto& t : ts) {
    if (!first) h += ",";
    first = false;
    h += json_str(t.name) + ":{\"dtype\":" + json_str(t.dtype) + ",\"shape\":[";
    for (size_t i = 0; i < t.shape.size(); ++i) h += (i ? "," : "") + std::to_string(t.shape[i]);
    h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + t.nbytes) + "]}";
    off += t.nbytes;
  }
  h += "}";
  while (h.size() % 8) h += ' ';
  const std::string tmp = path + ".tmp";
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot write " + tmp);
  const uint64_t hl = h.size();
  bool ok = fwrite(&hl, 8, 1, f) == 1 && fwrite(h.data(), 1, h.size(), f) == h.size();
  for (auto& t : ts)
    if (ok && t.nbytes) ok = fwrite(t.data, 1, t.nbytes, f) == t.nbytes;
  ok = (fclose(f) == 0) && ok;
  if (!ok || rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("write failed: " + path);
}

std::string file_digest_hex(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("cannot read " + path);
  std::vector<uint8_t> buf((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  return hex(digest256({{buf.data(), buf.size()}}));
}

std::vector<std::string> verify_checksums(const std::string& dir) {
  std::ifstream in(dir + "/checksums.txt");
  if (!in) throw std::runtime_error("no checksums.txt in " + dir);
  std::vector<std::string> bad;
  std::string line;
  while (std::getline(in, line)) {
    if (line.empty()) continue;
    std::istringstream ls(line);
    std::string h, name;
    ls >> h >> name;
    if (name.empty()) throw std::runtime_error("malformed checksums.txt line: " + line);
    struct stat st;
    if (stat((dir + "/" + name).c_str(), &st) != 0 || file_digest_hex(dir + "/" + name) != h) bad.push_back(name);
  }
  return bad;
}

// ------------------------------------------------------------------ materializer
namespace {

struct Item {
  const SafetensorsFile* file;
  std::string name;         // source tensor name
  bool quant = false, fp8 = false, cast = false;
  uint64_t out_bytes = 0;
};

SrcType src_type(const std::string& dt, const std::string& name) {
  if (dt == "F32") return SrcType::F32;
  if (dt == "BF16") return SrcType::BF16;
  if (dt == "F16") return SrcType::F16;
  throw std::invalid_argument(name + ": cannot quantize / cast dtype " + dt);
}

}  // namespace

MaterializeReport materialize_nvfp4(const MaterializeOptions& o) {
  MaterializeReport rep;
  std::vector<std::unique_ptr<SafetensorsFile>> files;
  for (auto& p : o.inputs) files.emplace_back(new SafetensorsFile(p));
  rep.files = (int)files.size();
  std::vector<Item> items;
  std::set<std::string> seen, quant_found;
  for (auto& f : files) {
    for (auto& n : f->keys()) {
      if (!seen.insert(n).second) throw std::invalid_argument("tensor in more than one input file: " + n);
      const TensorInfo& ti = f->info(n);
      Item it{f.get(), n};
      const uint64_t nb = ti.end - ti.begin;
      rep.bytes_in += nb;
      const std::string base = n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0 ? n.substr(0, n.size() - 7) : "";
      if (!base.empty() && o.fp8_rows.count(base)) {
        if (ti.shape.size() != 2) throw std::invalid_argument(n + ": FP8-row needs a 2-D weight");
        it.fp8 = true;
        quant_found.insert(base);
        it.out_bytes = (uint64_t)ti.shape[0] * ti.shape[1] + (uint64_t)ti.shape[0] * 4;
      } else if (!base.empty() && o.quantize.count(base)) {
        if (ti.shape.size() != 2 || ti.shape[1] % 16)
          throw std::invalid_argument(n + ": NVFP4 needs a 2-D weight with a multiple of 16 columns");
        it.quant = true;
        quant_found.insert(base);
        const uint64_t r = ti.shape[0], c = ti.shape[1];
        it.out_bytes = r * c / 2 + r * c / 16 + 4;
      } else {
        it.cast = o.cast_bf16.count(n) && ti.dtype != "BF16";
        uint64_t numel = 1;
        for (auto d : ti.shape) numel *= (uint64_t)d;
        it.out_bytes = it.cast ? numel * 2 : nb;
      }
      rep.tensors_in++;
      items.push_back(it);
    }
  }
  for (auto& q : o.quantize)
    if (!quant_found.count(q)) throw std::invalid_argument("weight to quantize not found: " + q + ".weight");
  for (auto& q : o.fp8_rows)
    if (!quant_found.count(q)) throw std::invalid_argument("weight to quantize not found: " + q + ".weight");
  std::sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.name < b.name; });
  // shard plan
  std::vector<std::vector<const Item*>> shards(1);
  uint64_t cur = 0;
  for (auto& it : items) {
    if (!shards.back().empty() && cur + it.out_bytes > o.shard_bytes) {
      shards.emplace_back();
      cur = 0;
    }
    shards.back().push_back(&it);
    cur += it.out_bytes;
  }
  mkdir(o.out_dir.c_str(), 0755);
  std::map<std::string, std::string> wmap;
  char fn[64];
  for (size_t si = 0; si < shards.size(); ++si) {
    snprintf(fn, sizeof fn, "model-%05zu-of-%05zu.safetensors", si + 1, shards.size());
    std::vector<OutTensor> out;
    std::vector<std::vector<uint8_t>> owned;
    owned.reserve(shards[si].size() * 3);
    for (const Item* it : shards[si]) {
      const TensorInfo& ti = it->file->info(it->name);
      const uint8_t* src = it->file->data(it->name);
      if (it->fp8) {
        const int64_t r = ti.shape[0], c = ti.shape[1];
        const SrcType st = src_type(ti.dtype, it->name);
        owned.emplace_back((size_t)(r * c));
        auto& qb = owned.back();
        owned.emplace_back((size_t)(r * 4));
        auto& sb = owned.back();
        quantize_fp8_rows(src, st, r, c, qb.data(), reinterpret_cast<float*>(sb.data()), o.threads);
        const std::string base = it->name.substr(0, it->name.size() - 7);
        out.push_back({base + ".weight", "F8_E4M3", {r, c}, qb.data(), qb.size()});
        out.push_back({base + ".weight_scale", "F32", {r}, sb.data(), sb.size()});
        wmap[base + ".weight"] = fn;
        wmap[base + ".weight_scale"] = fn;
        rep.quantized++;
      } else if (it->quant) {
        const int64_t r = ti.shape[0], c = ti.shape[1];
        const SrcType st = src_type(ti.dtype, it->name);
        owned.emplace_back((size_t)(r * c / 2));
        auto& pk = owned.back();
        owned.emplace_back((size_t)(r * c / 16));
        auto& sf = owned.back();
        owned.emplace_back(4);
        auto& gb = owned.back();
        const float g = quantize_nvfp4(src, st, r, c, 0.f, pk.data(), sf.data(), o.threads);
        memcpy(gb.data(), &g, 4);
        // quantization error (relative Frobenius norm), a numerics report for the overlay
        double num = 0, den = 0;
        for (int64_t i = 0; i < r; ++i)
          for (int64_t j = 0; j < c; ++j) {
            const double w = to_float(src, st, (size_t)(i * c + j));
            const uint8_t code = (pk[(size_t)(i * c + j) / 2] >> ((j & 1) * 4)) & 15;
            const double q = (double)e2m1_value(code) * e4m3_to_float(sf[(size_t)(i * (c / 16) + j / 16)]) * g;
            num += (w - q) * (w - q);
            den += w * w;
          }
        const double rel = den > 0 ? std::sqrt(num / den) : 0.0;
        if (rel > rep.max_rel_err) {
          rep.max_rel_err = rel;
          rep.worst = it->name;
        }
        const std::string base = it->name.substr(0, it->name.size() - 7);
        out.push_back({base + ".weight", "U8", {r, c / 2}, pk.data(), pk.size()});
        out.push_back({base + ".weight_scale", "F8_E4M3", {r, c / 16}, sf.data(), sf.size()});
        out.push_back({base + ".weight_scale_2", "F32", {}, gb.data(), 4});
        for (int k = 0; k < 3; ++k) wmap[out[out.size() - 1 - k].name] = fn;
        rep.quantized++;
      } else if (it->cast) {
        const SrcType st = src_type(ti.dtype, it->name);
        const size_t n = it->out_bytes / 2;
        owned.emplace_back(n * 2);
        auto& b = owned.back();
        RoundNearest rn;
        for (size_t i = 0; i < n; ++i) {
          const float v = to_float(src, st, i);
          uint32_t u;
          memcpy(&u, &v, 4);
          uint16_t h;
          if ((u & 0x7fffffffu) > 0x7f800000u) h = 0x7fc0;  // NaN
          else h = (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);  // round half to even
          memcpy(b.data() + 2 * i, &h, 2);
        }
        out.push_back({it->name, "BF16", ti.shape, b.data(), b.size()});
        wmap[it->name] = fn;
      } else {
        out.push_back({it->name, ti.dtype, ti.shape, src, ti.end - ti.begin});
        wmap[it->name] = fn;
      }
    }
    const std::string path = o.out_dir + "/" + fn;
    write_safetensors(path, out, o.meta);
    struct stat st;
    if (stat(path.c_str(), &st) == 0) rep.bytes_out += (uint64_t)st.st_size;
    rep.checksums[fn] = file_digest_hex(path);
  }
  // index + checksums
  {
    std::string j = "{\n \"metadata\": {";
    bool f = true;
    for (auto& kv : o.meta) {
      j += (f ? "" : ",") + std::string("\n  ") + json_str(kv.first) + ": " + json_str(kv.second);
      f = false;
    }
    j += f ? "},\n \"weight_map\": {" : "\n },\n \"weight_map\": {";
    f = true;
    for (auto& kv : wmap) {
      j += (f ? "" : ",") + std::string("\n  ") + json_str(kv.first) + ": " + json_str(kv.second);
      f = false;
    }
    j += "\n }\n}\n";
    std::ofstream(o.out_dir + "/model.safetensors.index.json") << j;
    std::ofstream cs(o.out_dir + "/checksums.txt");
    for (auto& kv : rep.checksums) cs << kv.second << "  " << kv.first << "\n";
  }
  return rep;
}

}  // namespace rkt_rt
