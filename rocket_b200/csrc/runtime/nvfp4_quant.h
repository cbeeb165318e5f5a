// Host NVFP4 quantizer and the offline checkpoint materializer (C++).
//
// NVFP4 triplet of a linear weight W [N, K] (K % 16 == 0):
//   name.weight          U8       [N, K/2]   e2m1 codes, low nibble = even column
//   name.weight_scale    F8_E4M3  [N, K/16]  block scale per 16 columns (row-major)
//   name.weight_scale_2  F32      []         tensor scale g = amax / (448 * 6)
// with  W[n, k] ~= e2m1(code) * e4m3(scale[n, k/16]) * g.  Block scale bits are
// e4m3(blockamax / 6 / g) (round to nearest even, saturating at 448); every value
// is then divided by (scale * g) and rounded to the nearest e2m1 magnitude
// {0, .5, 1, 1.5, 2, 3, 4, 6} with ties to the even code.  The arithmetic order is
// that of the Python codec (fuel/nvfp4.py) so both produce identical bytes.
//
// `materialize_nvfp4` turns a bf16 / fp32 / fp16 safetensors checkpoint into a
// fuel directory: listed weights become triplets, others are copied (optionally
// cast to bf16), output is sharded with a model.safetensors.index.json weight map
// and a checksums.txt of 256-bit digests per shard, so a loader can authenticate
// the files before use.
//
// Counterpart of the reference's native overlay materializer
// (scripts/numerics/materialize-nvfp4-overlay.cc) and fuel checksum script
// (scripts/fuels/build-checksums-blake3.py); the codec follows the layout the
// reference documents at engines/glm5-moe-nvfp4-2b/src/nvfp4.h:1-36.
#pragma once
#include <cstdint>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace rkt_rt {

enum class SrcType { F32, BF16, F16 };

uint8_t e4m3_from_float(float v);  // RNE, saturating at +-448
float e4m3_to_float(uint8_t b);
uint8_t e2m1_code(float q);        // 4-bit code: bit 3 sign, bits 0-2 magnitude index
float e2m1_value(uint8_t code);

float to_float(const void* src, SrcType t, size_t i);
float tensor_amax(const void* src, SrcType t, size_t n, int threads);

// Quantize rows [rows, cols] with the given tensor scale (g <= 0: amax / 2688).
// packed: rows * cols/2 bytes; sf: rows * cols/16 bytes.  Returns g.
float quantize_nvfp4(const void* src, SrcType t, int64_t rows, int64_t cols, float g,
                     uint8_t* packed, uint8_t* sf, int threads);

// FP8-row: per-row scale s_r = amax_r / 448 (1 for a zero row), q = e4m3(w / s_r).
void quantize_fp8_rows(const void* src, SrcType t, int64_t rows, int64_t cols, uint8_t* q, float* scale,
                       int threads);

// Row-major scales [rows, k_sf] -> tcgen05 512-byte atom layout (zero padded):
// atom (r/128, s/4) k-fastest, byte (r%32)*16 + ((r%128)/32)*4 + s%4.
size_t sf_swizzled_bytes(int64_t rows, int64_t k_sf);
void swizzle_sf(const uint8_t* sf_linear, int64_t rows, int64_t k_sf, uint8_t* out);

struct MaterializeOptions {
  std::vector<std::string> inputs;        // .safetensors files
  std::string out_dir;
  std::set<std::string> quantize;         // linear names (without ".weight") to store as NVFP4
  std::set<std::string> fp8_rows;         // linear names to store as FP8-row (e4m3 + fp32 row scales)
  std::set<std::string> cast_bf16;        // full tensor names written as bf16
  uint64_t shard_bytes = 4ull << 30;
  int threads = 0;                        // 0 = hardware concurrency
  std::map<std::string, std::string> meta;
};

struct MaterializeReport {
  int files = 0;
  int tensors_in = 0;
  int quantized = 0;
  uint64_t bytes_in = 0;
  uint64_t bytes_out = 0;
  double max_rel_err = 0.0;               // max over quantized weights of ||W - Q(W)||_F / ||W||_F
  std::string worst;                      // the weight that reached it
  std::map<std::string, std::string> checksums;  // shard file -> hex digest
};

MaterializeReport materialize_nvfp4(const MaterializeOptions& o);

// hex digest256 of a whole file; verify every entry of dir/checksums.txt.
std::string file_digest_hex(const std::string& path);
// Returns the names of shards whose digest does not match (empty: all good).
std::vector<std::string> verify_checksums(const std::string& dir);

// Minimal safetensors writer: tensors in name order, header padded to 8 bytes,
// written to path.tmp then renamed.
struct OutTensor {
  std::string name, dtype;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  uint64_t nbytes = 0;
};
void write_safetensors(const std::string& path, std::vector<OutTensor> tensors,
                       const std::map<std::string, std::string>& meta);

}  // namespace rkt_rt
