// Host-side weight formats of codon-infer: architecture presets, CODQ header, file-size
// autodetection, tensor layouts of grouped_canonical_v1 / sequential_hf / CODQ files, the Q8_0 and
// Q4_0 quantizers (bit-exact) and the tokenizer.
#include "formats.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <thread>
#include <vector>

namespace esm {

bool config_preset(int arch, esm_config* out) {
  // EsmConfig::esm2_8m() .. esm2_3b(), src/lib.rs:87-150.
  static const int kTable[5][4] = {
      {320, 1280, 6, 20}, {480, 1920, 12, 20}, {640, 2560, 30, 20}, {1280, 5120, 33, 20}, {2560, 10240, 36, 40}};
  if (arch < 0 || arch > 4) return false;
  out->dim = kTable[arch][0];
  out->hidden_dim = kTable[arch][1];
  out->n_layers = kTable[arch][2];
  out->n_heads = kTable[arch][3];
  out->vocab_size = 33;
  out->max_seq_len = 1024;
  out->arch = arch;
  return true;
}

int64_t lm_head_floats(const esm_config& c) {
  // EsmConfig::lm_head_floats, src/lib.rs:190-192.
  return 3LL * c.dim + static_cast<int64_t>(c.dim) * c.dim + static_cast<int64_t>(c.vocab_size) * c.dim + c.vocab_size;
}

int64_t grouped_canonical_floats(const esm_config& c) {
  // EsmConfig::grouped_canonical_floats, src/lib.rs:195-204.
  const int64_t d = c.dim, F = c.hidden_dim;
  return c.vocab_size * d + c.n_layers * (4 * d * d + 9 * d + 2 * d * F + F) + 2 * d + lm_head_floats(c);
}

int64_t sequential_hf_floats(const esm_config& c) {
  // EsmConfig::sequential_hf_floats, src/lib.rs:212-218.
  const int64_t head_dim = c.dim / c.n_heads;
  return grouped_canonical_floats(c) + head_dim / 2 + static_cast<int64_t>(c.n_layers) * c.n_heads + 1;
}

bool detect_from_file_len(uint64_t len, esm_config* out) {
  // EsmConfig::detect_from_file_len, src/lib.rs:228-275: exact sizes first, then size bands.
  switch (len) {
    case 30091652ull: case 30092168ull: return config_preset(0, out);
    case 134067972ull: case 134068984ull: return config_preset(1, out);
    case 592642692ull: case 592645160ull: return config_preset(2, out);
    case 2604339332ull: case 2604342104ull: return config_preset(3, out);
    case 11356354692ull: case 11356360584ull: case 11357091972ull: return config_preset(4, out);
    default: break;
  }
  if (len >= 3000000000ull) return config_preset(4, out);
  if (len >= 2000000000ull) return config_preset(3, out);
  if (len >= 600000000ull) return config_preset(3, out);
  if (len >= 450000000ull) return config_preset(2, out);
  if (len >= 140000000ull) return config_preset(2, out);
  if (len >= 80000000ull) return config_preset(1, out);
  if (len >= 30500000ull) return config_preset(1, out);
  if (len >= 20000000ull) return config_preset(0, out);
  if (len >= 6000000ull) return config_preset(0, out);
  return false;
}

std::string CodqHeader::validate(const esm_config* cfg) const {
  // CodqHeader::validate / to_config, src/lib.rs:953-1036.
  if (std::memcmp(magic, "CODQ", 4) != 0) return "Invalid CODQ magic";
  if (version != 1) return "Unsupported CODQ version: " + std::to_string(version) + ", expected 1";
  esm_config preset;
  if (!config_preset(static_cast<int>(arch), &preset))
    return "Unknown architecture ID in CODQ header: " + std::to_string(arch);
  const esm_config& c = cfg ? *cfg : preset;
  if (cfg && static_cast<int>(arch) != cfg->arch)
    return "CODQ arch mismatch: header has " + std::to_string(arch) + ", expected " + std::to_string(cfg->arch);
  if (static_cast<int>(n_layers) != c.n_layers || static_cast<int>(dim) != c.dim ||
      static_cast<int>(hidden_dim) != c.hidden_dim || static_cast<int>(vocab_size) != c.vocab_size)
    return "CODQ dimension mismatch for arch " + std::to_string(arch);
  return "";
}

int64_t matrix_bytes(int dtype, int64_t elems) {
  if (dtype == ESM_DTYPE_Q8_0) return elems / 32 * 36;
  if (dtype == ESM_DTYPE_Q4_0) return elems / 32 * 20;
  return elems * 4;
}

void tensor_layout(const esm_config& c, int dtype, int64_t out_bytes[ESM_NUM_TENSORS]) {
  // Tensor sizes in the EsmWeights{,Q8,Q4} field order (src/lib.rs:369-389, 764-783, 1175-1193);
  // the classifier (index 19) is whatever remains and is filled in by the caller.
  const int64_t d = c.dim, F = c.hidden_dim, nl = c.n_layers, V = c.vocab_size;
  const int64_t vec = nl * d * 4;
  out_bytes[0] = (dtype == ESM_DTYPE_Q8_0) ? matrix_bytes(ESM_DTYPE_Q8_0, V * d) : V * d * 4;
  out_bytes[1] = vec;
  out_bytes[2] = vec;
  for (int i : {3, 5, 7, 9}) out_bytes[i] = matrix_bytes(dtype, nl * d * d);
  for (int i : {4, 6, 8, 10}) out_bytes[i] = vec;
  out_bytes[11] = vec;
  out_bytes[12] = vec;
  out_bytes[13] = matrix_bytes(dtype, nl * F * d);
  out_bytes[14] = nl * F * 4;
  out_bytes[15] = matrix_bytes(dtype, nl * d * F);
  out_bytes[16] = vec;
  out_bytes[17] = d * 4;
  out_bytes[18] = d * 4;
  out_bytes[19] = 0;
}

namespace {

void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
  unsigned hw = std::thread::hardware_concurrency();
  int64_t nthr = std::max<int64_t>(1, std::min<int64_t>(hw ? hw : 1, n / 65536 + 1));
  if (nthr == 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  const int64_t chunk = (n + nthr - 1) / nthr;
  for (int64_t t = 0; t < nthr; ++t) {
    const int64_t s = t * chunk, e = std::min(n, s + chunk);
    if (s >= e) break;
    th.emplace_back([=, &fn] { fn(s, e); });
  }
  for (auto& t : th) t.join();
}

// Rust `f32 as i32`: truncation toward zero, saturating, NaN -> 0.
int32_t sat_i32(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483647.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(x);
}

}  // namespace

void quantize_q8(const float* src, int64_t n, uint8_t* dst) {
  // BlockQ8_0::quantize, src/lib.rs:648-660: d = max|x| / 127, q = clamp(round(x / d), +-127),
  // with round = half away from zero and the reciprocal computed once (id = 1/d).
  parallel_for(n / 32, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const float* x = src + b * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) amax = std::fabs(x[i]) > amax ? std::fabs(x[i]) : amax;
      const float d = amax / 127.0f;
      const float id = (d == 0.0f) ? 0.0f : 1.0f / d;
      uint8_t* o = dst + b * 36;
      std::memcpy(o, &d, 4);
      for (int i = 0; i < 32; ++i) {
        float r = std::roundf(x[i] * id);
        r = std::min(std::max(r, -127.0f), 127.0f);
        o[4 + i] = static_cast<uint8_t>(static_cast<int8_t>(sat_i32(r)));
      }
    }
  });
}

void quantize_q4(const float* src, int64_t n, uint8_t* dst) {
  // BlockQ4_0::quantize, src/lib.rs:1054-1071: m = the first element of largest magnitude (sign
  // kept), d = m / -8, q = clamp(round(x / d) + 8, 0, 15); element j in the low nibble of byte j,
  // element j + 16 in its high nibble.
  parallel_for(n / 32, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) {
      const float* x = src + b * 32;
      float m = 0.0f;
      for (int i = 0; i < 32; ++i)
        if (std::fabs(x[i]) > std::fabs(m)) m = x[i];
      const float d = (m == 0.0f) ? 0.0f : m / -8.0f;
      const float id = (d == 0.0f) ? 0.0f : 1.0f / d;
      uint8_t* o = dst + b * 20;
      std::memcpy(o, &d, 4);
      for (int j = 0; j < 16; ++j) {
        // `as i32 + 8` wraps like the reference's release build (reachable only when 1/d
        // overflows, i.e. for blocks whose largest magnitude is subnormal).
        int32_t lo = static_cast<int32_t>(static_cast<uint32_t>(sat_i32(std::roundf(x[j] * id))) + 8u);
        int32_t hi = static_cast<int32_t>(static_cast<uint32_t>(sat_i32(std::roundf(x[j + 16] * id))) + 8u);
        lo = std::min(std::max(lo, 0), 15);
        hi = std::min(std::max(hi, 0), 15);
        o[4 + j] = static_cast<uint8_t>((lo & 0x0F) | ((hi & 0x0F) << 4));
      }
    }
  });
}

int tokenize(const char* seq, int32_t* out, int32_t cap, int32_t* n_out) {
  // Tokenizer::encode, src/lib.rs:6511-6521: "<mask_1>" and "<mask>" become '*' first; ids:
  // L A G V S E R T I D P K Q N F Y M H W C = 4..23, X B U Z O . - = 24..30, * = 32, else <unk> = 3.
  std::string s(seq);
  for (const char* pat : {"<mask_1>", "<mask>"}) {
    size_t p;
    while ((p = s.find(pat)) != std::string::npos) s.replace(p, std::strlen(pat), "*");
  }
  static const char kAlpha[] = "LAGVSERTIDPKQNFYMHWCXBUZO.-";
  std::vector<int32_t> ids;
  ids.reserve(s.size() + 2);
  ids.push_back(0);
  for (size_t i = 0; i < s.size();) {
    // Decode one UTF-8 code point; anything outside the table is <unk>.
    unsigned char c = static_cast<unsigned char>(s[i]);
    size_t adv = (c < 0x80) ? 1 : (c >> 5) == 0x6 ? 2 : (c >> 4) == 0xE ? 3 : (c >> 3) == 0x1E ? 4 : 1;
    int32_t id = 3;
    if (adv == 1) {
      if (c == '*') {
        id = 32;
      } else {
        const char* f = std::strchr(kAlpha, static_cast<char>(c));
        if (f && c != 0) id = 4 + static_cast<int32_t>(f - kAlpha);
      }
    }
    ids.push_back(id);
    i += adv;
  }
  ids.push_back(2);
  *n_out = static_cast<int32_t>(ids.size());
  if (static_cast<int32_t>(ids.size()) > cap) return ESM_ECAPACITY;
  std::copy(ids.begin(), ids.end(), out);
  return ESM_OK;
}

}  // namespace esm
