// Host-side weight formats of codon-infer: architecture presets, CODQ header, file-size
// autodetection, tensor layouts of grouped_canonical_v1 / sequential_hf / CODQ files, the Q8_0,
// Q4_0 and Q3_LUT quantizers (bit-exact; this file is compiled without floating-point
// contraction, so every product and sum rounds on its own as in the reference) and the tokenizer.
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
  if (dtype == ESM_DTYPE_Q3_LUT) return elems / 32 * 14;
  return elems * 4;
}

int matrix_dtype(int model_dtype, int tensor) {
  // EsmWeights::quantize_q3 (src/lib.rs:609-633): a Q3_LUT model keeps Q4_0 attention matrices and
  // stores fc1 / fc2 (tensors 13, 15) as Q3_LUT; the other model types use one type throughout.
  if (model_dtype == ESM_DTYPE_Q3_LUT) return (tensor == 13 || tensor == 15) ? ESM_DTYPE_Q3_LUT : ESM_DTYPE_Q4_0;
  return model_dtype;
}

void tensor_layout(const esm_config& c, int dtype, int64_t out_bytes[ESM_NUM_TENSORS]) {
  // Tensor sizes in the EsmWeights{,Q8,Q4} field order (src/lib.rs:369-389, 764-783, 1175-1193);
  // the classifier (index 19) is whatever remains and is filled in by the caller.
  const int64_t d = c.dim, F = c.hidden_dim, nl = c.n_layers, V = c.vocab_size;
  const int64_t vec = nl * d * 4;
  out_bytes[0] = (dtype == ESM_DTYPE_Q8_0) ? matrix_bytes(ESM_DTYPE_Q8_0, V * d) : V * d * 4;
  out_bytes[1] = vec;
  out_bytes[2] = vec;
  for (int i : {3, 5, 7, 9}) out_bytes[i] = matrix_bytes(matrix_dtype(dtype, i), nl * d * d);
  for (int i : {4, 6, 8, 10}) out_bytes[i] = vec;
  out_bytes[11] = vec;
  out_bytes[12] = vec;
  out_bytes[13] = matrix_bytes(matrix_dtype(dtype, 13), nl * F * d);
  out_bytes[14] = nl * F * 4;
  out_bytes[15] = matrix_bytes(matrix_dtype(dtype, 15), nl * d * F);
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

uint16_t q3_scale_to_half(float v) {
  // f32_to_f16, src/lib.rs:1291-1312: the exponent rebiased and the mantissa truncated; zero for
  // f32 subnormals and for results below the half range, infinity above it, NaN payload kept.
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  const uint32_t sign = (bits >> 31) & 1u, frac = bits & 0x7FFFFFu;
  const int exp = static_cast<int>((bits >> 23) & 0xFFu);
  if (exp == 0) return static_cast<uint16_t>(sign << 15);
  if (exp == 0xFF) return static_cast<uint16_t>((sign << 15) | 0x7C00u | std::min<uint32_t>(frac >> 13, 0x3FFu));
  const int e = exp - 127 + 15;
  if (e >= 31) return static_cast<uint16_t>((sign << 15) | 0x7C00u);
  if (e <= 0) return static_cast<uint16_t>(sign << 15);
  return static_cast<uint16_t>((sign << 15) | (static_cast<uint32_t>(e) << 10) | (frac >> 13));
}

float q3_half_to_scale(uint16_t h) {
  // f16_to_f32, src/lib.rs:1314-1337 (half subnormals normalised).
  const uint32_t sign = static_cast<uint32_t>(h >> 15) << 31;
  const int exp = (h >> 10) & 0x1F;
  uint32_t frac = h & 0x3FFu, bits;
  if (exp == 0) {
    if (frac == 0) {
      bits = sign;
    } else {
      int shift = 0;
      while ((frac & 0x400u) == 0) {
        frac <<= 1;
        ++shift;
      }
      bits = sign | (static_cast<uint32_t>(127 - 15 + 1 - shift) << 23) | ((frac & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (frac << 13);
  } else {
    bits = sign | (static_cast<uint32_t>(exp + 127 - 15) << 23) | (frac << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

namespace {

// CENTROIDS_Q3, src/lib.rs:1339: magnitudes of the four levels, in units of the block scale.
constexpr float kQ3Levels[4] = {0.0955f, 0.3030f, 0.5496f, 0.8849f};

// Index of the level nearest to mag / scale (the first of equally near ones) and its distance.
inline int q3_nearest(float mag, float scale, float* dist) {
  int best = 0;
  float dmin = std::fabs(mag - scale * kQ3Levels[0]);
  for (int k = 1; k < 4; ++k) {
    const float dk = std::fabs(mag - scale * kQ3Levels[k]);
    if (dk < dmin) {
      dmin = dk;
      best = k;
    }
  }
  *dist = dmin;
  return best;
}

void quantize_q3_block(const float* x, uint8_t* o) {
  // BlockQ3_LUT::quantize, src/lib.rs:1353-1458: signs apart, magnitudes on four levels times a
  // per-block scale. Four starting scales (max/level3, max, 2.2 rms, 1.6 rms), each refined by four
  // rounds of nearest-level assignment and least-squares scale; the scale is rounded to half (the
  // truncating conversion above) and the start with the smallest squared error on that rounded
  // scale wins (the first on ties).
  uint32_t signs = 0;
  float mag[32], max_abs = 0.0f, sum_sq = 0.0f;
  for (int i = 0; i < 32; ++i) {
    if (x[i] < 0.0f) signs |= 1u << i;
    mag[i] = std::fabs(x[i]);
    if (mag[i] > max_abs) max_abs = mag[i];
    sum_sq += mag[i] * mag[i];
  }
  std::memset(o, 0, 14);
  if (max_abs < 1e-8f) return;
  const float rms = std::sqrt(sum_sq / 32.0f);
  const float starts[4] = {max_abs / kQ3Levels[3], max_abs, rms * 2.2f, rms * 1.6f};
  float best_err = 3.40282347e38f;
  uint16_t best_half = 0;
  uint8_t best_idx[32] = {};
  for (float s0 : starts) {
    float s = std::fmax(s0, 1e-8f);  // f32::max: a NaN operand yields the other one
    uint8_t idx[32];
    float unused;
    for (int round = 0; round < 4; ++round) {
      float num = 0.0f, den = 0.0f;
      for (int i = 0; i < 32; ++i) {
        idx[i] = static_cast<uint8_t>(q3_nearest(mag[i], s, &unused));
        const float lv = kQ3Levels[idx[i]];
        num += mag[i] * lv;
        den += lv * lv;
      }
      if (den > 1e-8f) s = num / den;
    }
    const uint16_t half = q3_scale_to_half(s);
    const float sq = q3_half_to_scale(half);
    float err = 0.0f;
    for (int i = 0; i < 32; ++i) {
      idx[i] = static_cast<uint8_t>(q3_nearest(mag[i], sq, &unused));
      const float diff = mag[i] - sq * kQ3Levels[idx[i]];
      err += diff * diff;
    }
    if (err < best_err) {
      best_err = err;
      best_half = half;
      std::memcpy(best_idx, idx, 32);
    }
  }
  std::memcpy(o, &signs, 4);  // little-endian sign bits
  for (int b = 0; b < 8; ++b)
    o[4 + b] = static_cast<uint8_t>((best_idx[4 * b] & 3) | ((best_idx[4 * b + 1] & 3) << 2) |
                                    ((best_idx[4 * b + 2] & 3) << 4) | ((best_idx[4 * b + 3] & 3) << 6));
  std::memcpy(o + 12, &best_half, 2);
}

}  // namespace

void quantize_q3(const float* src, int64_t n, uint8_t* dst) {
  parallel_for(n / 32, [&](int64_t b0, int64_t b1) {
    for (int64_t b = b0; b < b1; ++b) quantize_q3_block(src + b * 32, dst + b * 14);
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
