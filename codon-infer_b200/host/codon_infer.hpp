// C++ host API over the B200 C ABI that keeps codon-infer's own interface for the encoder forward
// and its callers: the names, argument meaning and failure behaviour of EsmConfig,
// EsmWeights{,Q8,Q4,Q3}, Block{Q8_0,Q4_0,Q3_LUT}, BidirectionalRunState, Tokenizer,
// log_softmax_canonical, the forward_bidirectional* family, load_model_weights and the DMS and
// contacts pipelines (codon-infer v1.12.0, src/lib.rs, src/main.rs, src/pipeline.rs). A Rust
// caller binds the C ABI directly (see the integration notes); C++ callers and the C++ tests use
// this header.
//
// Failure behaviour mirrors the reference: loader errors are thrown as IoError carrying the
// io::ErrorKind the reference would return (NotFound, InvalidData, UnexpectedEof); misuse that
// panics in the reference (a sequence longer than the state's max_len) throws std::logic_error.
// Weights live on one GPU: every EsmWeights* object owns one device context.
#pragma once

#include <algorithm>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <functional>
#include <limits>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/esm_b200.h"

namespace codon_infer {

enum class ErrorKind { NotFound, InvalidData, UnexpectedEof, Other };

class IoError : public std::runtime_error {
 public:
  IoError(ErrorKind k, const std::string& m) : std::runtime_error(m), kind_(k) {}
  ErrorKind kind() const { return kind_; }

 private:
  ErrorKind kind_;
};

enum class EsmModelArch { Esm2_8M = 0, Esm2_35M = 1, Esm2_150M = 2, Esm2_650M = 3, Esm2_3B = 4 };

// EsmConfig, src/lib.rs:76-150.
struct EsmConfig {
  size_t dim = 0, hidden_dim = 0, n_layers = 0, n_heads = 0, vocab_size = 33, max_seq_len = 1024;
  EsmModelArch arch = EsmModelArch::Esm2_8M;

  static EsmConfig preset(EsmModelArch a) {
    esm_config c;
    if (esm_config_preset(static_cast<int32_t>(a), &c) != ESM_OK) throw std::invalid_argument("unknown arch");
    return from_c(c);
  }
  static EsmConfig esm2_8m() { return preset(EsmModelArch::Esm2_8M); }
  static EsmConfig esm2_35m() { return preset(EsmModelArch::Esm2_35M); }
  static EsmConfig esm2_150m() { return preset(EsmModelArch::Esm2_150M); }
  static EsmConfig esm2_650m() { return preset(EsmModelArch::Esm2_650M); }
  static EsmConfig esm2_3b() { return preset(EsmModelArch::Esm2_3B); }
  size_t head_dim() const { return dim / n_heads; }

  // EsmConfig::detect_from_file, src/lib.rs:277-297.
  static EsmConfig detect_from_file(const std::string& path) {
    esm_config c;
    int32_t dt = 0;
    const int rc = esm_config_detect_file(path.c_str(), &c, &dt);
    if (rc == ESM_EIO) throw IoError(ErrorKind::NotFound, "cannot open " + path);
    if (rc != ESM_OK) throw IoError(ErrorKind::InvalidData, "unrecognized ESM-2 weights file " + path);
    return from_c(c);
  }

  esm_config to_c() const {
    esm_config c;
    c.dim = static_cast<int32_t>(dim);
    c.hidden_dim = static_cast<int32_t>(hidden_dim);
    c.n_layers = static_cast<int32_t>(n_layers);
    c.n_heads = static_cast<int32_t>(n_heads);
    c.vocab_size = static_cast<int32_t>(vocab_size);
    c.max_seq_len = static_cast<int32_t>(max_seq_len);
    c.arch = static_cast<int32_t>(arch);
    return c;
  }
  static EsmConfig from_c(const esm_config& c) {
    EsmConfig e;
    e.dim = c.dim;
    e.hidden_dim = c.hidden_dim;
    e.n_layers = c.n_layers;
    e.n_heads = c.n_heads;
    e.vocab_size = c.vocab_size;
    e.max_seq_len = c.max_seq_len;
    e.arch = static_cast<EsmModelArch>(c.arch);
    return e;
  }
};

// BlockQ8_0 / BlockQ4_0, src/lib.rs:640-673, 1043-1088 (byte layout of the on-disk formats).
struct BlockQ8_0 {
  float d;
  int8_t qs[32];
  static BlockQ8_0 quantize(const float* src) {
    BlockQ8_0 b;
    esm_quantize_q8(src, 32, &b);
    return b;
  }
  void dequantize_to(float* dst) const {
    for (int i = 0; i < 32; ++i) dst[i] = static_cast<float>(qs[i]) * d;
  }
};
struct BlockQ4_0 {
  float d;
  uint8_t qs[16];
  static BlockQ4_0 quantize(const float* src) {
    BlockQ4_0 b;
    esm_quantize_q4(src, 32, &b);
    return b;
  }
  void dequantize_to(float* dst) const {
    for (int j = 0; j < 16; ++j) {
      dst[j] = static_cast<float>(static_cast<int>(qs[j] & 0x0F) - 8) * d;
      dst[j + 16] = static_cast<float>(static_cast<int>((qs[j] >> 4) & 0x0F) - 8) * d;
    }
  }
};
static_assert(sizeof(BlockQ8_0) == 36 && sizeof(BlockQ4_0) == 20, "block sizes of the CODQ format");

// f32_to_f16 / f16_to_f32 of the reference (src/lib.rs:1291-1337): the Q3_LUT scale encoding, which
// truncates the mantissa and has no subnormal halves.
inline uint16_t f32_to_f16(float v) {
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
inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h >> 15) << 31;
  const int exp = (h >> 10) & 0x1F;
  uint32_t frac = h & 0x3FFu, bits;
  if (exp == 0 && frac == 0) {
    bits = sign;
  } else if (exp == 0) {
    int shift = 0;
    while ((frac & 0x400u) == 0) {
      frac <<= 1;
      ++shift;
    }
    bits = sign | (static_cast<uint32_t>(127 - 15 + 1 - shift) << 23) | ((frac & 0x3FFu) << 13);
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (frac << 13);
  } else {
    bits = sign | (static_cast<uint32_t>(exp + 127 - 15) << 23) | (frac << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// BlockQ3_LUT, src/lib.rs:1343-1501: 32 sign bits, 32 two-bit level indices, the f16 scale.
#pragma pack(push, 1)
struct BlockQ3_LUT {
  uint8_t signs[4];
  uint8_t indices[8];
  uint16_t scale;
  static BlockQ3_LUT quantize(const float* src) {
    BlockQ3_LUT b;
    esm_quantize_q3(src, 32, &b);
    return b;
  }
  void dequantize_to(float* dst) const {
    static const float kLevels[4] = {0.0955f, 0.3030f, 0.5496f, 0.8849f};  // CENTROIDS_Q3
    const float s = f16_to_f32(scale);
    uint32_t sg;
    std::memcpy(&sg, signs, 4);
    for (int i = 0; i < 32; ++i) {
      const float lv = kLevels[(indices[i / 4] >> (2 * (i % 4))) & 3];
      dst[i] = ((sg >> i) & 1u) ? -lv * s : lv * s;
    }
  }
};
#pragma pack(pop)
static_assert(sizeof(BlockQ3_LUT) == 14, "BlockQ3_LUT is 14 bytes");

inline std::vector<BlockQ8_0> quantize_slice_to_q8(const std::vector<float>& src) {
  if (src.size() % 32) throw std::logic_error("Source length must be a multiple of 32");
  std::vector<BlockQ8_0> out(src.size() / 32);
  esm_quantize_q8(src.data(), static_cast<int64_t>(src.size()), out.data());
  return out;
}
inline std::vector<BlockQ4_0> quantize_slice_to_q4(const std::vector<float>& src) {
  if (src.size() % 32) throw std::logic_error("Source length must be a multiple of 32");
  std::vector<BlockQ4_0> out(src.size() / 32);
  esm_quantize_q4(src.data(), static_cast<int64_t>(src.size()), out.data());
  return out;
}

inline std::vector<BlockQ3_LUT> quantize_slice_to_q3_lut(const std::vector<float>& src) {
  if (src.size() % 32) throw std::logic_error("Source length must be a multiple of 32");
  std::vector<BlockQ3_LUT> out(src.size() / 32);
  esm_quantize_q3(src.data(), static_cast<int64_t>(src.size()), out.data());
  return out;
}

// Tokenizer, src/lib.rs:6509-6531.
struct Tokenizer {
  static std::vector<size_t> encode(const std::string& text) {
    std::vector<int32_t> ids(text.size() + 2);
    int32_t n = 0;
    if (esm_tokenize(text.c_str(), ids.data(), static_cast<int32_t>(ids.size()), &n) != ESM_OK)
      throw std::logic_error("tokenizer capacity");
    return std::vector<size_t>(ids.begin(), ids.begin() + n);
  }
  // Tokenizer::decode, src/lib.rs:6523-6530: '\0' where the reference returns None.
  static char decode(size_t id) {
    static const char kAlphabet[] = "LAGVSERTIDPKQNFYMHWCXBUZO.-";
    if (id >= 4 && id <= 30) return kAlphabet[id - 4];
    return id == 32 ? '*' : '\0';
  }
};

// log_softmax_canonical, src/lib.rs:4426-4441.
inline std::vector<float> log_softmax_canonical(const float* logits) {
  std::vector<float> out(33, -std::numeric_limits<float>::infinity());
  float mx = -std::numeric_limits<float>::infinity();
  for (int i = 4; i <= 23; ++i) mx = logits[i] > mx ? logits[i] : mx;
  float s = 0.0f;
  for (int i = 4; i <= 23; ++i) s += std::exp(logits[i] - mx);
  const float lse = mx + std::log(s);
  for (int i = 4; i <= 23; ++i) out[i] = logits[i] - lse;
  return out;
}

// A weight set resident on one GPU (the device context that owns it).
class DeviceWeights {
 public:
  DeviceWeights(const DeviceWeights&) = delete;
  DeviceWeights& operator=(const DeviceWeights&) = delete;
  ~DeviceWeights() {
    if (ctx_) esm_ctx_destroy(ctx_);
  }
  esm_ctx* ctx() const { return ctx_; }
  int32_t dtype() const { return dtype_; }
  const EsmConfig& config() const { return cfg_; }
  size_t reserved_len() const { return reserved_len_; }
  bool reserved_contacts() const { return reserved_contacts_; }
  void reserve(size_t max_len, bool contacts) {
    check(esm_reserve(ctx_, static_cast<int32_t>(max_len), 1, static_cast<int32_t>(max_len), contacts ? 1 : 0));
    reserved_len_ = max_len;
    reserved_contacts_ = contacts;
  }
  // The contact regression head (EsmConfig::contact_head_weights, src/lib.rs:154-177) is an input
  // here: n_layers * n_heads weights (layer-major) and the bias.
  // Workspace for batches (the mutational scans run many windows per forward).
  void reserve_batch(size_t max_tokens, size_t max_seqs, size_t max_len, bool contacts) {
    check(esm_reserve(ctx_, static_cast<int32_t>(max_tokens), static_cast<int32_t>(max_seqs),
                      static_cast<int32_t>(max_len), contacts ? 1 : 0));
    reserved_len_ = max_len;
    reserved_contacts_ = contacts;
  }
  void set_contact_head(const std::vector<float>& weights, float bias) {
    check(esm_set_contact_head(ctx_, weights.data(), static_cast<int32_t>(weights.size()), bias));
    has_contact_head_ = true;
  }
  bool has_contact_head() const { return has_contact_head_; }
  void check(int rc) const {
    if (rc == ESM_OK) return;
    const std::string msg = esm_last_error(ctx_);
    if (rc == ESM_EIO) throw IoError(ErrorKind::UnexpectedEof, msg);
    if (rc == ESM_EFORMAT) throw IoError(ErrorKind::InvalidData, msg);
    if (rc == ESM_ECAPACITY) throw std::logic_error(msg);
    throw IoError(ErrorKind::Other, msg);
  }

 protected:
  DeviceWeights(int device, const EsmConfig& cfg, int32_t dtype) : cfg_(cfg), dtype_(dtype) {
    if (esm_ctx_create(device, &ctx_) != ESM_OK) throw IoError(ErrorKind::Other, "no usable B200 device");
  }
  EsmConfig cfg_;
  int32_t dtype_;
  esm_ctx* ctx_ = nullptr;
  size_t reserved_len_ = 0;
  bool reserved_contacts_ = false;
  bool has_contact_head_ = false;

  void load_file(const std::string& path) {
    const esm_config c = cfg_.to_c();
    check(esm_load_file(ctx_, path.c_str(), &c));
  }
  void load_file_quantized(const std::string& path, int32_t dtype) {
    const esm_config c = cfg_.to_c();
    check(esm_load_file_quantized(ctx_, path.c_str(), &c, dtype));
  }
};

// dtype field of a CODQ header (magic, version, dtype as little-endian u32 at bytes 0, 4, 8), or
// -1 for a header-less file. Throws NotFound when the file cannot be opened.
inline int32_t codq_dtype(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw IoError(ErrorKind::NotFound, "cannot open " + path);
  unsigned char h[12] = {0};
  f.read(reinterpret_cast<char*>(h), sizeof(h));
  if (f.gcount() < static_cast<std::streamsize>(sizeof(h)) || std::memcmp(h, "CODQ", 4) != 0) return -1;
  return static_cast<int32_t>(h[8] | (h[9] << 8) | (h[10] << 16) | (static_cast<uint32_t>(h[11]) << 24));
}

// EsmWeights / EsmWeightsQ8 / EsmWeightsQ4 (src/lib.rs:299-307, 676-687, 1125-1136): from_file
// accepts exactly what the reference loaders accept (CODQ header or header-less layouts).
#define CODON_INFER_WEIGHTS(NAME, DTYPE)                                                              \
  class NAME : public DeviceWeights {                                                                 \
   public:                                                                                            \
    static std::unique_ptr<NAME> from_file(const std::string& path, const EsmConfig& cfg, int device = 0) { \
      const int32_t file_dtype = codq_dtype(path);                                                    \
      if (file_dtype >= 0 && file_dtype != DTYPE)                                                     \
        throw IoError(ErrorKind::InvalidData, "CODQ dtype " + std::to_string(file_dtype) + " is not " #NAME); \
      std::unique_ptr<NAME> w(new NAME(device, cfg));                                                 \
      w->load_file(path);                                                                             \
      return w;                                                                                       \
    }                                                                                                 \
                                                                                                      \
   private:                                                                                           \
    NAME(int device, const EsmConfig& cfg) : DeviceWeights(device, cfg, DTYPE) {}                     \
  };
CODON_INFER_WEIGHTS(EsmWeights, ESM_DTYPE_FP32)
CODON_INFER_WEIGHTS(EsmWeightsQ8, ESM_DTYPE_Q8_0)
CODON_INFER_WEIGHTS(EsmWeightsQ4, ESM_DTYPE_Q4_0)
CODON_INFER_WEIGHTS(EsmWeightsQ3, ESM_DTYPE_Q3_LUT)
#undef CODON_INFER_WEIGHTS

// QuantizationMode / LoadedWeights / load_model_weights (src/lib.rs:2255-2261, src/main.rs:119-244):
// the weights of a file as stored, or an FP32 file quantized while loading.
enum class QuantizationMode { Fp32, Q8_0, Q4_0, Q3_LUT };
struct LoadedWeights {
  EsmConfig config;
  QuantizationMode mode = QuantizationMode::Fp32;
  std::unique_ptr<DeviceWeights> weights;
};
class AnyWeights : public DeviceWeights {
 public:
  AnyWeights(int device, const EsmConfig& cfg, int32_t dtype) : DeviceWeights(device, cfg, dtype) {}
  using DeviceWeights::load_file;
  using DeviceWeights::load_file_quantized;
};
inline LoadedWeights load_model_weights(const std::string& path, std::optional<QuantizationMode> quant = std::nullopt,
                                        int device = 0) {
  EsmConfig cfg;
  try {
    cfg = EsmConfig::detect_from_file(path);
  } catch (const IoError& e) {
    if (e.kind() == ErrorKind::NotFound) throw;
    cfg = EsmConfig::esm2_8m();  // load_model_weights falls back to the 8M config (src/main.rs:185-188)
  }
  esm_config cc;
  int32_t dtype = ESM_DTYPE_FP32;
  if (esm_config_detect_file(path.c_str(), &cc, &dtype) != ESM_OK) dtype = ESM_DTYPE_FP32;
  if (dtype == ESM_DTYPE_FP32) {  // header-less files: the name hints of src/main.rs:190-240
    if (path.find("q3") != std::string::npos) dtype = ESM_DTYPE_Q3_LUT;
    else if (path.find("q4") != std::string::npos) dtype = ESM_DTYPE_Q4_0;
    else if (path.find("q8") != std::string::npos) dtype = ESM_DTYPE_Q8_0;
  }
  const int32_t target = (dtype == ESM_DTYPE_FP32 && quant && *quant != QuantizationMode::Fp32)
                             ? static_cast<int32_t>(*quant)  // enum order = CODQ dtype ids
                             : dtype;
  std::unique_ptr<AnyWeights> w(new AnyWeights(device, cfg, target));
  if (target != dtype) w->load_file_quantized(path, target);
  else w->load_file(path);
  LoadedWeights out;
  out.config = cfg;
  out.mode = static_cast<QuantizationMode>(target);
  out.weights = std::move(w);
  return out;
}

// BidirectionalRunState, src/lib.rs:2488-2544: the outputs the pipelines read.
struct BidirectionalRunState {
  size_t max_len;
  std::vector<float> x;              // [max_len * dim]   LN_f(x) after the forward
  std::vector<float> logits;         // [max_len * vocab]
  std::vector<float> contact_probs;  // [max_len * max_len], row-major over the first n*n entries
  bool compute_contacts = true;

  BidirectionalRunState(const EsmConfig& cfg, size_t max_len_)
      : max_len(max_len_),
        x(max_len_ * cfg.dim),
        logits(max_len_ * cfg.vocab_size),
        contact_probs(max_len_ * max_len_) {}
};

// The on_layer hook of the _ext forwards (Option<&mut dyn FnMut(usize, &[f32])>): called with the
// layer index and the residual stream after that layer, seq_len * dim floats. An empty function is
// None.
using OnLayer = std::function<void(size_t, const float*, size_t)>;

namespace detail {
inline void run(const std::vector<size_t>& tokens, DeviceWeights& w, BidirectionalRunState& state,
                const OnLayer& on_layer = nullptr) {
  const size_t L = tokens.size();
  if (L > state.max_len)  // src/lib.rs:5106 (assert!)
    throw std::logic_error("Sequence length " + std::to_string(L) + " exceeds max_len " +
                           std::to_string(state.max_len));
  const size_t n = L >= 2 ? L - 2 : 0;
  // Contact maps need the regression head (an input here, set with set_contact_head).
  const bool contacts = state.compute_contacts && n > 0 && w.has_contact_head();
  if (w.reserved_len() < state.max_len || (contacts && !w.reserved_contacts())) w.reserve(state.max_len, contacts);
  std::vector<int32_t> toks(tokens.begin(), tokens.end());
  const int32_t len = static_cast<int32_t>(L);
  std::vector<float> cmap(contacts ? n * n : 0);
  if (on_layer) {
    // The states of all layers come back with the forward; the hook then sees them in layer
    // order, with the same arguments as the reference's in-loop calls (src/lib.rs:5368-5370).
    esm_config loaded{};
    w.check(esm_get_config(w.ctx(), &loaded, nullptr));
    const size_t nl = static_cast<size_t>(loaded.n_layers), slice = L * static_cast<size_t>(loaded.dim);
    std::vector<float> layers(nl * slice);
    w.check(esm_forward_ext(w.ctx(), toks.data(), &len, 1, len, state.logits.data(), state.x.data(),
                            contacts ? cmap.data() : nullptr, layers.data()));
    for (size_t l = 0; l < nl; ++l) on_layer(l, layers.data() + l * slice, slice);
  } else {
    w.check(esm_forward(w.ctx(), toks.data(), &len, 1, len, state.logits.data(), state.x.data(),
                        contacts ? cmap.data() : nullptr));
  }
  if (contacts) std::copy(cmap.begin(), cmap.end(), state.contact_probs.begin());
}
}  // namespace detail

// forward_bidirectional{,_parallel} (FP32), _q8, _q4 (src/lib.rs:5078-5095, 5442-5448, 5790-5798).
// num_threads is accepted for signature compatibility; the work runs on the GPU.
inline void forward_bidirectional_parallel(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeights& w,
                                           BidirectionalRunState& state, size_t /*num_threads*/) {
  detail::run(tokens, w, state);
}
inline void forward_bidirectional(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeights& w,
                                  BidirectionalRunState& state) {
  detail::run(tokens, w, state);
}
inline void forward_bidirectional_q8(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeightsQ8& w,
                                     BidirectionalRunState& state, size_t /*num_threads*/) {
  detail::run(tokens, w, state);
}
inline void forward_bidirectional_q4(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeightsQ4& w,
                                     BidirectionalRunState& state, size_t /*num_threads*/) {
  detail::run(tokens, w, state);
}
inline void forward_bidirectional_q3(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeightsQ3& w,
                                     BidirectionalRunState& state, size_t /*num_threads*/) {
  detail::run(tokens, w, state);
}
// The _ext forms (src/lib.rs:5097-5103, 5800-5807, 6159-6165): the same forward, plus on_layer.
inline void forward_bidirectional_parallel_ext(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/,
                                               EsmWeights& w, BidirectionalRunState& state, size_t /*num_threads*/,
                                               const OnLayer& on_layer) {
  detail::run(tokens, w, state, on_layer);
}
inline void forward_bidirectional_q4_ext(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeightsQ4& w,
                                         BidirectionalRunState& state, size_t /*num_threads*/,
                                         const OnLayer& on_layer) {
  detail::run(tokens, w, state, on_layer);
}
inline void forward_bidirectional_q3_ext(const std::vector<size_t>& tokens, const EsmConfig& /*cfg*/, EsmWeightsQ3& w,
                                         BidirectionalRunState& state, size_t /*num_threads*/,
                                         const OnLayer& on_layer) {
  detail::run(tokens, w, state, on_layer);
}

// ---- pipelines (src/pipeline.rs) ---------------------------------------------------------------

struct FastaRecord {  // src/fasta.rs:5-9
  std::string id, header, sequence;
};

enum class DmsScoringMode { MaskedMarginal, WildtypeMarginal };  // src/pipeline.rs:14-19

// DmsPositionRow, src/export.rs:7-44: mean over the 19 non-zero deltas and its category.
struct DmsPositionRow {
  size_t pos = 0;  // 1-based
  char wt = 0;
  std::array<float, 20> deltas{};
  float mean_delta_logp = 0.0f;
  float entropy = 0.0f;
  const char* category = "";
  static DmsPositionRow make(size_t pos, char wt, const float* d, float entropy) {
    DmsPositionRow r;
    r.pos = pos;
    r.wt = wt;
    float sum = 0.0f;
    for (int i = 0; i < 20; ++i) {
      r.deltas[i] = d[i];
      if (d[i] != 0.0f) sum += d[i];
    }
    r.mean_delta_logp = sum / 19.0f;
    r.entropy = entropy;
    r.category = r.mean_delta_logp <= -3.8f   ? "Catalytic / Strictly Intolerant"
                 : r.mean_delta_logp <= -2.2f ? "Conserved Structural Core"
                                              : "Tolerated Variable";
    return r;
  }
};

struct DmsPipelineResult {  // src/pipeline.rs:22-30
  std::string protein_id, sequence;
  std::vector<DmsPositionRow> rows;
  double elapsed_ms = 0.0, muts_per_sec = 0.0;
  size_t catalytic_sites_detected = 0;
  DmsScoringMode scoring_mode = DmsScoringMode::MaskedMarginal;
};

// run_pipeline_dms_with_mode (src/pipeline.rs:76-316) without the progress bar and theme: every
// window (masked variants, or wild-type windows) runs through the GPU forward in batches.
inline DmsPipelineResult run_pipeline_dms_with_mode(const FastaRecord& record, size_t window_size, size_t stride,
                                                    const EsmConfig& cfg, DeviceWeights& w, size_t /*num_threads*/,
                                                    DmsScoringMode mode) {
  const std::string& seq = record.sequence;
  const size_t n = seq.size();
  if (n == 0) throw std::logic_error("Sequence cannot be empty");
  const size_t win = (n <= window_size || window_size == 0) ? std::min(n, cfg.max_seq_len)
                                                            : std::min(window_size, cfg.max_seq_len);
  const std::vector<size_t> toks = Tokenizer::encode(seq);
  std::vector<int32_t> residues(toks.begin() + 1, toks.end() - 1);
  const size_t batch = std::min<size_t>(n, 256);
  w.reserve_batch(batch * (win + 2), batch, win + 2, false);
  std::vector<float> deltas(n * 20), entropy(n);
  const auto t0 = std::chrono::steady_clock::now();
  if (mode == DmsScoringMode::MaskedMarginal)
    w.check(esm_dms_masked_marginal(w.ctx(), residues.data(), static_cast<int32_t>(n), static_cast<int32_t>(window_size),
                                    deltas.data(), entropy.data()));
  else
    w.check(esm_dms_wildtype_marginal(w.ctx(), residues.data(), static_cast<int32_t>(n),
                                      static_cast<int32_t>(window_size), static_cast<int32_t>(stride), deltas.data(),
                                      entropy.data()));
  const double secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  DmsPipelineResult r;
  r.protein_id = record.id;
  r.sequence = seq;
  r.scoring_mode = mode;
  for (size_t p = 0; p < n; ++p) {
    r.rows.push_back(DmsPositionRow::make(p + 1, seq[p], &deltas[p * 20], entropy[p]));
    if (r.rows.back().mean_delta_logp <= -3.8f) ++r.catalytic_sites_detected;
  }
  r.elapsed_ms = secs * 1000.0;
  r.muts_per_sec = secs > 0.0 ? static_cast<double>(n * 20) / secs : 0.0;
  return r;
}

// The DMS convenience forms (src/pipeline.rs:33-74), without the terminal theme.
inline DmsPipelineResult run_pipeline_dms_parallel(const FastaRecord& record, size_t window_size, size_t stride,
                                                   const EsmConfig& cfg, DeviceWeights& w, size_t num_threads) {
  return run_pipeline_dms_with_mode(record, window_size, stride, cfg, w, num_threads, DmsScoringMode::MaskedMarginal);
}
inline DmsPipelineResult run_pipeline_dms(const FastaRecord& record, size_t window_size, size_t stride,
                                          const EsmConfig& cfg, EsmWeights& w) {
  return run_pipeline_dms_parallel(record, window_size, stride, cfg, w, 1);
}

struct ContactPair {  // src/benchmark.rs:107-115
  size_t pos1 = 0;
  char res1 = 0;
  size_t pos2 = 0;
  char res2 = 0;
  float apc_score = 0.0f;
  bool is_cys_cys = false;
  bool is_known_disulfide = false;
};

struct ContactsPipelineResult {  // src/pipeline.rs:379-386; contact_probs holds the n x n map
  std::string protein_id;
  size_t sequence_length = 0;
  std::vector<size_t> cys_indices;
  float cys_enrichment_ratio = 0.0f;
  std::vector<ContactPair> top_contacts;
  std::vector<float> contact_probs;
};

// compute_pipeline_contacts_parallel (src/pipeline.rs:410-512): the forward with contacts and the
// pair ranking run on the GPU (esm_contacts_pipeline); at most 4096 top pairs. The weights need
// their contact regression head (set_contact_head).
inline ContactsPipelineResult compute_pipeline_contacts_parallel(const FastaRecord& record, size_t min_separation,
                                                                  float top_l_factor, std::optional<size_t> max_k,
                                                                  const EsmConfig& /*cfg*/, DeviceWeights& w,
                                                                  size_t /*num_threads*/) {
  const std::string& seq = record.sequence;
  const size_t n = seq.size();
  if (n < 4) throw std::logic_error("Sequence too short for contact prediction");
  if (w.reserved_len() < n + 2 || !w.reserved_contacts()) w.reserve(n + 2, true);
  ContactsPipelineResult r;
  r.protein_id = record.id;
  r.sequence_length = n;
  for (size_t i = 0; i < n; ++i)
    if (seq[i] == 'C') r.cys_indices.push_back(i);
  r.contact_probs.resize(n * n);
  std::vector<int32_t> p1(4096), p2(4096);
  std::vector<float> sc(4096);
  int32_t k = 0;
  w.check(esm_contacts_pipeline(w.ctx(), seq.c_str(), static_cast<int32_t>(min_separation),
                                max_k ? static_cast<int32_t>(std::min<size_t>(*max_k, 1u << 30)) : -1, top_l_factor,
                                nullptr, r.contact_probs.data(), p1.data(), p2.data(), sc.data(), &k,
                                &r.cys_enrichment_ratio));
  for (int32_t t = 0; t < k; ++t) {
    ContactPair c;
    c.pos1 = static_cast<size_t>(p1[t]);
    c.pos2 = static_cast<size_t>(p2[t]);
    c.res1 = seq[c.pos1];
    c.res2 = seq[c.pos2];
    c.apc_score = sc[t];
    c.is_cys_cys = c.is_known_disulfide = c.res1 == 'C' && c.res2 == 'C';
    r.top_contacts.push_back(c);
  }
  return r;
}

inline ContactsPipelineResult compute_pipeline_contacts(const FastaRecord& record, size_t min_separation,
                                                        float top_l_factor, std::optional<size_t> max_k,
                                                        const EsmConfig& cfg, EsmWeights& w) {
  return compute_pipeline_contacts_parallel(record, min_separation, top_l_factor, max_k, cfg, w, 1);
}

}  // namespace codon_infer
