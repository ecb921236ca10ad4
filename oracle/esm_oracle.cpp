// ESM-2 bidirectional encoder forward: CPU restatement of codon-infer's reference path.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity checker for the B200 library.
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it;
// the product (codon-infer_b200/) never links or calls it.
//
// Every routine restates the algorithm of the reference crate (Rust, std only) at the
// cited file:line of OsbaldoG/codon-infer v1.12.0, including its numerics:
//   * weights row-major [out, in], Q-blocks of 32 along `in`       src/lib.rs:2629-2634, 2389-2391
//   * BlockQ8_0 {f32 d; i8 qs[32]} 36 B, quantize/dequantize        src/lib.rs:640-673
//   * BlockQ4_0 {f32 d; u8 qs[16]} 20 B, lo nibble=j, hi=j+16, -8   src/lib.rs:1043-1088
//   * BlockQ3_LUT {u8 signs[4]; u8 idx[8]; u16 f16 scale} 14 B,
//     AM-LS quantizer, truncating f32<->f16, 4-level LUT decode       src/lib.rs:1291-1514
//   * Q3_LUT model: Q4_0 attention matrices, Q3_LUT fc1/fc2          src/lib.rs:609-633, 6159-6506
//   * tiled GEMM: dequantize a weight row to fp32 (q*d), then a
//     4-token x 16-lane fp32 FMA dot per output                       src/lib.rs:4446-4531, 4672-4756, 4776-4961
//   * two-pass LayerNorm, eps 1e-5                                   src/lib.rs:2556-2562
//   * GELU with the Abramowitz-Stegun 7.1.26 erf polynomial          src/lib.rs:3485-3498
//   * softmax (max-subtract, exp, scale by 1/sum)                     src/lib.rs:3500-3504
//   * rotate-half RoPE with f32 tables built from powf/cos/sin        src/lib.rs:2510-2522, 3533-3552
//   * token-dropout embedding scale 0.88/(1-#mask/L), <mask> rows 0   src/lib.rs:5117-5131, 5465-5479, 5826-5836
//   * contact head: symmetrize + APC + weighted sum, sigmoid at end   src/lib.rs:5036-5076, 5303-5312, 5373-5377
//   * LM head: LN(gelu(x Wd^T + bd)) Wdec^T + bdec, or x E^T fallback src/lib.rs:5389-5439, 5777-5786
//   * canonical log-softmax over ids 4..=23                          src/lib.rs:4426-4441
//
// Deliberate differences from the reference, none of which changes a result:
//   * the APC row-sum buffer is sized n instead of a fixed [f32; 1024], so n > 1024 works
//     (the reference indexes out of bounds there, src/lib.rs:5046);
//   * attention query rows of one head are split across threads (the reference runs the
//     attention loop on one thread); each row is still computed by exactly one thread in
//     the reference's order, and APC sums keep the reference's sequential order;
//   * the q.k dot product is summed sequentially instead of in 8-lane partial sums
//     (dot_product_head_avx, src/lib.rs:3292-3338), a difference of a few ulp per score.
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace {

struct BlockQ8 {
  float d;
  int8_t qs[32];
};
struct BlockQ4 {
  float d;
  uint8_t qs[16];
};
static_assert(sizeof(BlockQ8) == 36, "BlockQ8_0 is 36 bytes");
static_assert(sizeof(BlockQ4) == 20, "BlockQ4_0 is 20 bytes");
#pragma pack(push, 1)
struct BlockQ3 {
  uint8_t signs[4];    // bit i: element i is negative
  uint8_t indices[8];  // element i: bits 2 (i % 4) of byte i / 4
  uint16_t scale;      // f16 in the reference's own encoding
};
#pragma pack(pop)
static_assert(sizeof(BlockQ3) == 14, "BlockQ3_LUT is 14 bytes");

// Rust's f32::round: half away from zero (same as C roundf).
inline float rust_round(float x) { return std::roundf(x); }

// Float-to-int `as` cast in Rust saturates and maps NaN to 0.
inline int32_t rust_as_i32(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483647.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(x);
}

// BlockQ8_0::quantize, src/lib.rs:648-660.
BlockQ8 quantize_q8_block(const float* src) {
  float max_val = 0.0f;
  for (int i = 0; i < 32; ++i) {
    if (std::fabs(src[i]) > max_val) max_val = std::fabs(src[i]);
  }
  BlockQ8 b;
  b.d = max_val / 127.0f;
  const float id = (b.d == 0.0f) ? 0.0f : 1.0f / b.d;
  for (int i = 0; i < 32; ++i) {
    float r = rust_round(src[i] * id);
    r = std::min(std::max(r, -127.0f), 127.0f);
    b.qs[i] = static_cast<int8_t>(rust_as_i32(r));
  }
  return b;
}

// BlockQ4_0::quantize, src/lib.rs:1054-1071.
BlockQ4 quantize_q4_block(const float* src) {
  float max = 0.0f;
  for (int i = 0; i < 32; ++i) {
    if (std::fabs(src[i]) > std::fabs(max)) max = src[i];
  }
  BlockQ4 b;
  b.d = (max == 0.0f) ? 0.0f : max / -8.0f;
  const float id = (b.d == 0.0f) ? 0.0f : 1.0f / b.d;
  for (int j = 0; j < 16; ++j) {
    int32_t lo = rust_as_i32(rust_round(src[j] * id)) + 8;
    int32_t hi = rust_as_i32(rust_round(src[j + 16] * id)) + 8;
    lo = std::min(std::max(lo, 0), 15);
    hi = std::min(std::max(hi, 0), 15);
    b.qs[j] = static_cast<uint8_t>((lo & 0x0F) | ((hi & 0x0F) << 4));
  }
  return b;
}

// BlockQ8_0::dequantize_to, src/lib.rs:662-667.
void dequant_q8_row(const BlockQ8* blocks, int nblocks, float* dst) {
  for (int b = 0; b < nblocks; ++b)
    for (int i = 0; i < 32; ++i) dst[b * 32 + i] = static_cast<float>(blocks[b].qs[i]) * blocks[b].d;
}

// BlockQ4_0::dequantize_to, src/lib.rs:1074-1082.
void dequant_q4_row(const BlockQ4* blocks, int nblocks, float* dst) {
  for (int b = 0; b < nblocks; ++b) {
    for (int j = 0; j < 16; ++j) {
      const int lo = static_cast<int>(blocks[b].qs[j] & 0x0F) - 8;
      const int hi = static_cast<int>((blocks[b].qs[j] >> 4) & 0x0F) - 8;
      dst[b * 32 + j] = static_cast<float>(lo) * blocks[b].d;
      dst[b * 32 + j + 16] = static_cast<float>(hi) * blocks[b].d;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Thread fan-out: rows [0, n) are split into n_threads contiguous chunks of ceil(n / n_threads),
// the partition of run_tiled_*_slice (src/lib.rs:4776-4801, 4906-4935).
void parallel_chunks(int n, int n_threads, const std::function<void(int, int)>& fn) {
  if (n_threads <= 1 || n < 2) {
    fn(0, n);
    return;
  }
  const int chunk = (n + n_threads - 1) / n_threads;
  std::vector<std::thread> pool;
  for (int t = 0; t < n_threads; ++t) {
    const int s = t * chunk;
    if (s >= n) break;
    const int e = std::min(n, s + chunk);
    pool.emplace_back([=, &fn] { fn(s, e); });
  }
  for (auto& th : pool) th.join();
}

// Horizontal sum of 8 lanes: (lo128 + hi128), then movehl, then the last pair
// (hsum256_ps_avx, src/lib.rs:2563-2572).
__attribute__((target("avx2,fma"))) inline float hsum8(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 s = _mm_add_ps(lo, hi);
  __m128 h64 = _mm_movehl_ps(s, s);
  __m128 s64 = _mm_add_ps(s, h64);
  __m128 h32 = _mm_shuffle_ps(s64, s64, 0x55);
  return _mm_cvtss_f32(_mm_add_ss(s64, h32));
}

// dot_row_batch_m4_avx2_fma, src/lib.rs:4446-4531: out[p, col] = w_row . x[p] + bias for all
// tokens p, 4 tokens at a time, two 8-lane FMA accumulators over 16-float chunks, scalar tail.
__attribute__((target("avx2,fma"))) void dot_row_batch_m4(float* out, int out_stride, int out_col,
                                                        const float* x, const float* w_row, float bias,
                                                        int in_dim, int seq_len) {
  const int chunks16 = in_dim / 16;
  const int rem = chunks16 * 16;
  int p = 0;
  for (; p + 4 <= seq_len; p += 4) {
    const float* x0 = x + static_cast<size_t>(p) * in_dim;
    const float* x1 = x0 + in_dim;
    const float* x2 = x1 + in_dim;
    const float* x3 = x2 + in_dim;
    __m256 a0 = _mm256_setzero_ps(), b0 = _mm256_setzero_ps();
    __m256 a1 = _mm256_setzero_ps(), b1 = _mm256_setzero_ps();
    __m256 a2 = _mm256_setzero_ps(), b2 = _mm256_setzero_ps();
    __m256 a3 = _mm256_setzero_ps(), b3 = _mm256_setzero_ps();
    for (int c = 0; c < chunks16; ++c) {
      const int k = c * 16;
      const __m256 w0 = _mm256_loadu_ps(w_row + k);
      const __m256 w1 = _mm256_loadu_ps(w_row + k + 8);
      a0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x0 + k), a0);
      b0 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x0 + k + 8), b0);
      a1 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x1 + k), a1);
      b1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x1 + k + 8), b1);
      a2 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x2 + k), a2);
      b2 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x2 + k + 8), b2);
      a3 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(x3 + k), a3);
      b3 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(x3 + k + 8), b3);
    }
    float v0 = hsum8(_mm256_add_ps(a0, b0));
    float v1 = hsum8(_mm256_add_ps(a1, b1));
    float v2 = hsum8(_mm256_add_ps(a2, b2));
    float v3 = hsum8(_mm256_add_ps(a3, b3));
    for (int k = rem; k < in_dim; ++k) {
      const float wk = w_row[k];
      v0 += wk * x0[k];
      v1 += wk * x1[k];
      v2 += wk * x2[k];
      v3 += wk * x3[k];
    }
    out[static_cast<size_t>(p) * out_stride + out_col] = v0 + bias;
    out[static_cast<size_t>(p + 1) * out_stride + out_col] = v1 + bias;
    out[static_cast<size_t>(p + 2) * out_stride + out_col] = v2 + bias;
    out[static_cast<size_t>(p + 3) * out_stride + out_col] = v3 + bias;
  }
  for (; p < seq_len; ++p) {
    const float* xp = x + static_cast<size_t>(p) * in_dim;
    __m256 a = _mm256_setzero_ps(), b = _mm256_setzero_ps();
    for (int c = 0; c < chunks16; ++c) {
      const int k = c * 16;
      a = _mm256_fmadd_ps(_mm256_loadu_ps(w_row + k), _mm256_loadu_ps(xp + k), a);
      b = _mm256_fmadd_ps(_mm256_loadu_ps(w_row + k + 8), _mm256_loadu_ps(xp + k + 8), b);
    }
    float v = hsum8(_mm256_add_ps(a, b));
    for (int k = rem; k < in_dim; ++k) v += w_row[k] * xp[k];
    out[static_cast<size_t>(p) * out_stride + out_col] = v + bias;
  }
}

enum { DT_FP32 = 0, DT_Q8 = 1, DT_Q4 = 2, DT_Q3 = 3 };

// f32_to_f16, src/lib.rs:1291-1312 (exponent rebias, mantissa truncated, no subnormal halves).
uint16_t ref_f32_to_f16(float val) {
  uint32_t bits;
  std::memcpy(&bits, &val, 4);
  const uint32_t sign = (bits >> 31) & 1;
  const int32_t exp = static_cast<int32_t>((bits >> 23) & 0xFF);
  const uint32_t frac = bits & 0x7FFFFF;
  if (exp == 0) return static_cast<uint16_t>(sign << 15);
  if (exp == 0xFF) return static_cast<uint16_t>((sign << 15) | 0x7C00 | std::min<uint32_t>(frac >> 13, 0x3FF));
  const int32_t new_exp = exp - 127 + 15;
  if (new_exp >= 31) return static_cast<uint16_t>((sign << 15) | 0x7C00);
  if (new_exp <= 0) return static_cast<uint16_t>(sign << 15);
  return static_cast<uint16_t>((sign << 15) | (static_cast<uint32_t>(new_exp) << 10) | (frac >> 13));
}

// f16_to_f32, src/lib.rs:1314-1337.
float ref_f16_to_f32(uint16_t val) {
  const uint32_t sign = static_cast<uint32_t>(val >> 15) << 31;
  const int32_t exp = (val >> 10) & 0x1F;
  const uint32_t frac = val & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (frac == 0) {
      bits = sign;
    } else {
      uint32_t f = frac;
      int32_t shift = 0;
      while ((f & 0x400) == 0) {
        f <<= 1;
        shift += 1;
      }
      bits = sign | (static_cast<uint32_t>(127 - 15 + 1 - shift) << 23) | ((f & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000 | (frac << 13);
  } else {
    bits = sign | (static_cast<uint32_t>(exp + 127 - 15) << 23) | (frac << 13);
  }
  float r;
  std::memcpy(&r, &bits, 4);
  return r;
}

const float kCentroidsQ3[4] = {0.0955f, 0.3030f, 0.5496f, 0.8849f};  // src/lib.rs:1339

// BlockQ3_LUT::quantize, src/lib.rs:1355-1458: multi-start alternating minimization + least squares.
BlockQ3 quantize_q3_block(const float* src) {
  uint32_t signs_u32 = 0;
  float mags[32];
  float max_abs = 0.0f, sum_sq = 0.0f;
  for (int i = 0; i < 32; ++i) {
    const float v = src[i];
    if (v < 0.0f) signs_u32 |= 1u << i;
    const float a = std::fabs(v);
    mags[i] = a;
    if (a > max_abs) max_abs = a;
    sum_sq += a * a;
  }
  BlockQ3 out;
  std::memset(&out, 0, sizeof(out));
  if (max_abs < 1e-8f) return out;
  const float rms = std::sqrt(sum_sq / 32.0f);
  const float init_scales[4] = {max_abs / kCentroidsQ3[3], max_abs, rms * 2.2f, rms * 1.6f};
  float best_err = 3.40282347e38f;  // f32::MAX
  uint16_t best_scale_f16 = 0;
  uint8_t best_indices[32] = {};
  for (float s_init : init_scales) {
    float s = std::fmax(s_init, 1e-8f);  // f32::max
    uint8_t idx_arr[32] = {};
    for (int step = 0; step < 4; ++step) {
      float num = 0.0f, den = 0.0f;
      for (int i = 0; i < 32; ++i) {
        const float mag = mags[i];
        uint8_t best_k = 0;
        float min_d = std::fabs(mag - s * kCentroidsQ3[0]);
        for (int k = 1; k < 4; ++k) {
          const float dk = std::fabs(mag - s * kCentroidsQ3[k]);
          if (dk < min_d) {
            min_d = dk;
            best_k = static_cast<uint8_t>(k);
          }
        }
        idx_arr[i] = best_k;
        const float c = kCentroidsQ3[best_k];
        num += mag * c;
        den += c * c;
      }
      if (den > 1e-8f) s = num / den;
    }
    const uint16_t cand_f16 = ref_f32_to_f16(s);
    const float s_q = ref_f16_to_f32(cand_f16);
    float err_sq = 0.0f;
    for (int i = 0; i < 32; ++i) {
      const float mag = mags[i];
      uint8_t best_k = 0;
      float min_d = std::fabs(mag - s_q * kCentroidsQ3[0]);
      for (int k = 1; k < 4; ++k) {
        const float dk = std::fabs(mag - s_q * kCentroidsQ3[k]);
        if (dk < min_d) {
          min_d = dk;
          best_k = static_cast<uint8_t>(k);
        }
      }
      idx_arr[i] = best_k;
      const float diff = mag - s_q * kCentroidsQ3[best_k];
      err_sq += diff * diff;
    }
    if (err_sq < best_err) {
      best_err = err_sq;
      best_scale_f16 = cand_f16;
      std::memcpy(best_indices, idx_arr, 32);
    }
  }
  std::memcpy(out.signs, &signs_u32, 4);
  for (int byte_idx = 0; byte_idx < 8; ++byte_idx) {
    out.indices[byte_idx] = static_cast<uint8_t>(
        (best_indices[byte_idx * 4] & 0x03) | ((best_indices[byte_idx * 4 + 1] & 0x03) << 2) |
        ((best_indices[byte_idx * 4 + 2] & 0x03) << 4) | ((best_indices[byte_idx * 4 + 3] & 0x03) << 6));
  }
  out.scale = best_scale_f16;
  return out;
}

// BlockQ3_LUT::dequantize_to, src/lib.rs:1461-1501, per row (unpack_q3_lut_row, 4759-4764).
void dequant_q3_row(const BlockQ3* blocks, int nblocks, float* dst) {
  for (int b = 0; b < nblocks; ++b) {
    const float s = ref_f16_to_f32(blocks[b].scale);
    float lut[8];
    for (int k = 0; k < 4; ++k) {
      lut[k] = kCentroidsQ3[k] * s;
      lut[4 + k] = -kCentroidsQ3[k] * s;
    }
    uint32_t signs;
    std::memcpy(&signs, blocks[b].signs, 4);
    for (int i = 0; i < 32; ++i) {
      const uint32_t idx = (blocks[b].indices[i / 4] >> (2 * (i % 4))) & 0x03;
      const uint32_t sign = (signs >> i) & 1;
      dst[b * 32 + i] = lut[(sign << 2) | idx];
    }
  }
}

// matmul_tiled_{fp32,q8,q4,q3}_parallel, src/lib.rs:4803-4827, 4870-4894, 4937-4961, 4963-5031:
// out[p, i] = sum_k W[i, k] x[p, k] + bias[i]; weight rows are dequantized to fp32 first.
void tiled_gemm(int dtype, float* out, const float* x, const void* w, const float* bias, int in_dim,
                int out_dim, int seq_len, int n_threads) {
  const int nthr = (n_threads <= 1 || out_dim < 16) ? 1 : n_threads;
  parallel_chunks(out_dim, nthr, [&](int s, int e) {
    std::vector<float> wbuf(static_cast<size_t>(in_dim));
    const int bpr = in_dim / 32;
    for (int i = s; i < e; ++i) {
      const float* wrow;
      if (dtype == DT_FP32) {
        wrow = static_cast<const float*>(w) + static_cast<size_t>(i) * in_dim;
      } else if (dtype == DT_Q8) {
        dequant_q8_row(static_cast<const BlockQ8*>(w) + static_cast<size_t>(i) * bpr, bpr, wbuf.data());
        wrow = wbuf.data();
      } else if (dtype == DT_Q4) {
        dequant_q4_row(static_cast<const BlockQ4*>(w) + static_cast<size_t>(i) * bpr, bpr, wbuf.data());
        wrow = wbuf.data();
      } else {
        dequant_q3_row(static_cast<const BlockQ3*>(w) + static_cast<size_t>(i) * bpr, bpr, wbuf.data());
        wrow = wbuf.data();
      }
      dot_row_batch_m4(out, out_dim, i, x, wrow, bias[i], in_dim, seq_len);
    }
  });
}

// layer_norm, src/lib.rs:2556-2562.
void layer_norm(float* out, const float* x, const float* w, const float* b, int dim) {
  float sum = 0.0f;
  for (int i = 0; i < dim; ++i) sum += x[i];
  const float mean = sum / static_cast<float>(dim);
  float var = 0.0f;
  for (int i = 0; i < dim; ++i) {
    const float c = x[i] - mean;
    var += c * c;
  }
  var /= static_cast<float>(dim);
  const float inv = 1.0f / std::sqrt(var + 1e-5f);
  for (int i = 0; i < dim; ++i) out[i] = w[i] * (x[i] - mean) * inv + b[i];
}

// erf_f32 / gelu, src/lib.rs:3485-3498.
inline float erf_as(float x) {
  const float sign = (x < 0.0f) ? -1.0f : 1.0f;
  const float ax = std::fabs(x);
  const float t = 1.0f / (1.0f + 0.3275911f * ax);
  const float y = 1.0f - (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                          0.254829592f) *
                             t * std::exp(-ax * ax);
  return sign * y;
}
inline float gelu(float x) { return 0.5f * x * (1.0f + erf_as(x * 0.70710678118654752440f)); }

// softmax, src/lib.rs:3500-3504.
void softmax(float* x, int n) {
  float mx = -INFINITY;
  for (int i = 0; i < n; ++i) mx = std::max(mx, x[i]);
  float sum = 0.0f;
  for (int i = 0; i < n; ++i) {
    x[i] = std::exp(x[i] - mx);
    sum += x[i];
  }
  const float inv = 1.0f / sum;
  for (int i = 0; i < n; ++i) x[i] *= inv;
}

struct Config {
  int dim, hidden_dim, n_layers, n_heads, vocab_size;
};

struct Weights {
  int dtype;
  const void* tok_emb;  // fp32 [V, d] (FP32 and Q4 models) or BlockQ8_0 [V, d/32] (Q8 models)
  const float *ln1_w, *ln1_b;
  const void *wq, *wk, *wv, *wo;
  const float *bq, *bk, *bv, *bo;
  const float *ln2_w, *ln2_b;
  const void *fc1_w, *fc2_w;
  const float *fc1_b, *fc2_b;
  const float *lnf_w, *lnf_b;
  const float* classifier;
  int64_t classifier_len;
};

size_t weight_elems_bytes(int dtype, size_t elems) {
  if (dtype == DT_FP32) return elems * 4;
  if (dtype == DT_Q8) return elems / 32 * sizeof(BlockQ8);
  if (dtype == DT_Q3) return elems / 32 * sizeof(BlockQ3);
  return elems / 32 * sizeof(BlockQ4);
}

const void* byte_offset(const void* p, size_t bytes) { return static_cast<const uint8_t*>(p) + bytes; }

}  // namespace

extern "C" {

// --- quantizers -------------------------------------------------------------------------------
void orc_quantize_q8(const float* src, int64_t n, void* dst) {
  BlockQ8* out = static_cast<BlockQ8*>(dst);
  for (int64_t b = 0; b < n / 32; ++b) out[b] = quantize_q8_block(src + b * 32);
}
void orc_quantize_q4(const float* src, int64_t n, void* dst) {
  BlockQ4* out = static_cast<BlockQ4*>(dst);
  for (int64_t b = 0; b < n / 32; ++b) out[b] = quantize_q4_block(src + b * 32);
}
void orc_dequantize_q8(const void* src, int64_t n, float* dst) {
  dequant_q8_row(static_cast<const BlockQ8*>(src), static_cast<int>(n / 32), dst);
}
void orc_dequantize_q4(const void* src, int64_t n, float* dst) {
  dequant_q4_row(static_cast<const BlockQ4*>(src), static_cast<int>(n / 32), dst);
}
void orc_quantize_q3(const float* src, int64_t n, void* dst) {
  BlockQ3* out = static_cast<BlockQ3*>(dst);
  for (int64_t b = 0; b < n / 32; ++b) out[b] = quantize_q3_block(src + b * 32);
}
void orc_dequantize_q3(const void* src, int64_t n, float* dst) {
  dequant_q3_row(static_cast<const BlockQ3*>(src), static_cast<int>(n / 32), dst);
}

// --- single kernels, exposed for the known-answer tests ----------------------------------------
void orc_tiled_gemm(int dtype, float* out, const float* x, const void* w, const float* bias, int in_dim,
                    int out_dim, int seq_len, int n_threads) {
  tiled_gemm(dtype, out, x, w, bias, in_dim, out_dim, seq_len, n_threads);
}
void orc_layer_norm(float* out, const float* x, const float* w, const float* b, int dim) {
  layer_norm(out, x, w, b, dim);
}
float orc_gelu(float x) { return gelu(x); }
void orc_softmax(float* x, int n) { softmax(x, n); }

// log_softmax_canonical, src/lib.rs:4426-4441.
void orc_log_softmax_canonical(const float* logits, float* out33) {
  for (int i = 0; i < 33; ++i) out33[i] = -INFINITY;
  float mx = -INFINITY;
  for (int i = 4; i <= 23; ++i) mx = std::max(mx, logits[i]);
  float s = 0.0f;
  for (int i = 4; i <= 23; ++i) s += std::exp(logits[i] - mx);
  const float lse = mx + std::log(s);
  for (int i = 4; i <= 23; ++i) out33[i] = logits[i] - lse;
}

// RoPE tables, BidirectionalRunState::new, src/lib.rs:2510-2522.
void orc_rope_tables(int max_len, int head_dim, float* cos_out, float* sin_out) {
  const int half = head_dim / 2;
  for (int pos = 0; pos < max_len; ++pos) {
    for (int j = 0; j < half; ++j) {
      const float freq = 1.0f / std::pow(10000.0f, static_cast<float>(j * 2) / static_cast<float>(head_dim));
      const float val = static_cast<float>(pos) * freq;
      cos_out[pos * half + j] = std::cos(val);
      sin_out[pos * half + j] = std::sin(val);
    }
  }
}

// accumulate_head_apc, src/lib.rs:5036-5076 (row_sums sized n_res).
void orc_accumulate_head_apc(const float* head_att, float* contact_logits, int seq_len, int n_res, float w_lh) {
  if (n_res == 0 || w_lh == 0.0f) return;
  std::vector<float> row_sums(static_cast<size_t>(n_res));
  float total = 0.0f;
  for (int i = 0; i < n_res; ++i) {
    float r = 0.0f;
    const size_t row_i = static_cast<size_t>(i + 1) * seq_len;
    for (int j = 0; j < n_res; ++j) r += head_att[row_i + (j + 1)] + head_att[static_cast<size_t>(j + 1) * seq_len + (i + 1)];
    row_sums[i] = r;
    total += r;
  }
  const float inv_total = (std::fabs(total) > 1e-12f) ? 1.0f / total : 0.0f;
  for (int i = 0; i < n_res; ++i) {
    const float ri = row_sums[i] * inv_total;
    const size_t row_i = static_cast<size_t>(i + 1) * seq_len;
    float* out = contact_logits + static_cast<size_t>(i) * n_res;
    for (int j = 0; j < n_res; ++j) {
      const float s = head_att[row_i + (j + 1)] + head_att[static_cast<size_t>(j + 1) * seq_len + (i + 1)];
      out[j] += w_lh * (s - ri * row_sums[j]);
    }
  }
}

// --- the forward --------------------------------------------------------------------------------
// forward_bidirectional_parallel_ext (FP32, src/lib.rs:5097-5440), forward_bidirectional_q8
// (src/lib.rs:5442-5788) and forward_bidirectional_q4_ext (src/lib.rs:5800-6147), selected by
// `dtype`. Tensor pointers follow the EsmWeights field order (src/lib.rs:299-307).
// tensors[20] = {tok_emb, ln1_w, ln1_b, wq, bq, wk, bk, wv, bv, wo, bo, ln2_w, ln2_b,
//                fc1_w, fc1_b, fc2_w, fc2_b, lnf_w, lnf_b, classifier}
// Outputs: logits [L, V]; hidden [L, d] = LN_f(x) (state.x after the call) or NULL;
// contacts [n, n] with n = L-2 (state.contact_probs) or NULL to skip the contact head.
// on_layer, when non-NULL, receives the residual stream [L, d] after each layer
// (the on_layer hook of the _ext variants).
int orc_forward(const int* cfg5, int dtype, const void* const* tensors, int64_t classifier_len,
                const int32_t* tokens, int seq_len, int n_threads, const float* contact_w, float contact_b,
                float* logits, float* hidden, float* contacts,
                void (*on_layer)(int layer, const float* x, void* user), void* user) {
  const Config cfg{cfg5[0], cfg5[1], cfg5[2], cfg5[3], cfg5[4]};
  Weights W;
  W.dtype = dtype;
  W.tok_emb = tensors[0];
  W.ln1_w = static_cast<const float*>(tensors[1]);
  W.ln1_b = static_cast<const float*>(tensors[2]);
  W.wq = tensors[3];
  W.bq = static_cast<const float*>(tensors[4]);
  W.wk = tensors[5];
  W.bk = static_cast<const float*>(tensors[6]);
  W.wv = tensors[7];
  W.bv = static_cast<const float*>(tensors[8]);
  W.wo = tensors[9];
  W.bo = static_cast<const float*>(tensors[10]);
  W.ln2_w = static_cast<const float*>(tensors[11]);
  W.ln2_b = static_cast<const float*>(tensors[12]);
  W.fc1_w = tensors[13];
  W.fc1_b = static_cast<const float*>(tensors[14]);
  W.fc2_w = tensors[15];
  W.fc2_b = static_cast<const float*>(tensors[16]);
  W.lnf_w = static_cast<const float*>(tensors[17]);
  W.lnf_b = static_cast<const float*>(tensors[18]);
  W.classifier = static_cast<const float*>(tensors[19]);
  W.classifier_len = classifier_len;

  const int L = seq_len, d = cfg.dim, F = cfg.hidden_dim, H = cfg.n_heads, V = cfg.vocab_size;
  if (L <= 0 || d % 32 || F % 32 || d % H) return 1;
  const int dh = d / H, half = dh / 2;
  const float inv_scale = 1.0f / std::sqrt(static_cast<float>(dh));

  std::vector<float> x(static_cast<size_t>(L) * d), xb(static_cast<size_t>(L) * d);
  std::vector<float> q(static_cast<size_t>(L) * d), k(static_cast<size_t>(L) * d), v(static_cast<size_t>(L) * d);
  std::vector<float> out_att(static_cast<size_t>(L) * d);
  std::vector<float> hb(static_cast<size_t>(L) * std::max(F, d)), hb2(static_cast<size_t>(L) * std::max(F, d));
  std::vector<float> rope_cos(static_cast<size_t>(L) * half), rope_sin(static_cast<size_t>(L) * half);
  orc_rope_tables(L, dh, rope_cos.data(), rope_sin.data());

  // Embedding with token-dropout scaling.
  int mask_count = 0;
  for (int p = 0; p < L; ++p) mask_count += (tokens[p] == 32);
  const float ratio = static_cast<float>(mask_count) / static_cast<float>(L);
  const float embed_scale = (ratio >= 1.0f) ? 0.0f : (1.0f - 0.12f) / (1.0f - ratio);
  for (int p = 0; p < L; ++p) {
    float* xp = x.data() + static_cast<size_t>(p) * d;
    const int tok = tokens[p];
    if (tok == 32) {
      std::fill(xp, xp + d, 0.0f);
    } else if (dtype == DT_Q8) {
      dequant_q8_row(static_cast<const BlockQ8*>(W.tok_emb) + static_cast<size_t>(tok) * (d / 32), d / 32, xp);
      for (int i = 0; i < d; ++i) xp[i] *= embed_scale;
    } else {
      const float* e = static_cast<const float*>(W.tok_emb) + static_cast<size_t>(tok) * d;
      for (int i = 0; i < d; ++i) xp[i] = e[i] * embed_scale;
    }
  }

  const int n_res = std::max(L - 2, 0);
  const bool do_contacts = contacts != nullptr && n_res > 0;
  std::vector<float> head_att, contact_logits;
  if (do_contacts) {
    head_att.assign(static_cast<size_t>(L) * L, 0.0f);
    contact_logits.assign(static_cast<size_t>(n_res) * n_res, 0.0f);
  }
  std::vector<float> att_rows(static_cast<size_t>(L) * L);

  // forward_bidirectional_q3_ext (src/lib.rs:6159-6506) runs the attention projections as Q4_0
  // and fc1 / fc2 as Q3_LUT; the other model types use one matrix type throughout.
  const int dt_att = dtype == DT_Q3 ? DT_Q4 : dtype;
  const int dt_fc = dtype;
  const size_t mat_b = weight_elems_bytes(dt_att, static_cast<size_t>(d) * d);
  const size_t fc1_b = weight_elems_bytes(dt_fc, static_cast<size_t>(d) * F);
  const size_t fc2_b = weight_elems_bytes(dt_fc, static_cast<size_t>(F) * d);

  for (int l = 0; l < cfg.n_layers; ++l) {
    const float* ln1w = W.ln1_w + static_cast<size_t>(l) * d;
    const float* ln1b = W.ln1_b + static_cast<size_t>(l) * d;
    for (int p = 0; p < L; ++p) layer_norm(&xb[static_cast<size_t>(p) * d], &x[static_cast<size_t>(p) * d], ln1w, ln1b, d);
    tiled_gemm(dt_att, q.data(), xb.data(), byte_offset(W.wq, l * mat_b), W.bq + static_cast<size_t>(l) * d, d, d, L, n_threads);
    tiled_gemm(dt_att, k.data(), xb.data(), byte_offset(W.wk, l * mat_b), W.bk + static_cast<size_t>(l) * d, d, d, L, n_threads);
    tiled_gemm(dt_att, v.data(), xb.data(), byte_offset(W.wv, l * mat_b), W.bv + static_cast<size_t>(l) * d, d, d, L, n_threads);

    // apply_rope, src/lib.rs:3533-3552.
    for (int p = 0; p < L; ++p) {
      const float* c = &rope_cos[static_cast<size_t>(p) * half];
      const float* s = &rope_sin[static_cast<size_t>(p) * half];
      float* qp = &q[static_cast<size_t>(p) * d];
      float* kp = &k[static_cast<size_t>(p) * d];
      for (int h = 0; h < H; ++h) {
        for (int j = 0; j < half; ++j) {
          const int i0 = h * dh + j, i1 = h * dh + j + half;
          const float q0 = qp[i0], q1 = qp[i1], k0 = kp[i0], k1 = kp[i1];
          qp[i0] = q0 * c[j] - q1 * s[j];
          qp[i1] = q1 * c[j] + q0 * s[j];
          kp[i0] = k0 * c[j] - k1 * s[j];
          kp[i1] = k1 * c[j] + k0 * s[j];
        }
      }
    }

    // Attention loop, src/lib.rs:5206-5301 (query rows of a head split across threads).
    for (int h = 0; h < H; ++h) {
      parallel_chunks(L, n_threads, [&](int s, int e) {
        for (int p = s; p < e; ++p) {
          float* att = &att_rows[static_cast<size_t>(p) * L];
          const float* qh = &q[static_cast<size_t>(p) * d + h * dh];
          for (int t = 0; t < L; ++t) {
            const float* kh = &k[static_cast<size_t>(t) * d + h * dh];
            float score = 0.0f;
            for (int i = 0; i < dh; ++i) score += qh[i] * kh[i];
            att[t] = score * inv_scale;
          }
          softmax(att, L);
          if (do_contacts) std::memcpy(&head_att[static_cast<size_t>(p) * L], att, sizeof(float) * L);
          float* o = &out_att[static_cast<size_t>(p) * d + h * dh];
          std::fill(o, o + dh, 0.0f);
          for (int t = 0; t < L; ++t) {
            const float pr = att[t];
            const float* vh = &v[static_cast<size_t>(t) * d + h * dh];
            for (int i = 0; i < dh; ++i) o[i] += pr * vh[i];
          }
        }
      });
      if (do_contacts) {
        orc_accumulate_head_apc(head_att.data(), contact_logits.data(), L, n_res, contact_w[l * H + h]);
      }
    }

    tiled_gemm(dt_att, xb.data(), out_att.data(), byte_offset(W.wo, l * mat_b), W.bo + static_cast<size_t>(l) * d, d, d, L, n_threads);
    for (size_t i = 0; i < static_cast<size_t>(L) * d; ++i) x[i] += xb[i];

    const float* ln2w = W.ln2_w + static_cast<size_t>(l) * d;
    const float* ln2b = W.ln2_b + static_cast<size_t>(l) * d;
    for (int p = 0; p < L; ++p) layer_norm(&xb[static_cast<size_t>(p) * d], &x[static_cast<size_t>(p) * d], ln2w, ln2b, d);
    tiled_gemm(dt_fc, hb.data(), xb.data(), byte_offset(W.fc1_w, l * fc1_b), W.fc1_b + static_cast<size_t>(l) * F, d, F, L, n_threads);
    for (size_t i = 0; i < static_cast<size_t>(L) * F; ++i) hb2[i] = gelu(hb[i]);
    tiled_gemm(dt_fc, xb.data(), hb2.data(), byte_offset(W.fc2_w, l * fc2_b), W.fc2_b + static_cast<size_t>(l) * d, F, d, L, n_threads);
    for (size_t i = 0; i < static_cast<size_t>(L) * d; ++i) x[i] += xb[i];
    if (on_layer) on_layer(l, x.data(), user);
  }

  if (do_contacts) {
    for (size_t i = 0; i < contact_logits.size(); ++i)
      contacts[i] = 1.0f / (1.0f + std::exp(-(contact_logits[i] + contact_b)));
  }

  for (int p = 0; p < L; ++p) layer_norm(&xb[static_cast<size_t>(p) * d], &x[static_cast<size_t>(p) * d], W.lnf_w, W.lnf_b, d);
  std::memcpy(x.data(), xb.data(), sizeof(float) * L * d);
  if (hidden) std::memcpy(hidden, x.data(), sizeof(float) * L * d);

  const int64_t required = 3LL * d + static_cast<int64_t>(d) * d + static_cast<int64_t>(V) * d + V;
  if (W.classifier != nullptr && W.classifier_len >= required) {
    const float* lm_ln_w = W.classifier;
    const float* lm_ln_b = W.classifier + d;
    const float* dense_w = W.classifier + 2 * d;
    const float* dense_b = dense_w + static_cast<size_t>(d) * d;
    const float* dec_w = dense_b + d;
    const float* dec_b = dec_w + static_cast<size_t>(V) * d;
    tiled_gemm(DT_FP32, hb.data(), x.data(), dense_w, dense_b, d, d, L, n_threads);
    for (size_t i = 0; i < static_cast<size_t>(L) * d; ++i) hb2[i] = gelu(hb[i]);
    for (int p = 0; p < L; ++p) layer_norm(&xb[static_cast<size_t>(p) * d], &hb2[static_cast<size_t>(p) * d], lm_ln_w, lm_ln_b, d);
    tiled_gemm(DT_FP32, logits, xb.data(), dec_w, dec_b, d, V, L, n_threads);
  } else {
    std::vector<float> zero(static_cast<size_t>(V), 0.0f);
    tiled_gemm(dtype == DT_Q8 ? DT_Q8 : DT_FP32, logits, x.data(), W.tok_emb, zero.data(), d, V, L, n_threads);
  }
  return 0;
}

}  // extern "C"
