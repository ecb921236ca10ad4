// Memory-bound kernels of the encoder forward: sequence setup, embedding (+ first LayerNorm),
// LayerNorm, per-layer weight dequantization, LM-head decoder, output scatter.
//
// All are HBM-bound: one warp per token row, vectorised 16-byte accesses, grids sized to the
// number of rows (every row is independent).
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kRowWarps = 8;  // rows (warps) per 256-thread block

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two-pass LayerNorm statistics of a row held as float4 chunks by one warp: element index of
// chunk c of lane l is 4*(l + 32*c). layer_norm, src/lib.rs:2556-2562 (mean, biased variance,
// eps 1e-5, out = w*(x-mean)*inv + b).
template <int MAXC>
__device__ __forceinline__ void row_stats(const float4 (&v)[MAXC], int nchunks, int d, float& mean, float& inv) {
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c)
    if (c < nchunks) s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
  mean = warp_sum(s) / static_cast<float>(d);
  float q = 0.0f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    if (c < nchunks) {
      const float a = v[c].x - mean, b = v[c].y - mean, e = v[c].z - mean, f = v[c].w - mean;
      q += (a * a + b * b) + (e * e + f * f);
    }
  }
  const float var = warp_sum(q) / static_cast<float>(d);
  inv = 1.0f / sqrtf(var + 1e-5f);
}

constexpr int kMaxChunks = 20;  // d <= 2560 = 32 lanes * 4 floats * 20

// Row kernels are instantiated for the float4 chunks a lane holds, ceil(d / 128) for d = 320 .. 2560,
// so the register footprint (and with it the occupancy) follows the model width.
template <typename F>
void row_dispatch(int d, F&& launch) {
  switch ((d / 4 + 31) / 32) {
    case 1: launch(std::integral_constant<int, 1>{}); break;
    case 2: launch(std::integral_constant<int, 2>{}); break;
    case 3: launch(std::integral_constant<int, 3>{}); break;
    case 4: launch(std::integral_constant<int, 4>{}); break;
    case 5: launch(std::integral_constant<int, 5>{}); break;
    case 8: launch(std::integral_constant<int, 8>{}); break;
    case 10: launch(std::integral_constant<int, 10>{}); break;
    default: launch(std::integral_constant<int, kMaxChunks>{}); break;
  }
}

__global__ void seq_setup_kernel(const int32_t* __restrict__ tokens, const int32_t* __restrict__ cu, int32_t* pos,
                                 int32_t* seq_of, float* embed_scale) {
  const int b = blockIdx.x;
  const int start = cu[b], end = cu[b + 1];
  int masks = 0;
  for (int t = start + threadIdx.x; t < end; t += blockDim.x) {
    pos[t] = t - start;
    seq_of[t] = b;
    masks += (tokens[t] == 32);
  }
  __shared__ int red[32];
  masks = __reduce_add_sync(0xffffffffu, masks);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = masks;
  __syncthreads();
  if (threadIdx.x == 0) {
    int total = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += red[w];
    // mask_ratio_observed and embed_scale exactly as src/lib.rs:5115-5117 (f32 arithmetic).
    const int len = end - start;
    const float ratio = static_cast<float>(total) / static_cast<float>(len > 0 ? len : 1);
    embed_scale[b] = (ratio >= 1.0f) ? 0.0f : (1.0f - 0.12f) / (1.0f - ratio);
  }
}

template <int NCH>
__global__ void embed_ln_kernel(const int32_t* __restrict__ tokens, const int32_t* __restrict__ seq_of,
                                const float* __restrict__ embed_scale, const float* __restrict__ emb_f32,
                                const uint8_t* __restrict__ emb_q8, int V, int T, int d,
                                const float* __restrict__ ln_w, const float* __restrict__ ln_b, float* __restrict__ x,
                                __half* __restrict__ xn, int* err) {
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  int tok = tokens[row];
  if (tok < 0 || tok >= V) {
    if (lane == 0) atomicOr(err, kDevBadToken);
    tok = 32;  // zeros, like <mask>
  }
  const float sc = embed_scale[seq_of[row]];
  const int nchunks = (d / 4 - lane + 31) / 32;
  float4 v[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c >= nchunks) break;
    const int e = 4 * (lane + 32 * c);
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tok != 32) {
      if (emb_f32) {
        val = *reinterpret_cast<const float4*>(emb_f32 + static_cast<size_t>(tok) * d + e);
      } else {
        const size_t flat = static_cast<size_t>(tok) * d + e;
        const uint8_t* blk = emb_q8 + (flat / 32) * kQ8BlockBytes;
        const float ds = *reinterpret_cast<const float*>(blk);
        const char4 q = *reinterpret_cast<const char4*>(blk + 4 + (flat % 32));
        val = make_float4(static_cast<float>(q.x) * ds, static_cast<float>(q.y) * ds, static_cast<float>(q.z) * ds,
                          static_cast<float>(q.w) * ds);
      }
      val.x *= sc;
      val.y *= sc;
      val.z *= sc;
      val.w *= sc;
    }
    v[c] = val;
    *reinterpret_cast<float4*>(x + static_cast<size_t>(row) * d + e) = val;
  }
  float mean, inv;
  row_stats<NCH>(v, nchunks, d, mean, inv);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c >= nchunks) break;
    const int e = 4 * (lane + 32 * c);
    const float4 w = *reinterpret_cast<const float4*>(ln_w + e);
    const float4 bb = *reinterpret_cast<const float4*>(ln_b + e);
    __half2 h0 = __floats2half2_rn(w.x * (v[c].x - mean) * inv + bb.x, w.y * (v[c].y - mean) * inv + bb.y);
    __half2 h1 = __floats2half2_rn(w.z * (v[c].z - mean) * inv + bb.z, w.w * (v[c].w - mean) * inv + bb.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&h0);
    pk.y = *reinterpret_cast<uint32_t*>(&h1);
    *reinterpret_cast<uint2*>(xn + static_cast<size_t>(row) * d + e) = pk;
  }
}

template <int NCH>
__global__ void layernorm_kernel(const float* __restrict__ x, int T, int d, const float* __restrict__ w,
                                 const float* __restrict__ b, __half* __restrict__ out16, int ld16,
                                 float* __restrict__ out32) {
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nchunks = (d / 4 - lane + 31) / 32;
  float4 v[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c >= nchunks) break;
    v[c] = *reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * d + 4 * (lane + 32 * c));
  }
  float mean, inv;
  row_stats<NCH>(v, nchunks, d, mean, inv);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c >= nchunks) break;
    const int e = 4 * (lane + 32 * c);
    const float4 ww = *reinterpret_cast<const float4*>(w + e);
    const float4 bb = *reinterpret_cast<const float4*>(b + e);
    float4 o;
    o.x = ww.x * (v[c].x - mean) * inv + bb.x;
    o.y = ww.y * (v[c].y - mean) * inv + bb.y;
    o.z = ww.z * (v[c].z - mean) * inv + bb.z;
    o.w = ww.w * (v[c].w - mean) * inv + bb.w;
    if (out16) {
      __half2 h0 = __floats2half2_rn(o.x, o.y);
      __half2 h1 = __floats2half2_rn(o.z, o.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      *reinterpret_cast<uint2*>(out16 + static_cast<size_t>(row) * ld16 + e) = pk;
    }
    if (out32) *reinterpret_cast<float4*>(out32 + static_cast<size_t>(row) * d + e) = o;
  }
}

// BlockQ3_LUT (14 bytes, byte-aligned): 32 sign bits, 32 two-bit level indices (element e in bits
// 2 (e % 4) of byte e / 4), the scale as a half in the reference's own encoding (f16_to_f32,
// src/lib.rs:1314-1337, restated bit for bit). Element e = +-level[idx] * scale, the negative
// entries being (-level) * scale as the reference's lookup table holds them (src/lib.rs:1461-1501).
constexpr int kQ3BlockBytes = 14;
__device__ __forceinline__ float q3_half_to_float(uint32_t h) {
  const uint32_t sign = (h >> 15) << 31;
  const int exp = (h >> 10) & 0x1F;
  uint32_t frac = h & 0x3FFu;
  if (exp == 0) {
    if (frac == 0) return __uint_as_float(sign);
    int shift = 0;
    while ((frac & 0x400u) == 0) {
      frac <<= 1;
      ++shift;
    }
    return __uint_as_float(sign | (static_cast<uint32_t>(127 - 15 + 1 - shift) << 23) | ((frac & 0x3FFu) << 13));
  }
  if (exp == 31) return __uint_as_float(sign | 0x7F800000u | (frac << 13));
  return __uint_as_float(sign | (static_cast<uint32_t>(exp + 127 - 15) << 23) | (frac << 13));
}
// Elements [8 part, 8 part + 8) of the Q3_LUT block at `blk`.
__device__ __forceinline__ void q3_part(const uint8_t* blk, int part, float* v) {
  const float s = q3_half_to_float(static_cast<uint32_t>(blk[12]) | (static_cast<uint32_t>(blk[13]) << 8));
  const uint32_t sg = blk[part];
  const uint32_t ix = static_cast<uint32_t>(blk[4 + 2 * part]) | (static_cast<uint32_t>(blk[5 + 2 * part]) << 8);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t k = (ix >> (2 * e)) & 3u;  // CENTROIDS_Q3, src/lib.rs:1339
    const float lv = k == 0 ? 0.0955f : (k == 1 ? 0.3030f : (k == 2 ? 0.5496f : 0.8849f));
    v[e] = ((sg >> e) & 1u) ? __fmul_rn(-lv, s) : __fmul_rn(lv, s);
  }
}

// One thread per 32-element block: reads the block (fp32 or BlockQ8_0 / BlockQ4_0 bytes) and
// returns its 32 values as q*d in f32, as BlockQ8_0/BlockQ4_0::dequantize_to do
// (src/lib.rs:662-667, 1074-1082).
__device__ __forceinline__ void load_block(int dtype, const void* src, int64_t blk, float (&v)[32]) {
  if (dtype == 0) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(src) + blk * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 a = s[i];
      v[4 * i] = a.x;
      v[4 * i + 1] = a.y;
      v[4 * i + 2] = a.z;
      v[4 * i + 3] = a.w;
    }
  } else if (dtype == 1) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(src) + blk * kQ8BlockBytes);
    const float ds = __uint_as_float(w[0]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t q = w[1 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * i + j] = static_cast<float>(static_cast<int8_t>((q >> (8 * j)) & 0xFF)) * ds;
    }
  } else if (dtype == 2) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(src) + blk * kQ4BlockBytes);
    const float ds = __uint_as_float(w[0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t q = w[1 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t byte = (q >> (8 * j)) & 0xFF;
        v[4 * i + j] = static_cast<float>(static_cast<int>(byte & 0x0F) - 8) * ds;
        v[4 * i + j + 16] = static_cast<float>(static_cast<int>(byte >> 4) - 8) * ds;
      }
    }
  } else {
#pragma unroll
    for (int part = 0; part < 4; ++part) q3_part(static_cast<const uint8_t*>(src) + blk * kQ3BlockBytes, part, v + 8 * part);
  }
}

__device__ __forceinline__ void convert_block(int dtype, const void* src, int64_t blk, __half* dst) {
  float v[32];
  load_block(dtype, src, blk, v);
  uint4* o = reinterpret_cast<uint4*>(dst + blk * 32);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
    o[i] = *reinterpret_cast<uint4*>(h);
  }
}

struct LayerDst {
  __half* dst[6];
  int64_t blk_end[6];  // cumulative block counts
};

// Elements [8 part, 8 part + 8) of a 32-element block, as load_block gives them. For BlockQ4_0,
// elements 0..15 are the low nibbles of qs[0..15] and 16..31 the high nibbles, so part p reads the
// eight bytes qs[8 (p & 1) .. 8 (p & 1) + 8).
__device__ __forceinline__ void load_block_part(int dtype, const void* src, int64_t blk, int part, float (&v)[8]) {
  if (dtype == 0) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(src) + blk * 32 + part * 8);
    const float4 a = s[0], c = s[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
  } else if (dtype == 1) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(src) + blk * kQ8BlockBytes);
    const float ds = __uint_as_float(w[0]);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t q = w[1 + 2 * part + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[4 * i + j] = static_cast<float>(static_cast<int8_t>((q >> (8 * j)) & 0xFF)) * ds;
    }
  } else if (dtype == 3) {
    q3_part(static_cast<const uint8_t*>(src) + blk * kQ3BlockBytes, part, v);
  } else {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(src) + blk * kQ4BlockBytes);
    const float ds = __uint_as_float(w[0]);
    const int shift = part < 2 ? 0 : 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t q = w[1 + 2 * (part & 1) + i];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[4 * i + j] = static_cast<float>(static_cast<int>((q >> (8 * j + shift)) & 0x0F) - 8) * ds;
    }
  }
}

// A quarter block (8 elements) per thread, so each warp writes 512 contiguous bytes of fp16.
__global__ void dequant_layer_kernel(LayerSrc src, LayerDst dst, int64_t total_quarters) {
  for (int64_t g4 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g4 < total_quarters;
       g4 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = g4 >> 2;
    const int part = static_cast<int>(g4 & 3);
    // Matrix of block g, selected with constant indices (no local-memory copy of the arrays).
    const void* w = src.w[0];
    __half* o = dst.dst[0];
    int64_t base = 0;
    int dt = src.dtype[0];
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      if (g >= dst.blk_end[i]) {
        w = src.w[i + 1];
        o = dst.dst[i + 1];
        base = dst.blk_end[i];
        dt = src.dtype[i + 1];
      }
    }
    const int64_t blk = g - base;
    float v[8];
    load_block_part(dt, w, blk, part, v);
    __half2 h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(o + blk * 32 + part * 8) = *reinterpret_cast<uint4*>(h);
  }
}

__global__ void to_f16_kernel(int dtype, const void* src, int64_t nblocks, __half* dst) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < nblocks;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x)
    convert_block(dtype, src, g, dst);
}

__global__ void to_f32_kernel(int dtype, const void* src, int64_t nblocks, float* dst) {
  for (int64_t g = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; g < nblocks;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[32];
    load_block(dtype, src, g, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[g * 32 + i] = v[i];
  }
}

__global__ void gather_tokens_kernel(const int32_t* __restrict__ padded, const int32_t* __restrict__ cu, int Lmax,
                                     int32_t* __restrict__ packed) {
  const int b = blockIdx.x;
  const int start = cu[b], len = cu[b + 1] - start;
  for (int l = threadIdx.x; l < len; l += blockDim.x) packed[start + l] = padded[static_cast<size_t>(b) * Lmax + l];
}

__global__ void scatter_maps_kernel(const float* __restrict__ src, const int64_t* __restrict__ m_off,
                                    const int32_t* __restrict__ cu, int Lmax, float* __restrict__ dst) {
  const int b = blockIdx.y, i = blockIdx.x;
  const int np = Lmax - 2;
  const int n = cu[b + 1] - cu[b] - 2;
  float* o = dst + (static_cast<size_t>(b) * np + i) * np;
  for (int j = threadIdx.x; j < np; j += blockDim.x)
    o[j] = (i < n && j < n) ? src[m_off[b] + static_cast<int64_t>(i) * n + j] : 0.0f;
}

// LM head tail (src/lib.rs:5405-5428): optional LayerNorm of the row, then V dot products in fp32.
template <int NCH>
__global__ void lm_decoder_kernel(const float* __restrict__ in, int T, int d, int do_ln, const float* __restrict__ ln_w,
                                  const float* __restrict__ ln_b, const float* __restrict__ W,
                                  const float* __restrict__ bias, int V, float* __restrict__ logits) {
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const int nchunks = (d / 4 - lane + 31) / 32;
  float4 v[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (c >= nchunks) break;
    v[c] = *reinterpret_cast<const float4*>(in + static_cast<size_t>(row) * d + 4 * (lane + 32 * c));
  }
  if (do_ln) {
    float mean, inv;
    row_stats<NCH>(v, nchunks, d, mean, inv);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      if (c >= nchunks) break;
      const int e = 4 * (lane + 32 * c);
      const float4 ww = *reinterpret_cast<const float4*>(ln_w + e);
      const float4 bb = *reinterpret_cast<const float4*>(ln_b + e);
      v[c].x = ww.x * (v[c].x - mean) * inv + bb.x;
      v[c].y = ww.y * (v[c].y - mean) * inv + bb.y;
      v[c].z = ww.z * (v[c].z - mean) * inv + bb.z;
      v[c].w = ww.w * (v[c].w - mean) * inv + bb.w;
    }
  }
  for (int o = 0; o < V; ++o) {
    const float* wr = W + static_cast<size_t>(o) * d;
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      if (c >= nchunks) break;
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(wr + 4 * (lane + 32 * c)));
      s += (v[c].x * w4.x + v[c].y * w4.y) + (v[c].z * w4.z + v[c].w * w4.w);
    }
    s = warp_sum(s);
    if (lane == 0) logits[static_cast<size_t>(row) * V + o] = s + (bias ? bias[o] : 0.0f);
  }
}

// Token-tiled form of lm_decoder_kernel for V <= kDecGroups * kDecOut outputs. A CTA takes
// kDecTok tokens: first their row statistics (one warp per row, as above), then the reduction over
// d in chunks of kDecK: the chunk's normalised activations [kDecTok][kDecK] and decoder columns
// [V][kDecK] are staged in shared memory, and thread (token t, group g) accumulates outputs
// g, g + kDecGroups, ... of token t. Every decoder element read from shared memory is a broadcast
// that serves a warp's 32 tokens.
constexpr int kDecTok = 64, kDecK = 80, kDecGroups = 4, kDecOut = 10;
constexpr int kDecLdX = kDecK + 4;  // padded row (conflict-free float4 reads across tokens)
template <int NCH>
__global__ void __launch_bounds__(256)
    lm_decoder_tiled_kernel(const float* __restrict__ in, int T, int d, int do_ln, const float* __restrict__ ln_w,
                            const float* __restrict__ ln_b, const float* __restrict__ W,
                            const float* __restrict__ bias, int V, float* __restrict__ logits) {
  __shared__ __align__(16) float xs[kDecTok * kDecLdX];
  __shared__ __align__(16) float ws[kDecGroups * kDecOut * kDecK];
  __shared__ float mean_s[kDecTok], inv_s[kDecTok];
  const int t0 = blockIdx.x * kDecTok;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (do_ln) {
    const int nchunks = (d / 4 - lane + 31) / 32;
    for (int rr = warp; rr < kDecTok; rr += 8) {
      const int row = t0 + rr;
      float mean = 0.0f, inv = 0.0f;
      if (row < T) {
        float4 v[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          if (c >= nchunks) break;
          v[c] = *reinterpret_cast<const float4*>(in + static_cast<size_t>(row) * d + 4 * (lane + 32 * c));
        }
        row_stats<NCH>(v, nchunks, d, mean, inv);
      }
      if (lane == 0) {
        mean_s[rr] = mean;
        inv_s[rr] = inv;
      }
    }
  }
  const int tok = threadIdx.x % kDecTok;
  const int grp = threadIdx.x / kDecTok;
  float acc[kDecOut];
#pragma unroll
  for (int i = 0; i < kDecOut; ++i) acc[i] = 0.0f;
  for (int k0 = 0; k0 < d; k0 += kDecK) {
    const int kc = min(kDecK, d - k0);  // multiple of 4
    __syncthreads();  // row statistics written / previous chunk consumed
    // Activations: kDecTok rows x kc columns, float4 per thread-step, normalised on the way in.
    for (int e = threadIdx.x; e < kDecTok * (kc / 4); e += 256) {
      const int r = e / (kc / 4), c4 = 4 * (e % (kc / 4));
      const int row = t0 + r;
      float4 x = row < T ? *reinterpret_cast<const float4*>(in + static_cast<size_t>(row) * d + k0 + c4)
                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (do_ln) {
        const float mu = mean_s[r], iv = inv_s[r];
        const float4 ww = *reinterpret_cast<const float4*>(ln_w + k0 + c4);
        const float4 bb = *reinterpret_cast<const float4*>(ln_b + k0 + c4);
        x.x = ww.x * (x.x - mu) * iv + bb.x;
        x.y = ww.y * (x.y - mu) * iv + bb.y;
        x.z = ww.z * (x.z - mu) * iv + bb.z;
        x.w = ww.w * (x.w - mu) * iv + bb.w;
      }
      *reinterpret_cast<float4*>(xs + r * kDecLdX + c4) = x;
    }
    // Decoder columns k0 .. k0 + kc of every output.
    for (int e = threadIdx.x; e < V * (kc / 4); e += 256) {
      const int o = e / (kc / 4), c4 = 4 * (e % (kc / 4));
      *reinterpret_cast<float4*>(ws + o * kDecK + c4) =
          __ldg(reinterpret_cast<const float4*>(W + static_cast<size_t>(o) * d + k0 + c4));
    }
    __syncthreads();
    const float* xr = xs + tok * kDecLdX;
    for (int k = 0; k < kc; k += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(xr + k);
#pragma unroll
      for (int i = 0; i < kDecOut; ++i) {
        const int o = grp + kDecGroups * i;
        if (o < V) {
          const float4 w4 = *reinterpret_cast<const float4*>(ws + o * kDecK + k);
          acc[i] += (xv.x * w4.x + xv.y * w4.y) + (xv.z * w4.z + xv.w * w4.w);
        }
      }
    }
  }
  const int row = t0 + tok;
  if (row < T) {
#pragma unroll
    for (int i = 0; i < kDecOut; ++i) {
      const int o = grp + kDecGroups * i;
      if (o < V) logits[static_cast<size_t>(row) * V + o] = acc[i] + (bias ? bias[o] : 0.0f);
    }
  }
}

__global__ void scatter_rows_kernel(const float* __restrict__ src, const int32_t* __restrict__ cu, int Lmax, int C,
                                    float* __restrict__ dst) {
  const int b = blockIdx.y;
  const int l = blockIdx.x;
  const int start = cu[b], len = cu[b + 1] - start;
  float* o = dst + (static_cast<size_t>(b) * Lmax + l) * C;
  if (l < len) {
    const float* s = src + static_cast<size_t>(start + l) * C;
    for (int c = threadIdx.x; c < C; c += blockDim.x) o[c] = s[c];
  } else {
    for (int c = threadIdx.x; c < C; c += blockDim.x) o[c] = 0.0f;
  }
}

// CANONICAL_AAS token ids: A C D E F G H I K L M N P Q R S T V W Y.
__constant__ int kCanonicalIds[20] = {5, 23, 13, 9, 18, 6, 21, 12, 15, 4, 20, 17, 14, 16, 10, 8, 11, 7, 22, 19};

__global__ void dms_score_kernel(const float* __restrict__ logits, int V, const int32_t* __restrict__ tok_row,
                                 const int32_t* __restrict__ wt_tok, int n, float* __restrict__ deltas,
                                 float* __restrict__ entropy) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= n) return;
  const float* lg = logits + static_cast<size_t>(tok_row[v]) * V;
  float mx = -INFINITY;
  for (int i = 4; i <= 23; ++i) mx = fmaxf(mx, lg[i]);
  float se = 0.0f;
  for (int i = 4; i <= 23; ++i) se += expf(lg[i] - mx);
  const float lse = mx + logf(se);
  float h = 0.0f;
  for (int i = 4; i <= 23; ++i) {
    const float lp = lg[i] - lse;
    const float pa = expf(lp);
    if (pa > 1e-12f) h -= pa * lp;
  }
  entropy[v] = h;
  const int wt = wt_tok[v];
  // log_softmax_canonical leaves -inf outside 4..=23, so a non-canonical wild type gives -inf - x.
  const float lwt = (wt >= 4 && wt <= 23) ? lg[wt] - lse : -INFINITY;
  for (int c = 0; c < 20; ++c) {
    const int aa = kCanonicalIds[c];
    deltas[static_cast<size_t>(v) * 20 + c] = (aa == wt) ? 0.0f : (lg[aa] - lse) - lwt;
  }
}

__global__ void wait_probe_kernel(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  // Phase 0 never completes: nobody arrives on the barrier.
  mbar_wait(&bar, 0, err, kDevTimeoutProbe, limit_ns);
}

int row_blocks(int T) { return (T + kRowWarps - 1) / kRowWarps; }

}  // namespace

cudaError_t launch_seq_setup(const int32_t* tokens, const int32_t* cu_seqlens, int B, int32_t* pos, int32_t* seq_of,
                             float* embed_scale, cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  seq_setup_kernel<<<B, 256, 0, s>>>(tokens, cu_seqlens, pos, seq_of, embed_scale);
  return cudaGetLastError();
}

cudaError_t launch_embed_ln(const int32_t* tokens, const int32_t* seq_of, const float* embed_scale,
                            const float* emb_f32, const void* emb_q8, int V, int T, int d, const float* ln_w,
                            const float* ln_b, float* x, __half* xn, int* err, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (d % 32 || d > 4 * 32 * kMaxChunks) return cudaErrorInvalidValue;
  row_dispatch(d, [&](auto nch) {
    embed_ln_kernel<decltype(nch)::value><<<row_blocks(T), 32 * kRowWarps, 0, s>>>(
        tokens, seq_of, embed_scale, emb_f32, static_cast<const uint8_t*>(emb_q8), V, T, d, ln_w, ln_b, x, xn, err);
  });
  return cudaGetLastError();
}

cudaError_t launch_layernorm(const float* x, int T, int d, const float* w, const float* b, __half* out16, int ld16,
                             float* out32, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (d % 4 || d > 4 * 32 * kMaxChunks) return cudaErrorInvalidValue;
  row_dispatch(d, [&](auto nch) {
    layernorm_kernel<decltype(nch)::value><<<row_blocks(T), 32 * kRowWarps, 0, s>>>(x, T, d, w, b, out16, ld16, out32);
  });
  return cudaGetLastError();
}

cudaError_t launch_dequant_layer(const LayerSrc& src, __half* wqkv, __half* wo, __half* w1, __half* w2,
                                 cudaStream_t s) {
  LayerDst dst;
  dst.dst[0] = wqkv;
  dst.dst[1] = wqkv + src.elems[0];
  dst.dst[2] = wqkv + src.elems[0] + src.elems[1];
  dst.dst[3] = wo;
  dst.dst[4] = w1;
  dst.dst[5] = w2;
  int64_t acc = 0;
  for (int m = 0; m < 6; ++m) {
    acc += src.elems[m] / 32;
    dst.blk_end[m] = acc;
  }
  const int threads = 256;
  int64_t blocks = (4 * acc + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  dequant_layer_kernel<<<static_cast<int>(blocks), threads, 0, s>>>(src, dst, 4 * acc);
  return cudaGetLastError();
}

int grid_for_blocks(int64_t nb) {
  int64_t blocks = (nb + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return static_cast<int>(blocks);
}

cudaError_t launch_to_f16(int dtype, const void* src, int64_t elems, __half* dst, cudaStream_t s) {
  const int64_t nb = elems / 32;
  if (nb <= 0) return cudaSuccess;
  to_f16_kernel<<<grid_for_blocks(nb), 256, 0, s>>>(dtype, src, nb, dst);
  return cudaGetLastError();
}

cudaError_t launch_to_f32(int dtype, const void* src, int64_t elems, float* dst, cudaStream_t s) {
  const int64_t nb = elems / 32;
  if (nb <= 0) return cudaSuccess;
  to_f32_kernel<<<grid_for_blocks(nb), 256, 0, s>>>(dtype, src, nb, dst);
  return cudaGetLastError();
}

cudaError_t launch_gather_tokens(const int32_t* padded, const int32_t* cu_seqlens, int B, int Lmax, int32_t* packed,
                                 cudaStream_t s) {
  if (B <= 0) return cudaSuccess;
  gather_tokens_kernel<<<B, 256, 0, s>>>(padded, cu_seqlens, Lmax, packed);
  return cudaGetLastError();
}

cudaError_t launch_scatter_maps(const float* src, const int64_t* m_off, const int32_t* cu_seqlens, int B, int Lmax,
                                float* dst, cudaStream_t s) {
  if (B <= 0 || Lmax <= 2) return cudaSuccess;
  scatter_maps_kernel<<<dim3(Lmax - 2, B), 256, 0, s>>>(src, m_off, cu_seqlens, Lmax, dst);
  return cudaGetLastError();
}

cudaError_t launch_lm_decoder(const float* in, int T, int d, int do_ln, const float* ln_w, const float* ln_b,
                              const float* W, const float* bias, int V, float* logits, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (d % 4 || d > 4 * 32 * kMaxChunks) return cudaErrorInvalidValue;
  // Token-tiled kernel when the outputs fit its per-thread slots (ESM vocabularies: V = 33).
  if (V <= kDecGroups * kDecOut) {
    row_dispatch(d, [&](auto nch) {
      lm_decoder_tiled_kernel<decltype(nch)::value><<<(T + kDecTok - 1) / kDecTok, 256, 0, s>>>(
          in, T, d, do_ln, ln_w, ln_b, W, bias, V, logits);
    });
    return cudaGetLastError();
  }
  row_dispatch(d, [&](auto nch) {
    lm_decoder_kernel<decltype(nch)::value><<<row_blocks(T), 32 * kRowWarps, 0, s>>>(in, T, d, do_ln, ln_w, ln_b, W,
                                                                                      bias, V, logits);
  });
  return cudaGetLastError();
}

cudaError_t launch_dms_score(const float* logits, int V, const int32_t* tok_row, const int32_t* wt_tok, int n,
                             float* deltas, float* entropy, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  dms_score_kernel<<<(n + 127) / 128, 128, 0, s>>>(logits, V, tok_row, wt_tok, n, deltas, entropy);
  return cudaGetLastError();
}

cudaError_t launch_wait_probe(int* err, uint64_t limit_ns, cudaStream_t s) {
  wait_probe_kernel<<<1, 1, 0, s>>>(err, limit_ns);
  return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const float* src, const int32_t* cu_seqlens, int B, int Lmax, int C, float* dst,
                                cudaStream_t s) {
  if (B <= 0 || Lmax <= 0) return cudaSuccess;
  dim3 grid(Lmax, B);
  scatter_rows_kernel<<<grid, 128, 0, s>>>(src, cu_seqlens, Lmax, C, dst);
  return cudaGetLastError();
}

}  // namespace esm
