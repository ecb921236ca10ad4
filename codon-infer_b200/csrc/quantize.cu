// Q8_0 / Q4_0 quantization on the device: BlockQ8_0::quantize and BlockQ4_0::quantize
// (src/lib.rs:648-660, 1054-1071) applied to every 32-element block of an FP32 array in device
// memory, so that FP32 weights can be quantized where they will be used (the reference quantizes
// on the host when a model is loaded with --q8 / --q4: EsmWeights::quantize_q8 / quantize_q4,
// src/lib.rs:559-607). Byte-for-byte the same blocks as the host quantizers of formats.cpp:
// IEEE division for d and 1/d, an unfused product x * (1/d), round half away from zero, and the
// same comparisons and saturating casts (NaN -> 0), so even non-finite inputs agree.
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.cuh"

namespace esm {

namespace {

// Rust `f32 as i32`: truncation toward zero, saturating, NaN -> 0.
__device__ __forceinline__ int32_t sat_i32(float x) {
  if (x != x) return 0;
  if (x >= 2147483647.0f) return INT32_MAX;
  if (x <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(x);
}

__device__ __forceinline__ void load32(const float* src, int64_t blk, float (&x)[32]) {
  const float4* s = reinterpret_cast<const float4*>(src + blk * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 a = s[i];
    x[4 * i] = a.x;
    x[4 * i + 1] = a.y;
    x[4 * i + 2] = a.z;
    x[4 * i + 3] = a.w;
  }
}

// One thread per block; a BlockQ8_0 is 36 bytes (d, then 32 int8), written as nine words.
__global__ void quantize_q8_kernel(const float* __restrict__ src, int64_t nblocks, uint8_t* __restrict__ dst) {
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[32];
    load32(src, b, x);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fabsf(x[i]) > amax ? fabsf(x[i]) : amax;
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = (d == 0.0f) ? 0.0f : __fdiv_rn(1.0f, d);
    uint32_t* o = reinterpret_cast<uint32_t*>(dst + b * 36);
    o[0] = __float_as_uint(d);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float r = roundf(__fmul_rn(x[4 * w + k], id));
        r = (r < -127.0f) ? -127.0f : r;  // std::max(r, -127) then std::min(., 127): NaN stays NaN
        r = (127.0f < r) ? 127.0f : r;
        word |= (static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(sat_i32(r))))) << (8 * k);
      }
      o[1 + w] = word;
    }
  }
}

// One thread per block; a BlockQ4_0 is 20 bytes (d, then 16 bytes: element j in the low nibble
// of byte j, element j + 16 in its high nibble), written as five words.
__global__ void quantize_q4_kernel(const float* __restrict__ src, int64_t nblocks, uint8_t* __restrict__ dst) {
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nblocks;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float x[32];
    load32(src, b, x);
    float m = 0.0f;  // the first element of largest magnitude, sign kept
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (fabsf(x[i]) > fabsf(m)) m = x[i];
    const float d = (m == 0.0f) ? 0.0f : __fdiv_rn(m, -8.0f);
    const float id = (d == 0.0f) ? 0.0f : __fdiv_rn(1.0f, d);
    uint32_t* o = reinterpret_cast<uint32_t*>(dst + b * 20);
    o[0] = __float_as_uint(d);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t word = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = 4 * w + k;
        // `as i32 + 8` wraps like the reference's release build (reachable only when 1/d
        // overflows, i.e. for blocks whose largest magnitude is subnormal).
        int32_t lo = static_cast<int32_t>(static_cast<uint32_t>(sat_i32(roundf(__fmul_rn(x[j], id)))) + 8u);
        int32_t hi = static_cast<int32_t>(static_cast<uint32_t>(sat_i32(roundf(__fmul_rn(x[j + 16], id)))) + 8u);
        lo = lo < 0 ? 0 : (lo > 15 ? 15 : lo);
        hi = hi < 0 ? 0 : (hi > 15 ? 15 : hi);
        word |= static_cast<uint32_t>((lo & 0x0F) | ((hi & 0x0F) << 4)) << (8 * k);
      }
      o[1 + w] = word;
    }
  }
}

int grid_for(int64_t nblocks) {
  int64_t g = (nblocks + 255) / 256;
  return static_cast<int>(g > 148 * 16 ? 148 * 16 : (g < 1 ? 1 : g));
}

}  // namespace

cudaError_t launch_quantize(int dtype, const float* src, int64_t nblocks, uint8_t* dst, cudaStream_t s) {
  if (nblocks <= 0) return cudaSuccess;
  if (dtype == 1) {
    quantize_q8_kernel<<<grid_for(nblocks), 256, 0, s>>>(src, nblocks, dst);
  } else if (dtype == 2) {
    quantize_q4_kernel<<<grid_for(nblocks), 256, 0, s>>>(src, nblocks, dst);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace esm
