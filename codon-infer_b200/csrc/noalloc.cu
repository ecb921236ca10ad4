// esm_matmul_tiled_noalloc: the dequantizing tensor-core GEMM of esm_matmul_tiled for callers that
// must not allocate device memory.
//
// Who needs it: a host that pre-reserves all device memory at start-up (a serving process with a
// fixed memory budget, or a framework whose caching allocator owns the GPU), a latency-critical
// pipeline that cannot afford cudaMalloc's implicit device-wide synchronisation in the middle of
// its work, or a plugin host that forbids its plugins any allocation. Such callers already own
// their input and output buffers; what esm_matmul_tiled allocates per call is only its scratch
// (the fp16 copies of the operands the tensor cores read, and a padded output when the output
// width is not a multiple of 16). Here that scratch is one file-scope device array of fixed size.
//
// Properties of the array, which every caller should know:
//   * It is kNoallocScratchBytes (32 MiB) of global memory on every GPU where this library's
//     device code is loaded, held until the process exits.
//   * Its device address is obtained once per device with cudaGetSymbolAddress (host code cannot
//     use the symbol itself). The first call on a device does that set-up and also loads the
//     kernels it uses, so that first call should come before any stream capture.
//   * Every call on a device shares that device's array and it keeps the previous call's contents:
//     this entry point clears what must start at zero (the padded bias) on every call. Calls that
//     overlap on the same device (different streams or host threads) race on the array and must be
//     serialised by the caller; calls on different devices use each device's own copy.
//   * The stream and the buffers must belong to the calling thread's current device, whose array
//     the call uses; a stream or output buffer of another device is refused (ESM_EINVAL).
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/esm_b200.h"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = static_cast<size_t>(ESM_NOALLOC_SCRATCH_BYTES);
static_assert(kNoallocScratchBytes % 256 == 0, "scratch size keeps 256-byte sub-allocations");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];
static __device__ int g_noalloc_err;

struct DeviceSlot {
  unsigned char* scratch = nullptr;
  int* err = nullptr;
  int num_sms = 0;
  bool ready = false;
};
constexpr int kMaxDevices = 64;
std::mutex g_slot_mu;
DeviceSlot g_slots[kMaxDevices];

// Once per device, with that device current: device addresses of the scratch array and of the
// error word (the host-side symbols are only stand-ins and must never reach a kernel).
int device_slot(DeviceSlot** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ESM_ECUDA;
  if (dev < 0 || dev >= kMaxDevices) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(g_slot_mu);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    void* scratch = nullptr;
    void* err = nullptr;
    if (cudaGetSymbolAddress(&scratch, g_noalloc_scratch) != cudaSuccess) return ESM_ECUDA;
    if (cudaGetSymbolAddress(&err, g_noalloc_err) != cudaSuccess) return ESM_ECUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return ESM_ECUDA;
    s.scratch = static_cast<unsigned char*>(scratch);
    s.err = static_cast<int*>(err);
    s.num_sms = sms;
    s.ready = true;
  }
  *out = &s;
  return ESM_OK;
}

size_t round256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

extern "C" int esm_matmul_tiled_noalloc(int32_t dtype, const float* d_x, const void* d_w, const float* d_bias,
                                        int32_t in_dim, int32_t out_dim, int32_t seq_len, float* d_out,
                                        void* stream) {
  if (dtype < ESM_DTYPE_FP32 || dtype > ESM_DTYPE_Q3_LUT) return ESM_EINVAL;
  if (!d_x || !d_w || !d_out || in_dim <= 0 || in_dim % 32 || out_dim <= 0 || seq_len <= 0) return ESM_EINVAL;
  // Vector loads and stores need 16-byte aligned fp32 operands; Q8_0 / Q4_0 blocks are read as
  // 32-bit words, Q3_LUT blocks byte by byte.
  const uintptr_t w_align = dtype == ESM_DTYPE_FP32 ? 15 : (dtype == ESM_DTYPE_Q3_LUT ? 0 : 3);
  if ((reinterpret_cast<uintptr_t>(d_x) & 15) || (reinterpret_cast<uintptr_t>(d_out) & 15) ||
      (reinterpret_cast<uintptr_t>(d_w) & w_align) || (reinterpret_cast<uintptr_t>(d_bias) & 3))
    return ESM_EINVAL;
  const int n_pad = (out_dim + 15) / 16 * 16;
  const int bn = esm::gemm_pick_bn_any(n_pad);
  const bool padded_out = n_pad != out_dim;
  const size_t x16_bytes = round256(static_cast<size_t>(seq_len) * in_dim * 2);
  const size_t w16_bytes = round256(static_cast<size_t>(out_dim) * in_dim * 2);
  const size_t bias_bytes = round256(static_cast<size_t>(n_pad) * 4);
  const size_t out_bytes = padded_out ? round256(static_cast<size_t>(seq_len) * n_pad * 4) : 0;
  if (x16_bytes + w16_bytes + bias_bytes + out_bytes > kNoallocScratchBytes) return ESM_ECAPACITY;

  DeviceSlot* slot = nullptr;
  int rc = device_slot(&slot);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The array used is the current device's: the stream and the output must be on that device.
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess) return ESM_ECUDA;
  if (s) {
    int sdev = -1;
    if (cudaStreamGetDevice(s, &sdev) != cudaSuccess) return ESM_EINVAL;
    if (sdev != cur) return ESM_EINVAL;
  }
  cudaPointerAttributes pa{};
  if (cudaPointerGetAttributes(&pa, d_out) != cudaSuccess) return ESM_EINVAL;
  if (pa.type == cudaMemoryTypeDevice && pa.device != cur) return ESM_EINVAL;
  __half* x16 = reinterpret_cast<__half*>(slot->scratch);
  __half* w16 = reinterpret_cast<__half*>(slot->scratch + x16_bytes);
  float* bias = reinterpret_cast<float*>(slot->scratch + x16_bytes + w16_bytes);
  float* out = padded_out ? reinterpret_cast<float*>(slot->scratch + x16_bytes + w16_bytes + bias_bytes) : d_out;

  // The array keeps the previous call's bytes: the bias padding and the error word start at zero.
  cudaError_t e = cudaMemsetAsync(bias, 0, static_cast<size_t>(n_pad) * 4, s);
  if (e == cudaSuccess && d_bias)
    e = cudaMemcpyAsync(bias, d_bias, static_cast<size_t>(out_dim) * 4, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(slot->err, 0, sizeof(int), s);
  if (e == cudaSuccess) e = esm::launch_to_f16(ESM_DTYPE_FP32, d_x, static_cast<int64_t>(seq_len) * in_dim, x16, s);
  if (e == cudaSuccess) e = esm::launch_to_f16(dtype, d_w, static_cast<int64_t>(out_dim) * in_dim, w16, s);
  if (e != cudaSuccess) return ESM_ECUDA;

  // Tensor maps over exactly seq_len x in_dim and out_dim x in_dim: the TMA fills rows past the
  // end with zeros, so no padded copies are needed.
  CUtensorMap ta, tb;
  if (!esm::make_tmap_f16(&ta, x16, static_cast<uint64_t>(seq_len), in_dim, in_dim, 128) ||
      !esm::make_tmap_f16(&tb, w16, static_cast<uint64_t>(out_dim), in_dim, in_dim, static_cast<uint32_t>(bn / 2)))
    return ESM_ECUDA;
  esm::GemmParams p{};
  p.M = seq_len;
  p.N = n_pad;
  p.K = in_dim;
  p.bias = bias;
  p.out = out;
  p.ldo = n_pad;
  p.err = slot->err;
  e = esm::gemm_launch(ta, tb, nullptr, bn, esm::kEpiStoreF32, 0, p, slot->num_sms, s, 1);
  if (e == cudaSuccess && padded_out)
    e = cudaMemcpy2DAsync(d_out, static_cast<size_t>(out_dim) * 4, out, static_cast<size_t>(n_pad) * 4,
                          static_cast<size_t>(out_dim) * 4, seq_len, cudaMemcpyDeviceToDevice, s);
  // The error word comes back on the call's own stream (no legacy-default-stream copy, which
  // would wait for every blocking stream of the device).
  int h_err = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&h_err, slot->err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return ESM_ECUDA;
  return h_err ? ESM_ETIMEOUT : ESM_OK;
}
