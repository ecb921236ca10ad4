// Persistent, warp-specialised tcgen05 GEMM for sm_100a: C[M,N] = A[M,K] . B[N,K]^T, fp16 operands,
// fp32 accumulation in tensor memory, fused epilogues (bias, RoPE, GELU, residual add).
//
// This replaces codon-infer's row-partitioned CPU GEMMs matmul_tiled_{fp32,q8,q4}_parallel
// (src/lib.rs:4803-4827, 4870-4894, 4937-4961) together with the elementwise passes that follow
// them on the hot path: apply_rope (src/lib.rs:3533-3552), gelu (3494-3498) and the residual
// adds (5325-5327, 5364-5366).
//
// CTA layout (192 threads, one CTA per SM):
//   warp 0      TMA producer: stages 128x64 A tiles and BNx64 B tiles (128-byte swizzle) into a
//               ring of shared-memory stages, completion tracked by mbarrier transaction bytes;
//   warp 1      allocates tensor memory and issues tcgen05.mma (M=128, N=BN, K=16) from one thread,
//               releasing each stage with tcgen05.commit;
//   warps 2..5  epilogue: tcgen05.ld of their 32-lane quarter of the accumulator, fused math,
//               stores to global memory.
// Two accumulator buffers in tensor memory let the epilogue of tile i overlap the mainloop of
// tile i+1. Every wait is bounded (globaltimer), so a broken pipeline reports an error instead of
// hanging the GPU.
#include <cstdio>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace esm {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle span of fp16
constexpr int kThreads = 192;
constexpr int kSmemBudget = 200 * 1024;

template <int BN>
struct GemmShape {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;   // TMEM columns between the two accumulators
  static constexpr int kTmemCols = 2 * kAccStride;
  static constexpr int kBarrierBytes = (2 * kStages + 5) * 8 + 16;
  static constexpr int kSmemBytes = kStages * kStageBytes + kBarrierBytes + 1024;  // +1024 for alignment
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 is a multiple of 16 in [16, 256]");
  static_assert(kBBytes % 1024 == 0, "B tile must keep stages 1024-byte aligned");
  static_assert(kStages >= 2, "need at least two stages");
};

__device__ __forceinline__ void store_f16x8(__half* dst, const float* v) {
  __half2 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}

template <int BN, int EPI, int DH>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const GemmParams p) {
  using S = GemmShape<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* acc_full = empty + S::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one_sync()) {
      const uint64_t pol_a = l2_policy_evict_normal();
      const uint64_t pol_b = l2_policy_evict_last();  // weights are re-read by every m-block
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / p.num_n_blocks;
        const int n_blk = tile - m_blk * p.num_n_blocks;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, m_blk * kBM, pol_a);
          tma_load_2d(sb, &tmap_b, &full[stage], kb * kBK, n_blk * BN, pol_b);
          ++fills;
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let the copies this thread may still have in flight (its last kStages fills) land
        // before the CTA exits; each wait is bounded as well.
        int s = stage;
        uint32_t ph = phase;
        for (int j = 0; j < S::kStages && j < fills; ++j) {
          if (--s < 0) {
            s = S::kStages - 1;
            ph ^= 1u;
          }
          mbar_wait(&full[s], ph, p.err, kDevTimeoutProducer);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one_sync()) {
      constexpr uint32_t idesc = umma_idesc_f16(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[buf], acc_phase ^ 1u, p.err, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * S::kAccStride);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            umma_f16(d_tmem, umma_sdesc_sw128(a_addr + k * 32), umma_sdesc_sw128(b_addr + k * 32), idesc,
                     (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        umma_commit(&acc_full[buf]);
      }
      if (!ok) {
        // Wait (bounded) for every MMA this thread issued before tensor memory is released.
        umma_commit(drain);
        mbar_wait(drain, 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32) belong to this warp
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int m_blk = tile / p.num_n_blocks;
      const int n_blk = tile - m_blk * p.num_n_blocks;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], acc_phase, p.err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int m = m_blk * kBM + row_in_tile;
      const bool row_ok = m < p.M;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * S::kAccStride);
      const int n0 = n_blk * BN;

      if constexpr (EPI == kEpiQkvRope) {
        constexpr int HALF = DH / 2;
        const int pos = row_ok ? __ldg(p.pos + m) : 0;
#pragma unroll 1
        for (int c = 0; c < BN; c += DH) {
          uint32_t r[DH];
#pragma unroll
          for (int i = 0; i < DH / 8; ++i) tmem_ld8(t_row + c + 8 * i, r + 8 * i);
          tmem_ld_wait();
          if (row_ok) {
            const int n = n0 + c;
            float v[DH];
#pragma unroll
            for (int i = 0; i < DH; ++i) v[i] = __uint_as_float(r[i]) + (p.bias ? __ldg(p.bias + n + i) : 0.0f);
            if (n < p.rope_cols) {
              const float2* tab = p.rope + static_cast<size_t>(pos) * HALF;
#pragma unroll
              for (int j = 0; j < HALF; ++j) {
                const float2 cs = __ldg(tab + j);
                const float x0 = v[j], x1 = v[j + HALF];
                v[j] = x0 * cs.x - x1 * cs.y;
                v[j + HALF] = x1 * cs.x + x0 * cs.y;
              }
            }
            __half* dst = static_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + n;
#pragma unroll
            for (int i = 0; i < DH / 8; ++i) store_f16x8(dst + 8 * i, v + 8 * i);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16(t_row + c, r);
          tmem_ld_wait();
          if (row_ok) {
            const int n = n0 + c;
            float v[16];
            if (p.bias) {
              const float4* b4 = reinterpret_cast<const float4*>(p.bias + n);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 b = __ldg(b4 + i);
                v[4 * i + 0] = __uint_as_float(r[4 * i + 0]) + b.x;
                v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + b.y;
                v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + b.z;
                v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + b.w;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
            }
            if constexpr (EPI == kEpiGeluF16) {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = gelu_as(v[i]);
              __half* dst = static_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + n;
              store_f16x8(dst, v);
              store_f16x8(dst + 8, v + 8);
            } else {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n);
              if constexpr (EPI == kEpiResidF32) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  float4 x = dst[i];
                  x.x += v[4 * i + 0];
                  x.y += v[4 * i + 1];
                  x.z += v[4 * i + 2];
                  x.w += v[4 * i + 3];
                  dst[i] = x;
                }
              } else {
                if constexpr (EPI == kEpiGeluF32) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) v[i] = gelu_as(v[i]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

template <int BN, int EPI, int DH>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int num_sms,
                       cudaStream_t stream) {
  using S = GemmShape<BN>;
  auto kern = gemm_tc_kernel<BN, EPI, DH>;
  static unsigned long long configured = 0;  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured |= (1ull << dev);
  }
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int grid = tiles < num_sms ? tiles : num_sms;
  if (grid <= 0) return cudaSuccess;
  kern<<<grid, kThreads, S::kSmemBytes, stream>>>(ta, tb, p);
  return cudaGetLastError();
}

template <int BN>
cudaError_t dispatch_epi(const CUtensorMap& ta, const CUtensorMap& tb, int epi, int dh, const GemmParams& p,
                         int num_sms, cudaStream_t s) {
  switch (epi) {
    case kEpiGeluF16: return launch_one<BN, kEpiGeluF16, 0>(ta, tb, p, num_sms, s);
    case kEpiResidF32: return launch_one<BN, kEpiResidF32, 0>(ta, tb, p, num_sms, s);
    case kEpiGeluF32: return launch_one<BN, kEpiGeluF32, 0>(ta, tb, p, num_sms, s);
    case kEpiStoreF32: return launch_one<BN, kEpiStoreF32, 0>(ta, tb, p, num_sms, s);
    case kEpiQkvRope:
      if constexpr (BN % 64 == 0) {
        if (dh == 64) return launch_one<BN, kEpiQkvRope, 64>(ta, tb, p, num_sms, s);
      }
      if constexpr (BN % 32 == 0) {
        if (dh == 32) return launch_one<BN, kEpiQkvRope, 32>(ta, tb, p, num_sms, s);
      }
      if constexpr (BN % 24 == 0) {
        if (dh == 24) return launch_one<BN, kEpiQkvRope, 24>(ta, tb, p, num_sms, s);
      }
      if constexpr (BN % 16 == 0) {
        if (dh == 16) return launch_one<BN, kEpiQkvRope, 16>(ta, tb, p, num_sms, s);
      }
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qres) == cudaSuccess &&
        qres == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  }
  return fn;
}

}  // namespace

bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                   uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows == 0 || box_rows > 256) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int gemm_pick_bn(int N, int head_dim) {
  static const int kCandidates[] = {256, 240, 192, 160, 128};
  for (int bn : kCandidates) {
    if (N % bn) continue;
    if (head_dim > 0 && bn % head_dim) continue;
    return bn;
  }
  return 0;
}

int gemm_pick_bn_any(int N) {
  static const int kCandidates[] = {256, 240, 192, 160, 128, 96, 64, 48, 32, 16};
  for (int bn : kCandidates)
    if (N % bn == 0) return bn;
  return 0;
}

cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, int bn, int epi, int head_dim, GemmParams p,
                        int num_sms, cudaStream_t stream) {
  if (p.M <= 0) return cudaSuccess;
  if (bn <= 0 || p.N % bn || p.K <= 0) return cudaErrorInvalidValue;
  p.num_m_blocks = (p.M + kBM - 1) / kBM;
  p.num_n_blocks = p.N / bn;
  switch (bn) {
    case 256: return dispatch_epi<256>(ta, tb, epi, head_dim, p, num_sms, stream);
    case 240: return dispatch_epi<240>(ta, tb, epi, head_dim, p, num_sms, stream);
    case 192: return dispatch_epi<192>(ta, tb, epi, head_dim, p, num_sms, stream);
    case 160: return dispatch_epi<160>(ta, tb, epi, head_dim, p, num_sms, stream);
    case 128: return dispatch_epi<128>(ta, tb, epi, head_dim, p, num_sms, stream);
    // Narrow tiles serve the plain fp32-output GEMM only (odd output widths of esm_matmul_tiled).
    case 96: return epi == kEpiStoreF32 ? launch_one<96, kEpiStoreF32, 0>(ta, tb, p, num_sms, stream) : cudaErrorInvalidValue;
    case 64: return epi == kEpiStoreF32 ? launch_one<64, kEpiStoreF32, 0>(ta, tb, p, num_sms, stream) : cudaErrorInvalidValue;
    case 48: return epi == kEpiStoreF32 ? launch_one<48, kEpiStoreF32, 0>(ta, tb, p, num_sms, stream) : cudaErrorInvalidValue;
    case 32: return epi == kEpiStoreF32 ? launch_one<32, kEpiStoreF32, 0>(ta, tb, p, num_sms, stream) : cudaErrorInvalidValue;
    case 16: return epi == kEpiStoreF32 ? launch_one<16, kEpiStoreF32, 0>(ta, tb, p, num_sms, stream) : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace esm
