// Persistent, warp-specialised tcgen05 GEMM for sm_100a: C[M,N] = A[M,K] . B[N,K]^T, fp16 operands,
// fp32 accumulation in tensor memory, fused epilogues (bias, RoPE, GELU, residual add).
//
// This replaces codon-infer's row-partitioned CPU GEMMs matmul_tiled_{fp32,q8,q4}_parallel
// (src/lib.rs:4803-4827, 4870-4894, 4937-4961) together with the elementwise passes that follow
// them on the hot path: apply_rope (src/lib.rs:3533-3552), gelu (3494-3498) and the residual
// adds (5325-5327, 5364-5366).
//
// CTA layout (320 threads, one CTA per SM):
//   warp 0      TMA producer: stages 128x64 A tiles and (BN/CG)x64 B tiles (128-byte swizzle) into a
//               ring of shared-memory stages, completion tracked by mbarrier transaction bytes;
//   warp 1      allocates tensor memory and issues tcgen05.mma from one thread, releasing each stage
//               with tcgen05.commit;
//   warps 2..9  epilogue: two warps per 32-lane quarter of the accumulator (tcgen05.ld only reaches
//               the quarter given by warp id mod 4), each taking half of the tile's columns.
// CG = 2 runs the tile on a CTA pair (cluster of 2, tcgen05 cta_group::2): one M = 256 x N = BN MMA
// per K step, each CTA holding 128 rows of A and BN/2 rows of B, so each SM streams half as many
// operand bytes per FLOP. The leader CTA issues the MMAs and counts both CTAs' TMA bytes on its
// barriers; each CTA's epilogue drains its own 128 accumulator rows.
// Two accumulator buffers in tensor memory let the epilogue of tile i overlap the mainloop of
// tile i+1. Every wait is bounded (globaltimer), so a broken pipeline reports an error instead of
// hanging the GPU. No load is multicast.
#include <atomic>
#include <cstdio>

#include "common.cuh"
#include "gemm_tc.cuh"

namespace esm {

namespace {

constexpr int kBK = 64;  // one 128-byte swizzle span of fp16
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kSmemBudget = 224 * 1024;  // operand ring + epilogue staging
constexpr int kStageChunk = 2048;         // one epilogue staging block: 32 rows x 64 bytes

template <int BN, int CG, bool TS>
struct GemmShape {
  static constexpr int kRows = 128;          // accumulator rows per CTA
  static constexpr int kBRows = BN / CG;     // B rows staged per CTA
  static constexpr int kABytes = kRows * kBK * 2;
  static constexpr int kBBytes = kBRows * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // Bulk-store epilogues keep two staging blocks per epilogue warp after the operand ring.
  static constexpr int kStagingBytes = TS ? kEpiWarps * 2 * kStageChunk : 0;
  static constexpr int kRing = kSmemBudget - kStagingBytes;
  static constexpr int kStages = (kRing / kStageBytes) > 8 ? 8 : (kRing / kStageBytes);
  static constexpr int kOffStaging = kStages * kStageBytes;
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;  // TMEM columns between the two accumulators
  static constexpr int kTmemCols = 2 * kAccStride;
  static constexpr int kBarrierBytes = (2 * kStages + 5) * 8 + 16;
  static constexpr int kSmemBytes = kOffStaging + kStagingBytes + kBarrierBytes + 1024;  // +1024 for alignment
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N is a multiple of 16 in [16, 256]");
  static_assert((BN / 2) % 8 == 0, "B half tiles must keep stages 1024-byte aligned");
  static_assert(kStages >= 2, "need at least two stages");
};

__device__ __forceinline__ void store_f16x8(__half* dst, const float* v) {
  __half2 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}

// GELU with the Abramowitz-Stegun erf of the reference, using the fast exp/divide intrinsics
// (relative error ~1e-6, far below the fp16 rounding of the output).
__device__ __forceinline__ float gelu_fast(float x) {
  const float z = x * 0.70710678118654752440f;
  const float az = fabsf(z);
  const float t = __fdividef(1.0f, 1.0f + 0.3275911f * az);
  const float poly = ((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f;
  float y = 1.0f - poly * t * __expf(-az * az);
  y = (z < 0.0f) ? -y : y;
  return 0.5f * x * (1.0f + y);
}

// Epilogue math and store of 16 consecutive accumulator columns [n, n + 16) of row m.
template <int EPI>
__device__ __forceinline__ void epi16(const GemmParams& p, int m, int n, const uint32_t* r) {
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
  if constexpr (EPI == kEpiGeluF16 || EPI == kEpiStoreF16) {
    if constexpr (EPI == kEpiGeluF16) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = gelu_fast(v[i]);
    }
    __half* dst = static_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + n;
    store_f16x8(dst, v);
    store_f16x8(dst + 8, v + 8);
  } else {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n);
    if constexpr (EPI == kEpiGeluF32) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = gelu_fast(v[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
}

// Writes one thread's 64-byte row segment (four 16-byte pieces) into a 32-row staging block laid
// out for a tensor map with 64-byte swizzle: piece c of row r sits at piece c ^ ((r >> 1) & 3).
__device__ __forceinline__ void stage_row64(uint8_t* blk, int r, const uint4* v) {
  const int sw = (r >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(blk + r * 64 + ((c ^ sw) << 4)) = v[c];
}

template <int BN, int EPI, int DH, int CG, bool TS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_out, const GemmParams p) {
  using S = GemmShape<BN, CG, TS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kOffStaging + S::kStagingBytes);
  uint64_t* empty = full + S::kStages;
  uint64_t* acc_full = empty + S::kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const int cluster_id = blockIdx.x / CG;
  const int num_clusters = gridDim.x / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps * CG);  // every epilogue warp of the pair arrives on the leader
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, S::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, S::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) {
    cluster_sync();  // barrier inits and the TMEM allocation are visible to the peer
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int num_kb = (p.K + kBK - 1) / kBK;

  if (warp == 0) {
    // ---------------- TMA producer (each CTA loads its own A rows and B half) ----------------
    if (elect_one_sync()) {
      const uint64_t pol_a = l2_policy_evict_normal();
      const uint64_t pol_b = l2_policy_evict_last();  // weights are re-read by every m-block
      int stage = 0;
      uint32_t phase = 0;
      int fills = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters) {
        const int m_blk = tile / p.num_n_blocks;
        const int n_blk = tile - m_blk * p.num_n_blocks;
        const int a_row = m_blk * (128 * CG) + 128 * static_cast<int>(rank);
        const int b_row = n_blk * BN + S::kBRows * static_cast<int>(rank);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          if constexpr (CG == 2) {
            // The leader's own arrive needs no cluster-scope release: the peer's bytes reach this
            // barrier through its TMA's complete_tx, and a per-stage cluster fence in this single
            // producer thread would throttle the whole pipeline.
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
            const uint32_t leader_full = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(sa, &tmap_a, leader_full, kb * kBK, a_row, pol_a);
            tma_load_2d_pair(sb, &tmap_b, leader_full, kb * kBK, b_row, pol_b);
          } else {
            mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
            tma_load_2d(sa, &tmap_a, &full[stage], kb * kBK, a_row, pol_a);
            // B arrives as two half tiles (the tensor map's box is BN/2 rows).
            tma_load_2d(sb, &tmap_b, &full[stage], kb * kBK, b_row, pol_b);
            tma_load_2d(sb + S::kBBytes / 2, &tmap_b, &full[stage], kb * kBK, b_row + BN / 2, pol_b);
          }
          ++fills;
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && (CG == 1 || rank == 0)) {
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
    // ---------------- MMA issuer (the leader CTA of a pair) ----------------
    if ((CG == 1 || rank == 0) && elect_one_sync()) {
      constexpr uint32_t idesc = umma_idesc_f16(128 * CG, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters, ++local) {
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
            const uint64_t ad = umma_sdesc_sw128(a_addr + k * 32);
            const uint64_t bd = umma_sdesc_sw128(b_addr + k * 32);
            if constexpr (CG == 2) {
              umma_f16_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            } else {
              umma_f16(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          if constexpr (CG == 2) {
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            umma_commit(&empty[stage]);
          }
          if (++stage == S::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (CG == 2) {
          umma_commit_pair(mapa_shared(smem_u32(&acc_full[buf]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&acc_full[buf]), 1));
        } else {
          umma_commit(&acc_full[buf]);
        }
      }
      if (!ok) {
        // Wait (bounded) for every MMA this thread issued before tensor memory is released.
        if constexpr (CG == 2) {
          umma_commit_pair(mapa_shared(smem_u32(drain), 0));
        } else {
          umma_commit(drain);
        }
        mbar_wait(drain, 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    const int quarter = warp & 3;             // TMEM lanes [32*quarter, 32*quarter + 32)
    const int half = (warp - 2) >> 2;         // which half of the tile's columns
    constexpr int kChunk = (EPI == kEpiQkvRope) ? DH : 16;
    constexpr int kSplit = ((BN / 2) / kChunk) * kChunk;
    const int c_begin = half ? kSplit : 0;
    const int c_end = half ? BN : kSplit;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t leader_acc_empty0 =
        (CG == 2) ? mapa_shared(smem_u32(&acc_empty[0]), 0) : smem_u32(&acc_empty[0]);
    int local = 0;
    int sbuf = 0;  // staging block of the next bulk store (bulk-store epilogues)
    (void)sbuf;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters, ++local) {
      const int m_blk = tile / p.num_n_blocks;
      const int n_blk = tile - m_blk * p.num_n_blocks;
      const int buf = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[buf], acc_phase, p.err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int m = m_blk * (128 * CG) + 128 * static_cast<int>(rank) + row_in_tile;
      const bool row_ok = m < p.M;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(buf * S::kAccStride);
      const int n0 = n_blk * BN;

      if constexpr (TS) {
        // Bulk-store epilogue: each warp writes 32-row x 64-byte blocks of its rows into a
        // swizzled staging block and one lane stores (or, for the residual, reduce-adds) the block
        // with the tensor map. Rows past M are clipped by the map.
        uint8_t* stg = smem + S::kOffStaging + (warp - 2) * (2 * kStageChunk);
        const int row0 = m_blk * (128 * CG) + 128 * static_cast<int>(rank) + quarter * 32;
        if constexpr (EPI == kEpiQkvRope) {
          constexpr int HALF = DH / 2;  // 32 or 16
          const int pos = row_ok ? __ldg(p.pos + m) : 0;
          float4 cs_all[HALF / 2];
          if (n0 + c_begin < p.rope_cols) {
            const float4* cs_row = reinterpret_cast<const float4*>(p.rope + static_cast<size_t>(pos) * HALF);
#pragma unroll
            for (int i = 0; i < HALF / 2; ++i) cs_all[i] = __ldg(cs_row + i);
          }
#pragma unroll 1
          for (int c = c_begin; c < c_end; c += DH) {
            const int n = n0 + c;
            if (lane == 0) bulk_wait_read<0>();  // both staging blocks are free again
            __syncwarp();
            if (n < p.rope_cols) {
              // DH 64: block 0 = rotated first half (columns [0, 32)), block 1 = second half.
              // DH 32: one block, the 16 first-half columns then the 16 second-half columns.
#pragma unroll
              for (int sub = 0; sub < HALF; sub += 16) {
                float4 b0[4], b1[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  b0[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n + sub) + i);
                  b1[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n + HALF + sub) + i);
                }
                const float4* cs = cs_all + sub / 2;
                uint32_t r0[16], r1[16];
                tmem_ld16(t_row + c + sub, r0);
                tmem_ld16(t_row + c + HALF + sub, r1);
                tmem_ld_wait();
                const float* bb0 = reinterpret_cast<const float*>(b0);
                const float* bb1 = reinterpret_cast<const float*>(b1);
                const float* cc = reinterpret_cast<const float*>(cs);
                __half2 h0[8], h1[8];
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                  const float x0a = __uint_as_float(r0[j]) + bb0[j], x0b = __uint_as_float(r0[j + 1]) + bb0[j + 1];
                  const float x1a = __uint_as_float(r1[j]) + bb1[j], x1b = __uint_as_float(r1[j + 1]) + bb1[j + 1];
                  h0[j / 2] = __floats2half2_rn(x0a * cc[2 * j] - x1a * cc[2 * j + 1],
                                                x0b * cc[2 * j + 2] - x1b * cc[2 * j + 3]);
                  h1[j / 2] = __floats2half2_rn(x1a * cc[2 * j] + x0a * cc[2 * j + 1],
                                                x1b * cc[2 * j + 2] + x0b * cc[2 * j + 3]);
                }
                const uint4* u0 = reinterpret_cast<const uint4*>(h0);
                const uint4* u1 = reinterpret_cast<const uint4*>(h1);
                const int sw = (lane >> 1) & 3;
                if constexpr (DH == 64) {
                  const int pc = sub / 8;  // 16 columns = two 16-byte pieces
#pragma unroll
                  for (int q = 0; q < 2; ++q) {
                    *reinterpret_cast<uint4*>(stg + lane * 64 + (((pc + q) ^ sw) << 4)) = u0[q];
                    *reinterpret_cast<uint4*>(stg + kStageChunk + lane * 64 + (((pc + q) ^ sw) << 4)) = u1[q];
                  }
                } else {
#pragma unroll
                  for (int q = 0; q < 2; ++q) {
                    *reinterpret_cast<uint4*>(stg + lane * 64 + ((q ^ sw) << 4)) = u0[q];
                    *reinterpret_cast<uint4*>(stg + lane * 64 + (((2 + q) ^ sw) << 4)) = u1[q];
                  }
                }
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmap_out, stg, n, row0);
                if constexpr (DH == 64) tma_store_2d(&tmap_out, stg + kStageChunk, n + 32, row0);
                bulk_commit();
              }
            } else {
              // V columns: acc + bias in fp16, 32 columns per staging block.
#pragma unroll
              for (int cc = 0; cc < DH; cc += 32) {
                uint8_t* blk = stg + (cc / 32) * kStageChunk;
                uint32_t r[16], r2[16];
                tmem_ld16(t_row + c + cc, r);
                tmem_ld16(t_row + c + cc + 16, r2);
                tmem_ld_wait();
                __half2 hv[16];
#pragma unroll
                for (int j = 0; j < 16; j += 2) {
                  hv[j / 2] = __floats2half2_rn(__uint_as_float(r[j]) + __ldg(p.bias + n + cc + j),
                                                __uint_as_float(r[j + 1]) + __ldg(p.bias + n + cc + j + 1));
                  hv[8 + j / 2] = __floats2half2_rn(__uint_as_float(r2[j]) + __ldg(p.bias + n + cc + 16 + j),
                                                    __uint_as_float(r2[j + 1]) + __ldg(p.bias + n + cc + 17 + j));
                }
                stage_row64(blk, lane, reinterpret_cast<const uint4*>(hv));
              }
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
#pragma unroll
                for (int cc = 0; cc < DH; cc += 32) tma_store_2d(&tmap_out, stg + (cc / 32) * kStageChunk, n + cc, row0);
                bulk_commit();
              }
            }
          }
        } else if constexpr (EPI == kEpiGeluF16) {
#pragma unroll 1
          for (int c = c_begin; c < c_end; c += 32) {
            uint8_t* blk = stg + sbuf * kStageChunk;
            float4 b[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) b[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n0 + c) + i);
            uint32_t r[32];
            tmem_ld16(t_row + c, *reinterpret_cast<uint32_t(*)[16]>(r));
            tmem_ld16(t_row + c + 16, *reinterpret_cast<uint32_t(*)[16]>(r + 16));
            if (lane == 0) bulk_wait_read<1>();  // the store that last used this block has read it
            tmem_ld_wait();
            const float* bb = reinterpret_cast<const float*>(b);
            __half2 hv[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2)
              hv[j / 2] = __floats2half2_rn(gelu_fast(__uint_as_float(r[j]) + bb[j]),
                                            gelu_fast(__uint_as_float(r[j + 1]) + bb[j + 1]));
            __syncwarp();
            stage_row64(blk, lane, reinterpret_cast<const uint4*>(hv));
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_out, blk, n0 + c, row0);
              bulk_commit();
            }
            sbuf ^= 1;
          }
        } else if constexpr (EPI == kEpiResidF32) {
#pragma unroll 1
          for (int c = c_begin; c < c_end; c += 16) {
            uint8_t* blk = stg + sbuf * kStageChunk;
            float4 b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              b[i] = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + n0 + c) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            uint32_t r[16];
            tmem_ld16(t_row + c, r);
            if (lane == 0) bulk_wait_read<1>();
            tmem_ld_wait();
            float4 v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              v[i] = make_float4(__uint_as_float(r[4 * i + 0]) + b[i].x, __uint_as_float(r[4 * i + 1]) + b[i].y,
                                 __uint_as_float(r[4 * i + 2]) + b[i].z, __uint_as_float(r[4 * i + 3]) + b[i].w);
            __syncwarp();
            stage_row64(blk, lane, reinterpret_cast<const uint4*>(v));
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_reduce_add_2d(&tmap_out, blk, n0 + c, row0);
              bulk_commit();
            }
            sbuf ^= 1;
          }
        }
      } else       if constexpr (EPI == kEpiQkvRope && (DH / 2) % 16 == 0) {
        // head_dim 32 / 64: rotate 16 (j, j + DH/2) pairs per step; the bias and cos/sin rows are
        // requested (float4) before the tensor-memory wait so their latency overlaps it.
        constexpr int HALF = DH / 2;
        const int pos = row_ok ? __ldg(p.pos + m) : 0;
        __half* dst_row = static_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo;
        // The (cos, sin) row of this thread's position is the same for every head: load it once.
        float4 cs_all[HALF / 2];
        if (row_ok && n0 + c_begin < p.rope_cols) {
          const float4* cs_row = reinterpret_cast<const float4*>(p.rope + static_cast<size_t>(pos) * HALF);
#pragma unroll
          for (int i = 0; i < HALF / 2; ++i) cs_all[i] = __ldg(cs_row + i);
        }
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += DH) {
          const int n = n0 + c;
          if (n < p.rope_cols) {
#pragma unroll
            for (int sub = 0; sub < HALF; sub += 16) {
              float4 b0[4], b1[4];
              if (row_ok) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  b0[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n + sub) + i);
                  b1[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n + HALF + sub) + i);
                }
              }
              const float4* cs = cs_all + sub / 2;
              uint32_t r0[16], r1[16];
              tmem_ld16(t_row + c + sub, r0);
              tmem_ld16(t_row + c + HALF + sub, r1);
              tmem_ld_wait();
              if (row_ok) {
                const float* bb0 = reinterpret_cast<const float*>(b0);
                const float* bb1 = reinterpret_cast<const float*>(b1);
                const float* cc = reinterpret_cast<const float*>(cs);  // (cos, sin) pairs
                float y0[16], y1[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const float x0 = __uint_as_float(r0[j]) + bb0[j];
                  const float x1 = __uint_as_float(r1[j]) + bb1[j];
                  y0[j] = x0 * cc[2 * j] - x1 * cc[2 * j + 1];
                  y1[j] = x1 * cc[2 * j] + x0 * cc[2 * j + 1];
                }
                store_f16x8(dst_row + n + sub, y0);
                store_f16x8(dst_row + n + sub + 8, y0 + 8);
                store_f16x8(dst_row + n + HALF + sub, y1);
                store_f16x8(dst_row + n + HALF + sub + 8, y1 + 8);
              }
            }
          } else {
#pragma unroll
            for (int sub = 0; sub < DH; sub += 16) {
              uint32_t r[16];
              tmem_ld16(t_row + c + sub, r);
              tmem_ld_wait();
              if (row_ok) epi16<kEpiStoreF16>(p, m, n + sub, r);
            }
          }
        }
      } else if constexpr (EPI == kEpiQkvRope) {
        constexpr int HALF = DH / 2;
        const int pos = row_ok ? __ldg(p.pos + m) : 0;
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += DH) {
          uint32_t r[DH];
#pragma unroll
          for (int i = 0; i < DH / 8; ++i) tmem_ld8(t_row + c + 8 * i, r + 8 * i);
          tmem_ld_wait();
          if (row_ok) {
            const int n = n0 + c;
            // Bias and (cos, sin) rows as float4: n * 4 and pos * HALF * 8 bytes are multiples of
            // 16 for head_dim 16 and 24.
            float v[DH];
            if (p.bias) {
              float4 b4[DH / 4];
#pragma unroll
              for (int i = 0; i < DH / 4; ++i) b4[i] = __ldg(reinterpret_cast<const float4*>(p.bias + n) + i);
              const float* bb = reinterpret_cast<const float*>(b4);
#pragma unroll
              for (int i = 0; i < DH; ++i) v[i] = __uint_as_float(r[i]) + bb[i];
            } else {
#pragma unroll
              for (int i = 0; i < DH; ++i) v[i] = __uint_as_float(r[i]);
            }
            if (n < p.rope_cols) {
              float4 cs4[HALF / 2];
              const float4* tab = reinterpret_cast<const float4*>(p.rope + static_cast<size_t>(pos) * HALF);
#pragma unroll
              for (int i = 0; i < HALF / 2; ++i) cs4[i] = __ldg(tab + i);
              const float* cc = reinterpret_cast<const float*>(cs4);  // (cos, sin) pairs
#pragma unroll
              for (int j = 0; j < HALF; ++j) {
                const float x0 = v[j], x1 = v[j + HALF];
                v[j] = x0 * cc[2 * j] - x1 * cc[2 * j + 1];
                v[j + HALF] = x1 * cc[2 * j] + x0 * cc[2 * j + 1];
              }
            }
            __half* dst = static_cast<__half*>(p.out) + static_cast<size_t>(m) * p.ldo + n;
#pragma unroll
            for (int i = 0; i < DH / 8; ++i) store_f16x8(dst + 8 * i, v + 8 * i);
            if (p.lo && n < p.rope_cols) {
              // Queries and keys also keep what fp16 rounding dropped, so that attention can form
              // its scores as q_hi k_hi + q_lo k_hi + q_hi k_lo, close to the fp32 product.
#pragma unroll
              for (int i = 0; i < DH; ++i) v[i] -= __half2float(__float2half_rn(v[i]));
              __half* lo = p.lo + static_cast<size_t>(m) * p.lo_ld + n;
#pragma unroll
              for (int i = 0; i < DH / 8; ++i) store_f16x8(lo + 8 * i, v + 8 * i);
            }
          }
        }
      } else if constexpr (EPI == kEpiResidF32) {
        // x += acc + bias as vector reductions performed in L2: the residual stream is never
        // read into the SM, so the epilogue issues its stores without waiting on loads.
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 16) {
          float4 b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            b[i] = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + n0 + c) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          uint32_t r[16];
          tmem_ld16(t_row + c, r);
          tmem_ld_wait();
          if (row_ok) {
            float* dst = static_cast<float*>(p.out) + static_cast<size_t>(m) * p.ldo + n0 + c;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              red_add_f32x4(dst + 4 * i, make_float4(__uint_as_float(r[4 * i + 0]) + b[i].x,
                                                      __uint_as_float(r[4 * i + 1]) + b[i].y,
                                                      __uint_as_float(r[4 * i + 2]) + b[i].z,
                                                      __uint_as_float(r[4 * i + 3]) + b[i].w));
          }
        }
      } else {
        int c = c_begin;
#pragma unroll 1
        for (; c + 32 <= c_end; c += 32) {
          uint32_t r[16], r2[16];
          tmem_ld16(t_row + c, r);
          tmem_ld16(t_row + c + 16, r2);
          tmem_ld_wait();
          if (row_ok) {
            epi16<EPI>(p, m, n0 + c, r);
            epi16<EPI>(p, m, n0 + c + 16, r2);
          }
        }
        if (c < c_end) {
          uint32_t r[16];
          tmem_ld16(t_row + c, r);
          tmem_ld_wait();
          if (row_ok) epi16<EPI>(p, m, n0 + c, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2) {
          mbar_arrive_cluster(leader_acc_empty0 + static_cast<uint32_t>(buf * sizeof(uint64_t)));
        } else {
          mbar_arrive(&acc_empty[buf]);
        }
      }
    }
    // Bulk stores still in flight complete before the CTA leaves.
    if constexpr (TS) {
      if (lane == 0) bulk_wait_all();
    }
  }

  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer no longer reads this CTA's smem or barriers
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2) {
      tmem_dealloc_pair(tmem_base, S::kTmemCols);
    } else {
      tmem_dealloc(tmem_base, S::kTmemCols);
    }
  }
}

template <int BN, int EPI, int DH, int CG, bool TS>
cudaError_t launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tout, const GemmParams& p,
                       int num_sms, cudaStream_t stream) {
  using S = GemmShape<BN, CG, TS>;
  auto kern = gemm_tc_kernel<BN, EPI, DH, CG, TS>;
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = S::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Tiles are split statically over the persistent CTAs, so every cluster must be resident at
  // once: a cluster of two needs two free SMs in one GPC, and the count of clusters that fit at the
  // same time can be below num_sms / 2.
  static std::atomic<int> resident[64] = {};
  int max_clusters = num_sms / CG;
  if (CG > 1 && dev < 64) {
    int n = resident[dev].load(std::memory_order_relaxed);
    if (n == 0) {
      cfg.gridDim = dim3(max_clusters * CG, 1, 1);
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = max_clusters;
      resident[dev].store(n, std::memory_order_relaxed);
    }
    max_clusters = n < max_clusters ? n : max_clusters;
  }
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int clusters = tiles < max_clusters ? tiles : max_clusters;
  if (clusters <= 0) return cudaSuccess;
  cfg.gridDim = dim3(clusters * CG, 1, 1);
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, tout, p);
}

// Plain epilogues (no output tensor map) and the bulk-store ones where the output map is given,
// the tile splits into whole 32-column blocks per epilogue warp, and the epilogue has a staged form.
template <int BN, int EPI, int DH, int CG>
cudaError_t launch_ts(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, const GemmParams& p,
                      int num_sms, cudaStream_t s) {
  constexpr bool kStaged = BN % 64 == 0 && (EPI == kEpiGeluF16 || EPI == kEpiResidF32 ||
                                            (EPI == kEpiQkvRope && (DH == 64 || DH == 32)));
  if constexpr (kStaged) {
    if (tout != nullptr) return launch_one<BN, EPI, DH, CG, true>(ta, tb, *tout, p, num_sms, s);
  }
  return launch_one<BN, EPI, DH, CG, false>(ta, tb, tout ? *tout : ta, p, num_sms, s);
}

template <int BN, int CG>
cudaError_t dispatch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, int epi, int dh,
                         const GemmParams& p, int num_sms, cudaStream_t s) {
  switch (epi) {
    case kEpiGeluF16: return launch_ts<BN, kEpiGeluF16, 0, CG>(ta, tb, tout, p, num_sms, s);
    case kEpiResidF32: return launch_ts<BN, kEpiResidF32, 0, CG>(ta, tb, tout, p, num_sms, s);
    case kEpiGeluF32: return launch_one<BN, kEpiGeluF32, 0, CG, false>(ta, tb, ta, p, num_sms, s);
    case kEpiStoreF32: return launch_one<BN, kEpiStoreF32, 0, CG, false>(ta, tb, ta, p, num_sms, s);
    case kEpiQkvRope:
      if constexpr (BN % 64 == 0) {
        if (dh == 64) return launch_ts<BN, kEpiQkvRope, 64, CG>(ta, tb, tout, p, num_sms, s);
      }
      if constexpr (BN % 32 == 0) {
        if (dh == 32) return launch_ts<BN, kEpiQkvRope, 32, CG>(ta, tb, tout, p, num_sms, s);
      }
      if constexpr (BN % 24 == 0) {
        if (dh == 24) return launch_one<BN, kEpiQkvRope, 24, CG, false>(ta, tb, ta, p, num_sms, s);
      }
      if constexpr (BN % 16 == 0) {
        if (dh == 16) return launch_one<BN, kEpiQkvRope, 16, CG, false>(ta, tb, ta, p, num_sms, s);
      }
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

template <int BN>
cudaError_t dispatch_cg(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, int epi, int dh, int cg,
                        const GemmParams& p, int num_sms, cudaStream_t s) {
  return cg == 2 ? dispatch_epi<BN, 2>(ta, tb, tout, epi, dh, p, num_sms, s)
                 : dispatch_epi<BN, 1>(ta, tb, tout, epi, dh, p, num_sms, s);
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

bool make_tmap_f16_box(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                       uint32_t box_rows, uint32_t box_cols, int swizzle_bytes) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr || (swizzle_bytes != 64 && swizzle_bytes != 128)) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows == 0 || box_rows > 256 ||
      box_cols * 2 != static_cast<uint32_t>(swizzle_bytes))
    return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_f16_heads(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads, uint32_t head_dim,
                         uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr || head_dim == 0 || head_dim > 32 || ((head_dim * 2) & 15)) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || box_rows == 0 || box_rows > 256) return false;
  // [rows][heads][head_dim] with a box 32 elements wide: columns head_dim..31 of every row are
  // outside the tensor and arrive as zeros.
  const cuuint64_t dims[3] = {head_dim, heads, rows};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * 2, ld * 2};
  const cuuint32_t box[3] = {32, 1, box_rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_out(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols, uint64_t ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (enc == nullptr || (elem_bytes != 2 && elem_bytes != 4)) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * elem_bytes) & 15) || rows == 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(64 / elem_bytes), 32};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int gemm_pick_bn(int N, int head_dim) {
  // Widths that are multiples of 64 first: their epilogue warps split the tile into whole
  // 32-column blocks, which the bulk-store epilogues need.
  static const int kCandidates[] = {256, 192, 128, 240, 160};
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

cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, int bn, int epi,
                        int head_dim, GemmParams p, int num_sms, cudaStream_t stream, int cta_pair) {
  if (p.M <= 0) return cudaSuccess;
  if (bn <= 0 || p.N % bn || p.K <= 0) return cudaErrorInvalidValue;
  // The CTA pair needs the wide tiles and at least two 128-row blocks of work.
  const int cg = (cta_pair && bn >= 128 && p.M > 128) ? 2 : 1;
  p.num_m_blocks = (p.M + 128 * cg - 1) / (128 * cg);
  p.num_n_blocks = p.N / bn;
  switch (bn) {
    case 256: return dispatch_cg<256>(ta, tb, tout, epi, head_dim, cg, p, num_sms, stream);
    case 240: return dispatch_cg<240>(ta, tb, tout, epi, head_dim, cg, p, num_sms, stream);
    case 192: return dispatch_cg<192>(ta, tb, tout, epi, head_dim, cg, p, num_sms, stream);
    case 160: return dispatch_cg<160>(ta, tb, tout, epi, head_dim, cg, p, num_sms, stream);
    case 128: return dispatch_cg<128>(ta, tb, tout, epi, head_dim, cg, p, num_sms, stream);
    // Narrow tiles serve the plain fp32-output GEMM only (odd output widths of esm_matmul_tiled).
    case 96:
      return epi == kEpiStoreF32 ? launch_one<96, kEpiStoreF32, 0, 1, false>(ta, tb, ta, p, num_sms, stream)
                               : cudaErrorInvalidValue;
    case 64:
      return epi == kEpiStoreF32 ? launch_one<64, kEpiStoreF32, 0, 1, false>(ta, tb, ta, p, num_sms, stream)
                               : cudaErrorInvalidValue;
    case 48:
      return epi == kEpiStoreF32 ? launch_one<48, kEpiStoreF32, 0, 1, false>(ta, tb, ta, p, num_sms, stream)
                               : cudaErrorInvalidValue;
    case 32:
      return epi == kEpiStoreF32 ? launch_one<32, kEpiStoreF32, 0, 1, false>(ta, tb, ta, p, num_sms, stream)
                               : cudaErrorInvalidValue;
    case 16:
      return epi == kEpiStoreF32 ? launch_one<16, kEpiStoreF32, 0, 1, false>(ta, tb, ta, p, num_sms, stream)
                               : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace esm
