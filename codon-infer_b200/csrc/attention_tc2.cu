// Bidirectional attention on tcgen05 for head_dim 64 and 32, two query tiles per CTA. Same contract as
// attention_kernel in attention.cu (packed varlen sequences, keys past a sequence's end masked, O in
// fp16, optional per-row log-sum-exp); replaces the reference attention loop (src/lib.rs:5206-5301).
//
// One CTA per (sequence, 256-query block, head); 320 threads; two CTAs per SM.
//   warps 0..3  softmax of query tile 0 (rows 0..127 of the block), one row per thread
//   warps 4..7  softmax of query tile 1 (rows 128..255)
//   warp 8      TMA producer: both Q tiles once, then 64-key K and V tiles into a 4-stage ring
//   warp 9      tcgen05.mma issuer
// The two query tiles share every K/V tile. Tensor memory (256 columns): S_t in [64 t, 64 t + 64),
// O_t in [128 + DH t, 128 + DH (t + 1)). Head_dim 64 tiles use 128-byte rows with the 128-byte
// swizzle, head_dim 32 tiles 64-byte rows with the 64-byte swizzle. The softmax writes P_t (fp16, two per column) over the first 32
// columns of S_t and O_t += P_t V is issued with A read from tensor memory, so P never touches
// shared memory. MMAs of one thread run in issue order, which orders every reuse of S_t:
//   S0_0 S1_0 | PV0_0 S0_1 | PV1_0 S1_1 | PV0_1 S0_2 | ...
// so the next S of a tile starts as soon as its P has been written, while the other tile's
// softmax runs. O is rescaled in tensor memory only when a row max grows past the threshold.
// All waits are bounded.
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kQ = 128;   // rows per query tile
constexpr int kKV = 64;   // keys per K/V tile
constexpr int kThreads2 = 320;
constexpr int kStages2 = 4;

// Tile geometry for head_dim DH (64: 128-byte rows, 128-byte swizzle; 32: 64-byte rows and swizzle).
template <int DH>
struct Tc2 {
  static constexpr int kQBytes = kQ * DH * 2;    // one query tile
  static constexpr int kKVBytes = kKV * DH * 2;  // one K or V tile
  static constexpr int kOffKV = 2 * kQBytes;
  static constexpr int kOffBar = kOffKV + kStages2 * 2 * kKVBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;
  static constexpr int kVStep = 16 * DH * 2;     // 16 keys of V
  __device__ static uint64_t kdesc(uint32_t a) { return DH == 64 ? umma_sdesc_sw128(a) : umma_sdesc_sw64(a); }
  __device__ static uint64_t vdesc(uint32_t a) { return DH == 64 ? umma_sdesc_sw128_mn(a) : umma_sdesc_sw64_mn(a); }
};
constexpr uint32_t kTmemCols2 = 256;
constexpr float kLog2e = 1.4426950408889634f;
// The running max used for P is refreshed only when a row's max grows by more than 2^8 (in the
// exp2 domain); until then P <= 256, exact in fp16's relative precision, and O and l share the
// stale max, so O / l and the log-sum-exp are unchanged.
constexpr float kRescaleThreshold = 8.0f;

// S_t = Q_t K_j^T into S_t's tensor-memory columns, then signal `bar`.
template <int DH>
__device__ __forceinline__ void issue_s(uint32_t tmem, uint32_t q_addr, uint32_t kv_addr, int t, int j, uint64_t* bar) {
  using G = Tc2<DH>;
  constexpr uint32_t idesc_qk = umma_idesc_f16(kQ, kKV);
  const uint32_t k_addr = kv_addr + (j % kStages2) * 2 * G::kKVBytes;
#pragma unroll
  for (int k = 0; k < DH / 16; ++k)
    umma_f16(tmem + t * kKV, G::kdesc(q_addr + t * G::kQBytes + k * 32), G::kdesc(k_addr + k * 32), idesc_qk, k > 0);
  umma_commit(bar);
}

// O_t += P_t V_j with P_t (64 keys = 32 columns of fp16 pairs) read from tensor memory.
template <int DH>
__device__ __forceinline__ void issue_pv(uint32_t tmem, uint32_t kv_addr, int t, int j, uint64_t* bar) {
  using G = Tc2<DH>;
  constexpr uint32_t idesc_pv = umma_idesc_f16(kQ, DH) | (1u << 16);  // B (V) is MN-major
  const uint32_t v_addr = kv_addr + (j % kStages2) * 2 * G::kKVBytes + G::kKVBytes;
#pragma unroll
  for (int k = 0; k < kKV / 16; ++k)
    umma_f16_ts(tmem + 128 + t * DH, tmem + t * kKV + k * 8, G::vdesc(v_addr + k * G::kVStep), idesc_pv,
                (j > 0 || k > 0) ? 1u : 0u);
  umma_commit(bar);
}

// POLY of every 8 column pairs take their exponentials on the FP32 pipe (poly_exp2) instead of the
// special-function unit, which is the bottleneck of the softmax at head_dim 64.
template <int DH, int POLY>
__global__ void __launch_bounds__(kThreads2, 2)
    attention_tc2_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_kv,
                         const AttnParams p) {
  using G = Tc2<DH>;
  constexpr int kQBytes = G::kQBytes, kKVBytes = G::kKVBytes, kOffKV = G::kOffKV, kOffBar = G::kOffBar;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                // [4]
  uint64_t* kv_empty = bars + 1 + kStages2;    // [4]
  uint64_t* s_full = bars + 1 + 2 * kStages2;  // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* o_full = p_full + 2;               // [2]
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int2 wk = p.work[blockIdx.x];
  const int b = wk.x, q0 = wk.y * (2 * kQ), h = blockIdx.y;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int nkv = (len + kKV - 1) / kKV;
  const bool has1 = q0 + kQ < len;  // the second query tile holds rows of this sequence

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols2);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------- TMA producer ----------------
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_kv);
      const uint64_t pol = l2_policy_evict_normal();
      mbar_arrive_expect_tx(q_full, has1 ? 2 * kQBytes : kQBytes);
      tma_load_2d(smem, &tmap_q, q_full, h * DH, start + q0, pol);
      if (has1) tma_load_2d(smem + kQBytes, &tmap_q, q_full, h * DH, start + q0 + kQ, pol);
      bool ok = true;
      int j = 0;
      for (; j < nkv; ++j) {
        const int st = j % kStages2;
        if (!mbar_wait(&kv_empty[st], ((j / kStages2) & 1) ^ 1u, p.err, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* dst = smem + kOffKV + st * 2 * kKVBytes;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKVBytes);
        tma_load_2d(dst, &tmap_kv, &kv_full[st], p.d + h * DH, start + j * kKV, pol);
        tma_load_2d(dst + kKVBytes, &tmap_kv, &kv_full[st], 2 * p.d + h * DH, start + j * kKV, pol);
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        mbar_wait(q_full, 0, p.err, kDevTimeoutProducer);
        for (int jj = (j - kStages2 > 0 ? j - kStages2 : 0); jj < j; ++jj)
          mbar_wait(&kv_full[jj % kStages2], (jj / kStages2) & 1, p.err, kDevTimeoutProducer);
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (elect_one_sync()) {
      const uint32_t q_addr = smem_u32(smem);
      const uint32_t kv_addr = smem_u32(smem + kOffKV);
      bool ok = mbar_wait_spin(q_full, 0, p.err, kDevTimeoutMma);
      if (ok && mbar_wait_spin(&kv_full[0], 0, p.err, kDevTimeoutMma)) {
        tc_fence_after();
        issue_s<DH>(tmem, q_addr, kv_addr, 0, 0, &s_full[0]);
        if (has1) issue_s<DH>(tmem, q_addr, kv_addr, 1, 0, &s_full[1]);
      } else {
        ok = false;
      }
      for (int j = 0; j < nkv && ok; ++j) {
        if (!mbar_wait_spin(&p_full[0], j & 1, p.err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        issue_pv<DH>(tmem, kv_addr, 0, j, &o_full[0]);
        const bool next = j + 1 < nkv;
        if (next) {
          if (!mbar_wait_spin(&kv_full[(j + 1) % kStages2], ((j + 1) / kStages2) & 1, p.err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s<DH>(tmem, q_addr, kv_addr, 0, j + 1, &s_full[0]);
        }
        if (has1) {
          if (!mbar_wait_spin(&p_full[1], j & 1, p.err, kDevTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          issue_pv<DH>(tmem, kv_addr, 1, j, &o_full[1]);
        }
        umma_commit(&kv_empty[j % kStages2]);
        if (has1 && next) issue_s<DH>(tmem, q_addr, kv_addr, 1, j + 1, &s_full[1]);
      }
      if (!ok) {
        umma_commit(drain);
        mbar_wait_spin(drain, 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- softmax: thread = query row of tile t ----------------
    const int t = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row inside the tile = TMEM lane
    if (t == 0 || has1) {
      const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t t_s = tmem + lane_off + t * kKV;
      const uint32_t t_o = tmem + lane_off + 128 + t * DH;
      const float c = p.scale * kLog2e;
      float mc = -INFINITY;  // running max in the exp2 domain (max score * c)
      float l = 0.0f;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        if (!mbar_wait_spin(&s_full[t], j & 1, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
        const int kvalid = len - j * kKV;  // keys of this tile inside the sequence (> 0)
        // Pass 1: row max, 32 columns at a time (only the last tile needs the key mask).
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t sv[32];
          tmem_ld32(t_s + hh * 32, sv);
          tmem_ld_wait();
          if (kvalid < kKV) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (hh * 32 + i >= kvalid) sv[i] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(sv[i]));
        }
        const float mraw =
            fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        const float mx = mraw * c;
        if (j == 0) {
          mc = mx;
        } else if (__any_sync(0xffffffffu, mx - mc > kRescaleThreshold)) {
          // Refresh the max of this warp's rows once the previous O += P V has landed.
          const float m_new = fmaxf(mc, mx);
          const float alpha = fast_exp2(mc - m_new);
          if (!mbar_wait_spin(&o_full[t], (j - 1) & 1, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < DH / 32; ++hh) {
            uint32_t o[32];
            tmem_ld32(t_o + hh * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(t_o + hh * 32, o);
          }
          tmem_st_wait();
          l *= alpha;
          mc = m_new;
        }
        // P = exp2(S c - m) as fp16 pairs over the first 32 columns of S.
        float rs[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          // Pass 2: S columns [32 hh, 32 hh + 32) -> P columns [16 hh, 16 hh + 16), which hold
          // scores this loop has already read.
          uint32_t sv[32];
          tmem_ld32(t_s + hh * 32, sv);
          tmem_ld_wait();
          if (kvalid < kKV) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (hh * 32 + i >= kvalid) sv[i] = __float_as_uint(-INFINITY);
          }
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = fmaf(__uint_as_float(sv[2 * i]), c, -mc);
            const float a1 = fmaf(__uint_as_float(sv[2 * i + 1]), c, -mc);
            const bool poly = (i & 7) < POLY;
            const float e0 = poly ? poly_exp2(a0) : fast_exp2(a0);
            const float e1 = poly ? poly_exp2(a1) : fast_exp2(a1);
            rs[(2 * i) & 7] += e0;
            rs[(2 * i + 1) & 7] += e1;
            __half2 hv = __floats2half2_rn(e0, e1);
            pk[i] = *reinterpret_cast<uint32_t*>(&hv);
          }
          tmem_st16(t_s + hh * 16, pk);
        }
        l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (ok && mbar_wait_spin(&o_full[t], (nkv - 1) & 1, p.err, kDevTimeoutEpilogue)) {
        tc_fence_after();
        const int row = q0 + t * kQ + r;
        const float inv = 1.0f / l;
        __half* dst = p.out + static_cast<size_t>(start + row) * p.d + h * DH;
#pragma unroll
        for (int hh = 0; hh < DH / 32; ++hh) {
          uint32_t o[32];
          tmem_ld32(t_o + hh * 32, o);
          tmem_ld_wait();
          if (row < len) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              __half2 hv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                hv[e] = __floats2half2_rn(__uint_as_float(o[8 * k + 2 * e]) * inv,
                                          __uint_as_float(o[8 * k + 2 * e + 1]) * inv);
              *reinterpret_cast<uint4*>(dst + hh * 32 + 8 * k) = *reinterpret_cast<uint4*>(hv);
            }
          }
        }
        if (row < len && p.lse) p.lse[static_cast<size_t>(h) * p.T + start + row] = (mc + log2f(l)) / kLog2e;
      }
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols2);
  }
}

template <int DH, int POLY>
cudaError_t launch_poly(const CUtensorMap& tm_q, const CUtensorMap& tm_kv, const AttnParams& p, cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc2_kernel<DH, POLY>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Tc2<DH>::kSmem);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  dim3 grid(p.n_work, p.H);
  attention_tc2_kernel<DH, POLY><<<grid, kThreads2, Tc2<DH>::kSmem, s>>>(tm_q, tm_kv, p);
  return cudaGetLastError();
}

template <int DH>
cudaError_t launch_dh2(const CUtensorMap& tm_q, const CUtensorMap& tm_kv, const AttnParams& p, int poly_eighths,
                       cudaStream_t s) {
  switch (poly_eighths) {
    case 0: return launch_poly<DH, 0>(tm_q, tm_kv, p, s);
    case 1: return launch_poly<DH, 1>(tm_q, tm_kv, p, s);
    case 2: return launch_poly<DH, 2>(tm_q, tm_kv, p, s);
    case 3: return launch_poly<DH, 3>(tm_q, tm_kv, p, s);
    case 4: return launch_poly<DH, 4>(tm_q, tm_kv, p, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_attention_tc2(const CUtensorMap& tm_q, const CUtensorMap& tm_kv, const AttnParams& p,
                                 int poly_eighths, cudaStream_t s) {
  if (p.n_work <= 0) return cudaSuccess;
  if (p.dh == 64) return launch_dh2<64>(tm_q, tm_kv, p, poly_eighths, s);
  if (p.dh == 32) return launch_dh2<32>(tm_q, tm_kv, p, poly_eighths, s);
  return cudaErrorInvalidValue;
}

}  // namespace esm
