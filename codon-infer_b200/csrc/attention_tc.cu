// Bidirectional attention on the 5th-generation tensor cores (tcgen05) for head_dim 64, the
// ESM-2 650M and 3B shape. Same contract as attention_kernel in attention.cu (packed varlen
// sequences, keys past a sequence's end masked, O in fp16, optional per-row log-sum-exp), which
// replaces the reference attention loop (src/lib.rs:5206-5301).
//
// One CTA per (sequence, 128-query tile, head); 192 threads; three CTAs per SM.
//   warp 0      TMA producer: Q tile once, then 64-key K and V tiles into a 2-stage ring.
//   warp 1      tcgen05.mma issuer (one thread): S = Q K^T (M 128, N 64, K 64) into tensor memory,
//               then O_j = P_j V_j (M 128, N 64, K 64) with V as an MN-major operand.
//   warps 2..5  softmax, one query row per thread: read S from tensor memory, online max/sum in
//               fp32 (exp2 on the special-function unit), P rounded to fp16 into shared memory in
//               the 128-byte-swizzled K-major layout the MMA reads. O accumulates across tiles in
//               tensor memory; it is rescaled there only when a row max grows past the threshold.
// Tensor memory: S in columns [0, 64), O in [64, 128). All waits are bounded.
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kQ = 128;   // query rows per CTA
constexpr int kKV = 64;   // keys per tile
constexpr int kD = 64;    // head dim
constexpr int kThreadsAt = 192;
constexpr int kQBytes = kQ * kD * 2;    // 16 KiB
constexpr int kKVBytes = kKV * kD * 2;  // 8 KiB
constexpr int kPBytes = kQ * kKV * 2;   // 16 KiB
constexpr int kOffK = kQBytes;
constexpr int kOffV = kOffK + 2 * kKVBytes;
constexpr int kOffP = kOffV + 2 * kKVBytes;
constexpr int kOffBar = kOffP + kPBytes;
constexpr int kSmemAt = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 128;  // S [0, 64), O [64, 128)
constexpr float kLog2e = 1.4426950408889634f;
// The running max used for P is refreshed only when a row's max grows by more than 2^8 (in the
// exp2 domain); until then P <= 256, exact in fp16's relative precision, and O and l share the
// stale max, so O / l and the log-sum-exp are unchanged.
constexpr float kRescaleThreshold = 8.0f;

// Pipeline per 64-key tile j (all waits bounded):
//   MMA:     S = Q K_j^T        after K_j landed and the softmax read S_{j-1}        -> s_full
//            O += P V_j         after P_j was written (O accumulates in tensor memory) -> o_full
//   softmax: read S_j (-> s_free); when a row max jumped past the threshold, wait for the previous
//            O += P V and rescale O in tensor memory; P_j = exp2(S c - m) into shared memory once
//            the previous P V has consumed the buffer (-> p_full).
// o_full can run at most one completion ahead of the softmax's waits (P V_{j+1} needs p_full of
// tile j+1), so parity waits stay unambiguous even where a wait is skipped.
__global__ void __launch_bounds__(kThreadsAt, 3)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_kv,
                        const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* o_full = bars + 8;
  uint64_t* drain = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int2 wk = p.work[blockIdx.x];
  const int b = wk.x, q0 = wk.y * kQ, h = blockIdx.y;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int nkv = (len + kKV - 1) / kKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem;       // S: columns [0, 64)
  const uint32_t t_o = tmem + 64;  // O: columns [64, 128)

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_kv);
      const uint64_t pol = l2_policy_evict_normal();
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem, &tmap_q, q_full, h * kD, start + q0, pol);
      bool ok = true;
      int j = 0;
      for (; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, p.err, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKVBytes);
        tma_load_2d(smem + kOffK + st * kKVBytes, &tmap_kv, &kv_full[st], p.d + h * kD, start + j * kKV, pol);
        tma_load_2d(smem + kOffV + st * kKVBytes, &tmap_kv, &kv_full[st], 2 * p.d + h * kD, start + j * kKV, pol);
      }
      if (!ok) {
        mbar_wait(q_full, 0, p.err, kDevTimeoutProducer);
        for (int jj = (j - 2 > 0 ? j - 2 : 0); jj < j; ++jj)
          mbar_wait(&kv_full[jj & 1], (jj >> 1) & 1, p.err, kDevTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc_qk = umma_idesc_f16(kQ, kKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kQ, kD) | (1u << 16);  // B (V) is MN-major
      const uint32_t q_addr = smem_u32(smem);
      const uint32_t p_addr = smem_u32(smem + kOffP);
      bool ok = mbar_wait_spin(q_full, 0, p.err, kDevTimeoutMma);
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_spin(&kv_full[st], ph, p.err, kDevTimeoutMma)) { ok = false; break; }
        if (j > 0 && !mbar_wait_spin(s_free, (j - 1) & 1, p.err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + kOffK + st * kKVBytes);
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_f16(t_s, umma_sdesc_sw128(q_addr + k * 32), umma_sdesc_sw128(k_addr + k * 32), idesc_qk, k > 0);
        umma_commit(s_full);
        if (!mbar_wait_spin(p_full, j & 1, p.err, kDevTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + kOffV + st * kKVBytes);
#pragma unroll
        for (int k = 0; k < kKV / 16; ++k)
          umma_f16(t_o, umma_sdesc_sw128(p_addr + k * 32), umma_sdesc_sw128_mn(v_addr + k * 2048), idesc_pv,
                   (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(o_full);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) {
        umma_commit(drain);
        mbar_wait_spin(drain, 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- softmax: thread = query row ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row inside the tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.scale * kLog2e;
    float mc = -INFINITY;  // running max in the exp2 domain (max score * c)
    float l = 0.0f;
    uint8_t* prow = smem + kOffP + r * 128;
    const int sw = r & 7;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      if (!mbar_wait_spin(s_full, j & 1, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      const int kvalid = len - j * kKV;  // keys of this tile inside the sequence (> 0)
      // Pass 1: row max (32 columns at a time keeps registers low). c > 0, so the max of the
      // scaled scores is c times the max of the raw ones; only the last tile needs the key mask.
      float mraw = -INFINITY;
      if (kvalid >= kKV) {
        // Tree reduction: 8 independent partial maxima keep the dependency chains short.
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = -INFINITY;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t t[32];
          tmem_ld32(t_s + lane_off + half * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(t[i]));
        }
        mraw = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      } else {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t t[32];
          tmem_ld32(t_s + lane_off + half * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (half * 32 + i < kvalid) mraw = fmaxf(mraw, __uint_as_float(t[i]));
        }
      }
      const float mx = mraw * c;
      if (j == 0) {
        mc = mx;
      } else if (__any_sync(0xffffffffu, mx - mc > kRescaleThreshold)) {
        // Refresh the max of this warp's rows: O (after the previous P V) and l scale by alpha.
        const float m_new = fmaxf(mc, mx);
        const float alpha = fast_exp2(mc - m_new);
        if (!mbar_wait_spin(o_full, (j - 1) & 1, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t t[32];
          tmem_ld32(t_o + lane_off + half * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * alpha);
          tmem_st32(t_o + lane_off + half * 32, t);
        }
        tmem_st_wait();
        l *= alpha;
        mc = m_new;
      }
      // The previous P V must have consumed the P buffer before it is overwritten.
      if (j > 0 && !mbar_wait_spin(o_full, (j - 1) & 1, p.err, kDevTimeoutEpilogue)) { ok = false; break; }
      // Pass 2: P = exp2(S c - m) in fp16 into the 128-byte swizzled K-major tile (16-byte chunk k
      // of row r at chunk k ^ (r & 7)); keys past the sequence end get P = 0.
      float rsp[8];  // independent partial row sums
#pragma unroll
      for (int u = 0; u < 8; ++u) rsp[u] = 0.0f;
      const bool full_tile = kvalid >= kKV;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t t[32];
        tmem_ld32(t_s + lane_off + half * 32, t);
        tmem_ld_wait();
        if (!full_tile) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (half * 32 + i >= kvalid) t[i] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float e[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            e[u] = fast_exp2(fmaf(__uint_as_float(t[8 * k + u]), c, -mc));
            rsp[u] += e[u];
          }
          __half2 hv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) hv[u] = __floats2half2_rn(e[2 * u], e[2 * u + 1]);
          const int chunk = half * 4 + k;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ sw) << 4)) = *reinterpret_cast<uint4*>(hv);
        }
      }
      l += ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(s_free);  // the next Q K^T may overwrite S
        mbar_arrive(p_full);
      }
    }
    if (ok && mbar_wait_spin(o_full, (nkv - 1) & 1, p.err, kDevTimeoutEpilogue)) {
      tc_fence_after();
      const int row = q0 + r;
      const float inv = 1.0f / l;
      __half* dst = p.out + static_cast<size_t>(start + row) * p.d + h * kD;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t t[32];
        tmem_ld32(t_o + lane_off + half * 32, t);
        tmem_ld_wait();
        if (row < len) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            __half2 hv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              hv[e] = __floats2half2_rn(__uint_as_float(t[8 * k + 2 * e]) * inv,
                                        __uint_as_float(t[8 * k + 2 * e + 1]) * inv);
            *reinterpret_cast<uint4*>(dst + half * 32 + 8 * k) = *reinterpret_cast<uint4*>(hv);
          }
        }
      }
      if (row < len && p.lse) p.lse[static_cast<size_t>(h) * p.T + start + row] = (mc + log2f(l)) / kLog2e;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_attention_tc(const CUtensorMap& tm_q, const CUtensorMap& tm_kv, const AttnParams& p,
                                cudaStream_t s) {
  if (p.n_work <= 0) return cudaSuccess;
  if (p.dh != kD) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAt);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  dim3 grid(p.n_work, p.H);
  attention_tc_kernel<<<grid, kThreadsAt, kSmemAt, s>>>(tm_q, tm_kv, p);
  return cudaGetLastError();
}

}  // namespace esm
