// Contact-head accumulation on the 5th-generation tensor cores (tcgen05) for head_dim 64, the
// ESM-2 650M and 3B shape. Same result as contact_accumulate_kernel in attention.cu; replaces the
// per-head part of the reference contact head (accumulate_head_apc, src/lib.rs:5036-5076, called
// for every head at 5303-5312).
//
// Per layer, every head h with a non-zero regression weight w_h contributes
//   M += w_h P_h                          (P_h = softmax rows of the attention, inner block only)
//   r_h[i] += rowsum_i(P_h) + colsum_i(P_h)   (APC sums of the symmetrised map P_h + P_h^T)
// over the inner block (tokens 1..n, n = L - 2). P_h is recomputed from Q, K and the row
// log-sum-exp that the attention kernel saved, so no per-head map is stored.
//
// The tile is computed transposed: S^T = K Q^T with M = 128 keys (tensor-memory lanes, one key per
// thread) and N = 64 queries. A thread then owns a key column of P: its column sum accumulates in
// a register, and it keeps 32 entries of M^T for its key in registers across all heads. M is only
// ever used as M + M^T, so storing M^T in place of M gives the same contacts. The row sums need no
// reduction: rows of P sum to one over all L keys, so the row sum over the inner keys is
// 1 - P[i, 0] - P[i, L-1], which contact_rowsum_kernel adds for every inner query from two dot
// products (keeping that term out of this kernel keeps the tiles that hold key 0 or L-1 as fast as
// the others).
//
// One CTA per (sequence, 128-key tile, 64-query tile); 320 threads; two CTAs per SM.
//   warp 0      TMA producer: the K and Q tiles of each contributing head into a 4-stage ring.
//   warp 1      tcgen05.mma issuer: S^T = K Q^T (M 128, N 64, K 64) into one of four TMEM buffers.
//   warps 2..9  two warps per TMEM lane quarter, each one key per thread over 32 of the queries:
//               copy its S^T slice to registers and release the buffer at once, then exp2(S c - lse)
//               (three in four on the special-function unit, one on the FP32 pipe), M^T and column
//               sums in registers; at the end M^T is staged through shared memory and added to M
//               with coalesced rows.
// Four S^T buffers let the MMAs run up to three heads ahead of the exponentials: with two, the
// round trip MMA -> softmax read -> buffer release -> next MMA set the pace, not the math.
// All waits are bounded; on a timeout the error word is set and M is left untouched.
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kKeys = 128;    // keys per tile (MMA M, TMEM lanes)
constexpr int kQry = 64;      // queries per tile (MMA N)
constexpr int kQHalf = 32;    // queries per epilogue thread
constexpr int kSBufs = 4;     // S^T buffers in tensor memory (64 columns each)
constexpr int kD = 64;        // head dim (MMA K)
constexpr int kThreadsCt = 320;
constexpr int kKBytes = kKeys * kD * 2;  // 16 KiB
constexpr int kQBytes = kQry * kD * 2;   // 8 KiB
constexpr int kStageBytes = kKBytes + kQBytes;
constexpr int kStages = 4;
constexpr int kOffLse = kStages * kStageBytes;  // [n_heads][64] lse * log2(e) (inf outside 1..n)
constexpr int kMaxHeads = 64;
constexpr int kStageStride = kQry + 1;  // floats per staged M^T row (conflict-free)
constexpr uint32_t kTmemCols = 256;     // four S^T buffers of 64 columns
constexpr float kLog2e = 1.4426950408889634f;

// M^T is staged over the operand ring and the log-sum-exp table once the head loop is done.
inline int contact_tc_smem_bytes(int H) {
  const int used = kOffLse + H * kQry * 4 + kMaxHeads * 8 + 256;
  const int stage = kKeys * kStageStride * 4;
  return (used > stage ? used : stage) + 1024;
}

__global__ void __launch_bounds__(kThreadsCt, 2)
    contact_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_q,
                      const ContactParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* lse_s = reinterpret_cast<float*>(smem + kOffLse);
  int* heads = reinterpret_cast<int*>(smem + kOffLse + p.H * kQry * 4);  // contributing heads
  float* wts = reinterpret_cast<float*>(heads + kMaxHeads);               // and their weights
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffLse + p.H * kQry * 4 + kMaxHeads * 8);
  uint64_t* full = bars + 0;                       // [kStages]
  uint64_t* empty = full + kStages;                // [kStages]
  uint64_t* s_full = empty + kStages;              // [kSBufs]
  uint64_t* s_free = s_full + kSBufs;              // [kSBufs]
  uint64_t* drain = s_free + kSBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* nh_s = reinterpret_cast<int*>(drain + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int4 tl = p.tiles[blockIdx.x];
  const int b = tl.x, k0 = tl.y * kKeys, q0 = tl.z * kQry;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int n = len - 2;

  if (warp == 0) {
    // Heads with a non-zero weight (H <= 64), compacted with ballots. Each CTA starts its head loop
    // at a different head, so the CTAs running at the same time do not all fetch the same K and Q
    // lines from L2 at once.
    const float w0 = lane < p.H ? p.w_layer[lane] : 0.0f;
    const float w1 = lane + 32 < p.H ? p.w_layer[lane + 32] : 0.0f;
    const unsigned m0 = __ballot_sync(0xffffffffu, w0 != 0.0f);
    const unsigned m1 = __ballot_sync(0xffffffffu, w1 != 0.0f);
    const int n0 = __popc(m0), nh = n0 + __popc(m1);
    const int rot = nh > 0 ? static_cast<int>(blockIdx.x % nh) : 0;
    const unsigned below = (1u << lane) - 1u;
    if (w0 != 0.0f) {
      const int slot = (__popc(m0 & below) - rot + nh) % nh;
      heads[slot] = lane;
      wts[slot] = w0;
    }
    if (w1 != 0.0f) {
      const int slot = (n0 + __popc(m1 & below) - rot + nh) % nh;
      heads[slot] = lane + 32;
      wts[slot] = w1;
    }
    if (lane == 0) *nh_s = nh;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kSBufs; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 8);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int nh = *nh_s;
  if (nh == 0 || n <= 0) return;
  // Row log-sum-exps of this query tile for every contributing head, in the exp2 domain; queries
  // outside the inner block get +inf so that their P is exactly 0.
  // All of a thread's loads are issued before the first store, so their latencies overlap.
  {
    constexpr int kIters = (kMaxHeads * kQry + kThreadsCt - 1) / kThreadsCt;
    float lv[kIters];
#pragma unroll
    for (int k = 0; k < kIters; ++k) {
      const int idx = threadIdx.x + k * kThreadsCt;
      const int t = idx / kQry, i = q0 + idx % kQry;
      lv[k] = (idx < nh * kQry && i >= 1 && i <= n) ? p.lse[static_cast<size_t>(heads[t]) * p.T + start + i] : INFINITY;
    }
#pragma unroll
    for (int k = 0; k < kIters; ++k) {
      const int idx = threadIdx.x + k * kThreadsCt;
      if (idx < nh * kQry) lse_s[idx] = -lv[k] * kLog2e;  // stored negated: the exponent is S c + lse_s
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // M^T[key, q0 + 32 * qh + c] summed over heads (epilogue threads), as packed FP32 pairs (c, c + 1).
  uint64_t acc2[kQHalf / 2];
#pragma unroll
  for (int c = 0; c < kQHalf / 2; ++c) acc2[c] = 0ull;
  bool ok = true;

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tmap_k);
      tma_prefetch_desc(&tmap_q);
      // Q and K of a layer are re-read by every tile of the sequence: keep them in L2 ahead of the
      // M accumulator, which streams through once per layer.
      const uint64_t pol = l2_policy_evict_last();
      int t = 0;
      for (; t < nh; ++t) {
        const int st = t % kStages;
        if (!mbar_wait(&empty[st], ((t / kStages) & 1) ^ 1u, p.err, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        const int h = heads[t];
        uint8_t* dst = smem + st * kStageBytes;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_2d(dst, &tmap_k, &full[st], p.d + h * kD, start + k0, pol);
        tma_load_2d(dst + kKBytes, &tmap_q, &full[st], h * kD, start + q0, pol);
      }
      if (!ok) {  // let the loads already in flight land before the CTA exits
        for (int tt = (t - kStages > 0 ? t - kStages : 0); tt < t; ++tt)
          mbar_wait(&full[tt % kStages], (tt / kStages) & 1, p.err, kDevTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc = umma_idesc_f16(kKeys, kQry);
      for (int t = 0; t < nh && ok; ++t) {
        const int st = t % kStages;  // operand stage
        const int sb = t % kSBufs;   // S^T buffer
        if (!mbar_wait(&full[st], (t / kStages) & 1, p.err, kDevTimeoutMma)) { ok = false; break; }
        if (t >= kSBufs && !mbar_wait(&s_free[sb], ((t / kSBufs) - 1) & 1, p.err, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + st * kStageBytes);
        const uint32_t q_addr = k_addr + kKBytes;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          umma_f16(tmem + sb * kQry, umma_sdesc_sw128(k_addr + k * 32), umma_sdesc_sw128(q_addr + k * 32), idesc,
                   k > 0);
        umma_commit(&s_full[sb]);
        umma_commit(&empty[st]);
      }
      if (!ok) {
        umma_commit(drain);
        mbar_wait(drain, 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- one key per thread, 32 queries per warp ----------------
    const int quarter = warp & 3;
    const int qh = (warp - 2) >> 2;      // which 32 queries of the tile
    const int kr = quarter * 32 + lane;  // key row inside the tile = TMEM lane
    const int key = k0 + kr;             // token index inside the sequence
    const bool inner_key = key >= 1 && key <= n;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_off + qh * kQHalf;
    const uint64_t c2 = f2_pack(p.scale * kLog2e, p.scale * kLog2e);
    float* const rbase = p.r + p.r_off[b] + static_cast<size_t>(p.head_base) * n;
    // Head t's P column: exponents, M^T += w P, and the column sum into r (APC).
    auto head = [&](const uint32_t (&sv)[kQHalf], int t) {
      const float w = wts[t];
      const float* lrow = lse_s + t * kQry + qh * kQHalf;
      const uint64_t w2 = f2_pack(w, w);
      uint64_t cs2 = 0ull;
#pragma unroll
      for (int g = 0; g < kQHalf / 4; ++g) {
        const float4 l4 = *reinterpret_cast<const float4*>(lrow + 4 * g);
        float a0, a1, a2, a3;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[4 * g]), __uint_as_float(sv[4 * g + 1])), c2, f2_pack(l4.x, l4.y)),
                  a0, a1);
        f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[4 * g + 2]), __uint_as_float(sv[4 * g + 3])), c2,
                         f2_pack(l4.z, l4.w)),
                  a2, a3);
        // One exponential in four on the FP32 pipe, the rest on the special-function unit.
        const uint64_t p01 = f2_pack(fast_exp2(a0), fast_exp2(a1));
        const uint64_t p23 = f2_pack(fast_exp2(a2), poly_exp2(a3));
        cs2 = f2_add(cs2, f2_add(p01, p23));
        acc2[2 * g] = f2_fma(w2, p01, acc2[2 * g]);
        acc2[2 * g + 1] = f2_fma(w2, p23, acc2[2 * g + 1]);
      }
      float x0, x1;
      f2_unpack(cs2, x0, x1);
      if (inner_key) atomicAdd(rbase + static_cast<size_t>(heads[t]) * n + (key - 1), x0 + x1);
    };
    for (int t = 0; t < nh; ++t) {
      const int sb = t % kSBufs;
      if (!mbar_wait(&s_full[sb], (t / kSBufs) & 1, p.err, kDevTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[kQHalf];
      tmem_ld32(t_s + sb * kQry, sv);
      tmem_ld_wait_regs(sv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);  // the MMA of head t + 4 may overwrite this buffer
      head(sv, t);
    }
  }
  // Every role is done with the operand ring (loads landed, MMAs complete) past this barrier.
  const int failed = __syncthreads_or(!ok);
  float* stage = reinterpret_cast<float*>(smem);
  if (!failed && warp >= 2) {
    const int kr = (warp & 3) * 32 + lane;
    const int qh = (warp - 2) >> 2;
#pragma unroll
    for (int cc = 0; cc < kQHalf / 2; ++cc) {
      float x0, x1;
      f2_unpack(acc2[cc], x0, x1);
      stage[kr * kStageStride + qh * kQHalf + 2 * cc] = x0;
      stage[kr * kStageStride + qh * kQHalf + 2 * cc + 1] = x1;
    }
  }
  __syncthreads();
  if (!failed && warp >= 2) {
    // M^T rows of this tile: row (key - 1), columns (q0 + c - 1), inner entries only. Each warp
    // reads eight of its row segments before writing them, so the loads overlap.
    float* Mb = p.M + p.m_off[b];
    const int wq = warp - 2;
    constexpr int kBatch = 8, kCols = kQry / 32;
#pragma unroll 1
    for (int r0 = 0; r0 < kKeys / 8; r0 += kBatch) {
      float mv[kBatch][kCols];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int key = k0 + wq + 8 * (r0 + k);
#pragma unroll
        for (int u = 0; u < kCols; ++u) {
          const int i = q0 + lane + 32 * u;
          mv[k][u] = (key >= 1 && key <= n && i >= 1 && i <= n) ? __ldcs(Mb + static_cast<size_t>(key - 1) * n + (i - 1)) : 0.0f;
        }
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int rr = wq + 8 * (r0 + k);
        const int key = k0 + rr;
#pragma unroll
        for (int u = 0; u < kCols; ++u) {
          const int i = q0 + lane + 32 * u;
          if (key >= 1 && key <= n && i >= 1 && i <= n)
            __stcs(Mb + static_cast<size_t>(key - 1) * n + (i - 1), mv[k][u] + stage[rr * kStageStride + lane + 32 * u]);
        }
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

// The row-sum half of the APC sums for every inner query i and contributing head h:
// r_h[i] += 1 - P[i, 0] - P[i, L-1], with P[i, k] = exp2(q_i . k_k * scale * log2(e) - lse_i log2(e))
// from the same fp16 Q and K and the attention's log-sum-exp (rows of P sum to one over all L keys).
// One thread per token; heads in a loop. Runs after contact_tc_kernel of the layer, on the same
// stream, so the plain read-modify-write of r does not meet that kernel's atomic column sums.
__global__ void contact_rowsum_kernel(const ContactParams p, const int32_t* __restrict__ seq_of) {
  const int tok = blockIdx.x * blockDim.x + threadIdx.x;
  if (tok >= p.T) return;
  const int b = seq_of[tok];
  const int start = p.cu_seqlens[b], len = p.cu_seqlens[b + 1] - start, n = len - 2;
  const int i = tok - start;
  if (i < 1 || i > n) return;
  const float c = p.scale * kLog2e;
  const size_t ld = static_cast<size_t>(3) * p.d;
  const __half* q = p.qkv + static_cast<size_t>(tok) * ld;
  const __half* k0 = p.qkv + static_cast<size_t>(start) * ld + p.d;
  const __half* k1 = p.qkv + static_cast<size_t>(start + len - 1) * ld + p.d;
  float* rb = p.r + p.r_off[b] + static_cast<size_t>(p.head_base) * n + (i - 1);
  for (int h = 0; h < p.H; ++h) {
    const float w = p.w_layer[h];
    if (w == 0.0f) continue;
    float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
    for (int e = 0; e < kD; e += 8) {
      const uint4 qv = *reinterpret_cast<const uint4*>(q + h * kD + e);
      const uint4 av = *reinterpret_cast<const uint4*>(k0 + h * kD + e);
      const uint4 bv = *reinterpret_cast<const uint4*>(k1 + h * kD + e);
      const __half2* qh = reinterpret_cast<const __half2*>(&qv);
      const __half2* ah = reinterpret_cast<const __half2*>(&av);
      const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 qf = __half22float2(qh[u]), af = __half22float2(ah[u]), bf = __half22float2(bh[u]);
        d0 = fmaf(qf.x, af.x, fmaf(qf.y, af.y, d0));
        d1 = fmaf(qf.x, bf.x, fmaf(qf.y, bf.y, d1));
      }
    }
    const float l2 = p.lse[static_cast<size_t>(h) * p.T + tok] * kLog2e;
    const float p0 = fast_exp2(fmaf(d0, c, -l2));
    const float p1 = fast_exp2(fmaf(d1, c, -l2));
    rb[static_cast<size_t>(h) * n] += (1.0f - p0) - p1;
  }
}

int contact_tc_tiles(int len, int4* out, int b) {
  const int kt = (len + kKeys - 1) / kKeys, qt = (len + kQry - 1) / kQry;
  if (out)
    for (int i = 0; i < kt; ++i)
      for (int j = 0; j < qt; ++j) out[i * qt + j] = make_int4(b, i, j, 0);
  return kt * qt;
}

cudaError_t launch_contact_tc(const CUtensorMap& tm_k128, const CUtensorMap& tm_q64, const ContactParams& p,
                              const int32_t* seq_of, cudaStream_t s) {
  if (p.n_tiles <= 0) return cudaSuccess;
  if (p.dh != kD || p.H > kMaxHeads) return cudaErrorInvalidValue;
  const int smem = contact_tc_smem_bytes(p.H);
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    // The largest head count (64) fixes the attribute once per device.
    cudaError_t e = cudaFuncSetAttribute(contact_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         contact_tc_smem_bytes(kMaxHeads));
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  contact_tc_kernel<<<p.n_tiles, kThreadsCt, smem, s>>>(tm_k128, tm_q64, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  contact_rowsum_kernel<<<(p.T + 127) / 128, 128, 0, s>>>(p, seq_of);
  return cudaGetLastError();
}

}  // namespace esm
