// Bidirectional attention on tcgen05 for head_dim 64 and 32 (and 16 / 24, zero-padded to 32 by the
// tensor maps) with two score buffers per query tile, so the tensor cores compute S(j + 2) while
// the softmax works on S(j) and S(j + 1). Same contract as
// attention_kernel in attention.cu (packed varlen sequences, keys past a sequence's end masked, O
// in fp16, optional per-row log-sum-exp); replaces the reference attention loop
// (src/lib.rs:5206-5301).
//
// One CTA per (sequence, 256-query block, head); 352 threads; two CTAs per SM.
//   warps 0..3  softmax of query tile 0 (rows 0..127 of the block), one row per thread
//   warps 4..7  softmax of query tile 1 (rows 128..255)
//   warp 8      TMA producer: both Q tiles once, then 32-key K and V tiles into an 8-stage ring
//   warp 9, 10  tcgen05.mma issuers of query tile 0 and 1
// Tensor memory (256 columns): S_{t,b} (tile t, buffer b, 32 keys) in [32 (2t + b), +32), O_t in
// [128 + 64 t, +64). Key tile j uses buffer j & 1. The softmax writes P (fp16 pairs) over the first
// 16 columns of S_{t,b} and O_t += P V is issued with A read from tensor memory. Per tile the MMA
// order is S(0) S(1) | PV(0) S(2) | PV(1) S(3) | ...: S(j + 2) overwrites the buffer PV(j) has
// read, and MMAs of one thread execute in issue order.
//
// One barrier per (tile, score buffer), step[t][b], carries every MMA completion the tile's softmax
// waits for: the tile's issuer commits S(b) to it in the prologue, and once per key tile j, after
// PV(j) S(j + 2), to step[t][j & 1]. Completion number n of step[t][b] (1-based) is therefore
// S(b + 2(n - 1)) and, for n >= 2, PV(b + 2(n - 2)). The softmax waits on each barrier in order and
// never more than one completion ahead of the last one it consumed on that barrier, so every parity
// wait is unambiguous. (A single barrier per tile for the PVs would not be: at the end PV(n - 2) may still be
// outstanding, and a parity wait for PV(n - 1) would match the completed phase of PV(n - 3).)
// O is rescaled in tensor memory only when the running max has gone stale (EXP 3, the default: a
// step's row sum against it exceeds p.rescale_sum; EXP 0..2: a step's row max exceeds it by more
// than 2^8), after PV(j - 1) has completed. All waits are bounded.
#include <atomic>

#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr int kQ = 128;   // rows per query tile
constexpr int kKV = 32;   // keys per K/V tile
constexpr int kThreads3 = 352;
constexpr int kStages3 = 8;
// Tile geometry for head_dim DH: 64 (128-byte rows, 128-byte swizzle) or 32 (64-byte rows and
// swizzle). The UMMA descriptors of both layouts differ only in the high word. With SPLIT (the
// zero-padded 16 / 24-wide heads) shared memory also holds the fp16 rounding residues of the two
// query tiles and of every key tile: Q_hi t0 | Q_hi t1 | Q_lo t0 | Q_lo t1, stages K | V | K_lo.
template <int DH, int SPLIT = 0>  // SPLIT: 0 plain scores, 2 with the query and key residues
struct Tc3 {
  static constexpr int kQBytes = kQ * DH * 2;    // one query tile
  static constexpr int kKVBytes = kKV * DH * 2;  // one K or V tile
  static constexpr int kStageTiles = SPLIT == 2 ? 3 : 2;
  static constexpr int kOffKV = (SPLIT ? 4 : 2) * kQBytes;
  static constexpr int kOffBar = kOffKV + kStages3 * kStageTiles * kKVBytes;
  static constexpr int kSmem = kOffBar + 256 + 1024;
  static constexpr uint32_t kDescHi = DH == 64 ? kSw128DescHi : kSw64DescHi;
};
constexpr uint32_t kTmemCols3 = 256;
constexpr float kLog2e = 1.4426950408889634f;
// The running max used for P is refreshed only when a row's max grows by more than 2^8 (in the
// exp2 domain); until then P <= 256, exact in fp16's relative precision, and O and l share the
// stale max, so O / l and the log-sum-exp are unchanged.
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ uint32_t s_col(int t, int b) { return static_cast<uint32_t>(kKV * (2 * t + b)); }
template <int DH>
__device__ __forceinline__ uint32_t o_col(int t) { return static_cast<uint32_t>(128 + DH * t); }

// POLY of every 8 column pairs take their exponentials on the FP32 pipe (poly_exp2) instead of the
// special-function unit. EXP selects the softmax arithmetic: 0 scalar FP32, 1 packed FP32 pairs
// (fma/add.f32x2) and three-input maxima, 2 the same with the exponentials taken on fp16 pairs,
// 3 packed pairs against the running max with no per-step row max (the step's row sum decides
// when the max is refreshed).
// PAD: the heads are p.dh = 16 or 24 wide and arrive through 3-D maps ([rows][3 H][p.dh], boxes
// 32 wide) zero-padded to DH = 32 columns, which changes neither Q K^T nor the first p.dh columns
// of P V; only p.dh output columns are stored. These heads also take their scores in split
// precision: tmap_qlo / tmap_klo read the fp16 rounding residues of the queries and keys
// ([rows][2 H][p.dh], written by the QKV projection) and S = Q_hi K_hi^T + Q_lo K_hi^T + Q_hi K_lo^T,
// which leaves only the products of two residues out of the fp32 score. (With peaked attention,
// as in trained models, fp16 queries and keys alone move the scores of the dominant keys by a few
// hundredths and the logits by about 1e-2.) Other head sizes pass tmap_q / tmap_kv again there.
template <int DH, int POLY, int EXP, bool PAD, int SPLIT>
__global__ void __launch_bounds__(kThreads3, 2)
    attention_tc3_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_kv,
                         const __grid_constant__ CUtensorMap tmap_qlo, const __grid_constant__ CUtensorMap tmap_klo,
                         const AttnParams p) {
  static_assert(!PAD || DH == 32, "padded heads use the 32-column tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  static_assert(SPLIT == (PAD ? 2 : 0), "the padded heads, and only they, take split scores");
  using G = Tc3<DH, SPLIT>;
  constexpr int kD = DH, kQBytes = G::kQBytes, kKVBytes = G::kKVBytes, kOffKV = G::kOffKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;               // [8]
  uint64_t* kv_empty = kv_full + kStages3;    // [8]
  uint64_t* step = kv_empty + kStages3;       // [2 tiles][2 buffers]: S and PV completions
  uint64_t* p_full = step + 4;                // [2 tiles][2 buffers]: P written
  uint64_t* drain = p_full + 4;               // [2 tiles]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int2 wk = p.work[blockIdx.x];
  const int b = wk.x, q0 = wk.y * (2 * kQ), h = blockIdx.y;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int nkv = (len + kKV - 1) / kKV;
  const int ntiles = q0 + kQ < len ? 2 : 1;  // the second query tile holds rows of this sequence

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages3; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], ntiles);  // one commit from each tile's MMA issuer
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&step[i], 1);
      mbar_init(&p_full[i], 4);
    }
    for (int t = 0; t < 2; ++t) mbar_init(&drain[t], 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, kTmemCols3);
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
      mbar_arrive_expect_tx(q_full, ntiles * kQBytes * (SPLIT ? 2 : 1));
      for (int t = 0; t < ntiles; ++t) {
        if constexpr (PAD) {
          tma_load_3d(smem + t * kQBytes, &tmap_q, q_full, 0, h, start + q0 + t * kQ, pol);
          if constexpr (SPLIT > 0)
            tma_load_3d(smem + (2 + t) * kQBytes, &tmap_qlo, q_full, 0, h, start + q0 + t * kQ, pol);
        } else {
          tma_load_2d(smem + t * kQBytes, &tmap_q, q_full, h * kD, start + q0 + t * kQ, pol);
        }
      }
      bool ok = true;
      int j = 0;
      for (; j < nkv; ++j) {
        const int st = j % kStages3;
        if (!mbar_wait(&kv_empty[st], ((j / kStages3) & 1) ^ 1u, p.err, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        uint8_t* dst = smem + kOffKV + st * G::kStageTiles * kKVBytes;
        mbar_arrive_expect_tx(&kv_full[st], G::kStageTiles * kKVBytes);
        if constexpr (PAD) {
          tma_load_3d(dst, &tmap_kv, &kv_full[st], 0, p.H + h, start + j * kKV, pol);
          tma_load_3d(dst + kKVBytes, &tmap_kv, &kv_full[st], 0, 2 * p.H + h, start + j * kKV, pol);
          if constexpr (SPLIT == 2)
            tma_load_3d(dst + 2 * kKVBytes, &tmap_klo, &kv_full[st], 0, p.H + h, start + j * kKV, pol);
        } else {
          tma_load_2d(dst, &tmap_kv, &kv_full[st], p.d + h * kD, start + j * kKV, pol);
          tma_load_2d(dst + kKVBytes, &tmap_kv, &kv_full[st], 2 * p.d + h * kD, start + j * kKV, pol);
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        mbar_wait(q_full, 0, p.err, kDevTimeoutProducer);
        for (int jj = (j - kStages3 > 0 ? j - kStages3 : 0); jj < j; ++jj)
          mbar_wait(&kv_full[jj % kStages3], (jj / kStages3) & 1, p.err, kDevTimeoutProducer);
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ---------------- MMA issuers: warp 9 for query tile 0, warp 10 for tile 1 ----------------
    // An issuer shares its SM sub-partition with four busy softmax warps and gets a fraction of the
    // issue slots, so each tile has its own (the two sit on different sub-partitions) and the loop
    // is kept to few instructions: descriptors are low words plus constant offsets and barriers
    // are precomputed shared-memory addresses. Each issuer's MMAs execute in its issue order, which
    // is all the buffer reuse of its tile relies on; the K/V stages are released by one commit from
    // each issuer (kv_empty counts ntiles arrivals).
    const int t = warp - 9;
    if (t < ntiles && elect_one_sync()) {
      constexpr uint32_t idesc_qk = umma_idesc_f16(kQ, kKV);
      constexpr uint32_t idesc_pv = umma_idesc_f16(kQ, kD) | (1u << 16);  // B (V) is MN-major
      constexpr uint32_t kStageLo = (G::kStageTiles * kKVBytes) >> 4, kVLo = kKVBytes >> 4, kQLo = kQBytes >> 4;
      constexpr uint32_t kVStepLo = (16 * kD * 2) >> 4;  // 16 keys of V
      const uint32_t q_lo = umma_sw128_lo(smem_u32(smem)) + t * kQLo;
      const uint32_t kv_lo = umma_sw128_lo(smem_u32(smem + kOffKV));
      const uint32_t bar_step = smem_u32(step + 2 * t), bar_e = smem_u32(kv_empty);
      const uint32_t d_o = tmem + o_col<DH>(t);
      // S_{t, j&1} = Q_t K_j^T.
      auto issue_s = [&](int j) {
        const uint32_t d = tmem + s_col(t, j & 1);
        const uint32_t b = kv_lo + (j % kStages3) * kStageLo;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) umma_f16_lo<G::kDescHi>(d, q_lo + 2 * k, b + 2 * k, idesc_qk, k);
        if constexpr (SPLIT == 2) {  // + Q_lo K_hi^T + Q_hi K_lo^T
#pragma unroll
          for (int k = 0; k < kD / 16; ++k) {
            umma_f16_lo<G::kDescHi>(d, q_lo + 2 * kQLo + 2 * k, b + 2 * k, idesc_qk, 1u);
            umma_f16_lo<G::kDescHi>(d, q_lo + 2 * k, b + 2 * kVLo + 2 * k, idesc_qk, 1u);
          }
        }
      };
      bool ok = mbar_wait_hint(q_full, 0, p.err, kDevTimeoutMma, p.wait_mma_ns);
      for (int j = 0; j < 2 && j < nkv && ok; ++j) {
        if (!mbar_wait_hint(&kv_full[j], 0, p.err, kDevTimeoutMma, p.wait_mma_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(j);
        umma_commit_addr(bar_step + 8 * j);
      }
      for (int j = 0; j < nkv && ok; ++j) {
        const int bj = j & 1;
        if (!mbar_wait_hint(&p_full[2 * t + bj], (j >> 1) & 1, p.err, kDevTimeoutMma, p.wait_mma_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // O_t += P_t V_j with P (32 keys = 16 columns of fp16 pairs) read from buffer j & 1.
        const uint32_t v = kv_lo + (j % kStages3) * kStageLo + kVLo;
#pragma unroll
        for (int k = 0; k < kKV / 16; ++k)
          umma_f16_ts_lo<G::kDescHi>(d_o, tmem + s_col(t, bj) + k * 8, v + k * kVStepLo, idesc_pv,
                                     (j > 0 || k > 0) ? 1u : 0u);
        umma_commit_addr(bar_e + 8 * (j % kStages3));
        if (j + 2 < nkv) {
          if (!mbar_wait_hint(&kv_full[(j + 2) % kStages3], ((j + 2) / kStages3) & 1, p.err, kDevTimeoutMma,
                              p.wait_mma_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(j + 2);
        }
        umma_commit_addr(bar_step + 8 * bj);
      }
      if (!ok) {
        umma_commit(&drain[t]);
        mbar_wait_spin(&drain[t], 0, p.err, kDevTimeoutMma);
      }
    }
  } else {
    // ---------------- softmax: thread = query row of tile t ----------------
    const int t = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row inside the tile = TMEM lane
    if (t < ntiles) {
      const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t t_o = tmem + lane_off + o_col<DH>(t);
      const float c = p.scale * kLog2e;
      float mc = -INFINITY;  // running max in the exp2 domain (max score * c)
      float l = 0.0f;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int bj = j & 1;
        if (!mbar_wait_spin(&step[2 * t + bj], (j >> 1) & 1, p.err, kDevTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_s = tmem + lane_off + s_col(t, bj);
        uint32_t pk[16];
        if constexpr (EXP == 3) {
          // No row max per step: P is exponentiated against the running max mc, and the step's
          // row sum tells whether mc has gone stale. Every P value is at most that sum, so while it
          // stays below p.rescale_sum (<= 2^15) P is finite in fp16 and O, l and the log-sum-exp
          // are exact for the stale max. Only a step whose sum exceeds it (any row of the warp)
          // takes the max of its 32 scores, rescales O and l after PV(j - 1) and recomputes P.
          // The FP32-pipe exponentials clamp their argument at 126, so a score far above mc gives
          // a huge but finite P and trips the check like the special-function unit's +inf does.
          uint32_t sv[32];
          const int kvalid = len - j * kKV;  // keys of this tile inside the sequence (> 0)
          // S(j) into registers, keys past the sequence's end at -inf. The refresh path reads it
          // again (P has not been written over it yet), so sv need not outlive the exponentials.
          auto load_s = [&]() {
            tmem_ld32(t_s, sv);
            tmem_ld_wait();
            if (kvalid < kKV) {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (i >= kvalid) sv[i] = __float_as_uint(-INFINITY);
            }
          };
          load_s();
          auto max32 = [&]() {
            float pm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              pm[u] = fmax3f(__uint_as_float(sv[u]), __uint_as_float(sv[u + 8]), __uint_as_float(sv[u + 16]));
#pragma unroll
            for (int u = 0; u < 8; ++u) pm[u] = fmaxf(pm[u], __uint_as_float(sv[u + 24]));
            return fmax3f(fmax3f(pm[0], pm[1], pm[2]), fmax3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7])) * c;
          };
          auto exps = [&]() {
            const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-mc, -mc);
            uint64_t rs2[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) rs2[u] = 0ull;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, nm2), a0, a1);
              const uint64_t e2 = (i & 7) < POLY ? poly_exp2_x2(fminf(a0, 126.0f), fminf(a1, 126.0f))
                                                 : f2_pack(fast_exp2(a0), fast_exp2(a1));
              rs2[i & 3] = f2_add(rs2[i & 3], e2);
              float e0, e1;
              f2_unpack(e2, e0, e1);
              __half2 hv = __floats2half2_rn(e0, e1);
              pk[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
            float r0, r1;
            f2_unpack(f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3])), r0, r1);
            return r0 + r1;
          };
          if (j == 0) mc = max32();
          float ls = exps();
          if (__any_sync(0xffffffffu, !(ls <= p.rescale_sum))) {
            // j >= 1 here: with the exact max of tile 0 every P of step 0 is at most 1.
            load_s();
            const float m_new = fmaxf(mc, max32());
            const float alpha = fast_exp2(mc - m_new);
            if (!mbar_wait_spin(&step[2 * t + ((j - 1) & 1)], (((j - 1) >> 1) + 1) & 1, p.err, kDevTimeoutEpilogue)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll 1
            for (int oc = 0; oc < kD; oc += 16) {
              uint32_t o[16];
              tmem_ld16(t_o + oc, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(t_o + oc, o);
            }
            tmem_st_wait();
            l *= alpha;
            mc = m_new;
            ls = exps();
          }
          l += ls;
        } else {
          uint32_t sv[32];
          tmem_ld32(t_s, sv);
          tmem_ld_wait();
          const int kvalid = len - j * kKV;  // keys of this tile inside the sequence (> 0)
          if (kvalid < kKV) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i >= kvalid) sv[i] = __float_as_uint(-INFINITY);
          }
          float mraw;
          if constexpr (EXP == 0) {
            float pm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pm[u] = fmaxf(__uint_as_float(sv[u]), __uint_as_float(sv[u + 8]));
#pragma unroll
            for (int i = 16; i < 32; ++i) pm[i & 7] = fmaxf(pm[i & 7], __uint_as_float(sv[i]));
            mraw = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
          } else {
            // Three-input maxima: 32 -> 8 -> 3 -> 1.
            float pm[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
              pm[u] = fmax3f(__uint_as_float(sv[u]), __uint_as_float(sv[u + 8]), __uint_as_float(sv[u + 16]));
#pragma unroll
            for (int u = 0; u < 8; ++u) pm[u] = fmaxf(pm[u], __uint_as_float(sv[u + 24]));
            mraw = fmax3f(fmax3f(pm[0], pm[1], pm[2]), fmax3f(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
          }
          const float mx = mraw * c;
          if (j == 0) {
            mc = mx;
          } else if (__any_sync(0xffffffffu, mx - mc > kRescaleThreshold)) {
            // Refresh the max of this warp's rows once O += P(j - 1) V has landed.
            const float m_new = fmaxf(mc, mx);
            const float alpha = fast_exp2(mc - m_new);
            // PV(j - 1) is completion number ((j - 1) >> 1) + 2 of step[(j - 1) & 1]: the phase with
            // 0-based index ((j - 1) >> 1) + 1.
            if (!mbar_wait_spin(&step[2 * t + ((j - 1) & 1)], (((j - 1) >> 1) + 1) & 1, p.err, kDevTimeoutEpilogue)) {
              ok = false;
              break;
            }
            tc_fence_after();
            // 16 columns at a time: the 32 scores of this tile stay live in registers meanwhile.
#pragma unroll 1
            for (int oc = 0; oc < kD; oc += 16) {
              uint32_t o[16];
              tmem_ld16(t_o + oc, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(t_o + oc, o);
            }
            tmem_st_wait();
            l *= alpha;
            mc = m_new;
          }
          // P = exp2(S c - m) as fp16 pairs over the first 16 columns of S_{t,b}.
          if constexpr (EXP == 0) {
            float rs[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
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
            l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
          } else if constexpr (EXP == 1) {
            // Packed FP32 pairs for the scale-and-shift and the row sum.
            const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-mc, -mc);
            uint64_t rs2[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) rs2[u] = 0ull;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, nm2), a0, a1);
              const uint64_t e2 = (i & 7) < POLY ? poly_exp2_x2(a0, a1) : f2_pack(fast_exp2(a0), fast_exp2(a1));
              rs2[i & 3] = f2_add(rs2[i & 3], e2);
              float e0, e1;
              f2_unpack(e2, e0, e1);
              __half2 hv = __floats2half2_rn(e0, e1);
              pk[i] = *reinterpret_cast<uint32_t*>(&hv);
            }
            float r0, r1, r2, r3;
            f2_unpack(f2_add(f2_add(rs2[0], rs2[1]), f2_add(rs2[2], rs2[3])), r0, r1);
            (void)r2;
            (void)r3;
            l += r0 + r1;
          } else {
            // The shifted scores rounded to fp16 pairs and exponentiated two per instruction: P comes
            // out packed, and the step's row sum is accumulated as fp16 pairs (four chains of four
            // pairs, each at most 2^10) before joining the fp32 total.
            const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(-mc, -mc);
            __half2 hs[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) hs[u] = __float2half2_rn(0.0f);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float a0, a1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[2 * i]), __uint_as_float(sv[2 * i + 1])), c2, nm2), a0, a1);
              __half2 ah = __floats2half2_rn(a0, a1);
              pk[i] = ex2_h2(*reinterpret_cast<uint32_t*>(&ah));
              hs[i & 3] = __hadd2(hs[i & 3], *reinterpret_cast<__half2*>(&pk[i]));
            }
            const float2 f01 = __half22float2(hs[0]), f23 = __half22float2(hs[1]);
            const float2 f45 = __half22float2(hs[2]), f67 = __half22float2(hs[3]);
            l += ((f01.x + f01.y) + (f23.x + f23.y)) + ((f45.x + f45.y) + (f67.x + f67.y));
          }

        }
        tmem_st16(t_s, pk);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[2 * t + bj]);
      }
      const int jl = nkv - 1;
      if (ok && mbar_wait_spin(&step[2 * t + (jl & 1)], ((jl >> 1) + 1) & 1, p.err, kDevTimeoutEpilogue)) {
        tc_fence_after();
        const int row = q0 + t * kQ + r;
        const float inv = 1.0f / l;
        const int dh_out = PAD ? p.dh : kD;  // stored columns (the padding is not part of the head)
        __half* dst = p.out + static_cast<size_t>(start + row) * p.d + h * dh_out;
#pragma unroll
        for (int hh = 0; hh < kD / 32; ++hh) {
          uint32_t o[32];
          tmem_ld32(t_o + hh * 32, o);
          tmem_ld_wait();
          if (row < len) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (PAD && 8 * k >= dh_out) break;
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
    tmem_dealloc(tmem, kTmemCols3);
  }
}

template <int DH, int POLY, int EXP, bool PAD = false, int SPLIT = PAD ? 2 : 0>
cudaError_t launch_poly3(const CUtensorMap& tm_q, const CUtensorMap& tm_kv32, const CUtensorMap& tm_qlo,
                         const CUtensorMap& tm_klo, const AttnParams& p, cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};  // one bit per device ordinal
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !(configured.load(std::memory_order_acquire) & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(attention_tc3_kernel<DH, POLY, EXP, PAD, SPLIT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Tc3<DH, SPLIT>::kSmem);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured.fetch_or(1ull << dev, std::memory_order_release);
  }
  dim3 grid(p.n_work, p.H);
  attention_tc3_kernel<DH, POLY, EXP, PAD, SPLIT><<<grid, kThreads3, Tc3<DH, SPLIT>::kSmem, s>>>(tm_q, tm_kv32, tm_qlo,
                                                                                                tm_klo, p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention_tc3(const CUtensorMap& tm_q, const CUtensorMap& tm_kv32, const CUtensorMap& tm_qlo,
                                 const CUtensorMap& tm_klo, const AttnParams& p, int poly_eighths, int exp_mode,
                                 cudaStream_t s) {
  if (p.n_work <= 0) return cudaSuccess;
  if (p.dh == 16 || p.dh == 24) {  // zero-padded to 32 columns by the 3-D maps
    if (exp_mode == 3) return poly_eighths == 0 ? launch_poly3<32, 0, 3, true>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s)
                                                : launch_poly3<32, 2, 3, true>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    if (exp_mode == 1) return poly_eighths == 0 ? launch_poly3<32, 0, 1, true>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s)
                                                : launch_poly3<32, 2, 1, true>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    return launch_poly3<32, 0, 0, true>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
  }
  if (p.dh == 32) {  // the default arithmetic, and scalar FP32 for comparison
    if (exp_mode == 3) return poly_eighths == 0 ? launch_poly3<32, 0, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s)
                                                : launch_poly3<32, 2, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    if (exp_mode == 1) return poly_eighths == 0 ? launch_poly3<32, 0, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s)
                                                : launch_poly3<32, 2, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    return launch_poly3<32, 0, 0>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
  }
  if (p.dh != 64) return cudaErrorInvalidValue;
  if (exp_mode == 2) return launch_poly3<64, 0, 2>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
  if (exp_mode == 3) {
    switch (poly_eighths) {
      case 0: return launch_poly3<64, 0, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      case 1: return launch_poly3<64, 1, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      case 2: return launch_poly3<64, 2, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      default: return launch_poly3<64, 3, 3>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    }
  }
  if (exp_mode == 1) {
    switch (poly_eighths) {
      case 0: return launch_poly3<64, 0, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      case 1: return launch_poly3<64, 1, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      case 2: return launch_poly3<64, 2, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
      default: return launch_poly3<64, 3, 1>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    }
  }
  switch (poly_eighths) {
    case 0: return launch_poly3<64, 0, 0>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    case 1: return launch_poly3<64, 1, 0>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
    default: return launch_poly3<64, 2, 0>(tm_q, tm_kv32, tm_qlo, tm_klo, p, s);
  }
}

}  // namespace esm
