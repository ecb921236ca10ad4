// Bidirectional multi-head attention over packed variable-length sequences, and its contact mode.
//
// Replaces the reference attention loop (src/lib.rs:5206-5301: q.k scores scaled by 1/sqrt(dh),
// softmax over every key of the sequence, P.V) and the contact head
// (accumulate_head_apc, src/lib.rs:5036-5076, called per head at 5303-5312, sigmoid at 5373-5377).
//
// attention_kernel: one CTA per (sequence, 64-query tile, head); 4 warps x 16 query rows; K/V
//   tiles of 64 keys double-buffered with cp.async; S = Q K^T and O = P V on the tensor cores
//   (mma.sync m16n8k16, fp16 in, fp32 accumulate); online softmax in fp32; keys past the
//   sequence's own length are masked, so every sequence is computed exactly as if alone.
//   Writes O (fp16) and the per-row log-sum-exp (for the contact mode).
// contact_accumulate_kernel: one CTA per 64x64 tile of a sequence's L x L map; loops over the
//   layer's heads with a non-zero regression weight, recomputes the normalised probabilities
//   from the saved log-sum-exp, and folds them straight into M += w * P plus the APC row/column
//   sums; no per-head map is ever stored.
// contact_finalize_kernel: C = M + M^T - sum_h (w_h / T_h) r_h r_h^T, sigmoid(C + b).
#include "common.cuh"
#include "kernels.cuh"

namespace esm {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int DH>
struct AttnShape {
  static constexpr int kDHP = (DH + 15) / 16 * 16;  // head dim padded to the MMA K step
  static constexpr int kStr = kDHP + 8;             // smem row stride in halves (conflict-free ldmatrix)
  static constexpr int kChunks = DH / 8;            // 16-byte chunks of real data per row
  static constexpr int kTile = 64 * kStr;           // halves per 64-row tile
};

// Loads rows [row0, row0 + 64) of one head (64 x DH halves) into a padded smem tile; rows at or
// past `len` are zero-filled.
template <int DH>
__device__ __forceinline__ void load_head_tile(__half* s, const __half* g, int row0, int len, int ld, int tid,
                                               int nthreads) {
  using S = AttnShape<DH>;
  for (int idx = tid; idx < 64 * S::kChunks; idx += nthreads) {
    const int r = idx / S::kChunks, c = idx - r * S::kChunks;
    const int row = row0 + r;
    const bool ok = row < len;
    const __half* src = g + static_cast<size_t>(ok ? row : 0) * ld + c * 8;
    cp_async16(s + r * S::kStr + c * 8, src, ok ? 16 : 0);
  }
}

template <int DH>
__device__ __forceinline__ void zero_pad_cols(__half* s, int ntiles, int tid, int nthreads) {
  using S = AttnShape<DH>;
  if constexpr (S::kDHP != DH) {
    for (int idx = tid; idx < ntiles * 64; idx += nthreads) {
      __half* row = s + idx * S::kStr;
      for (int c = DH; c < S::kDHP; ++c) row[c] = __float2half(0.0f);
    }
  }
}

// S(16 x 64) = Q(16 x DHP) . K(64 x DHP)^T for this warp's 16 rows (ACC: S += instead).
template <int DH, bool ACC = false>
__device__ __forceinline__ void qk_tile(float (&s)[8][4], const uint32_t (&qf)[AttnShape<DH>::kDHP / 16][4],
                                        const __half* sK, int lane) {
  using S = AttnShape<DH>;
  if constexpr (!ACC) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
  }
#pragma unroll
  for (int ks = 0; ks < S::kDHP / 16; ++ks) {
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int col = ks * 16 + ((lane >> 3) & 1) * 8;
      ldmatrix_x4(b, sK + key * S::kStr + col);
      mma16816(s[2 * np], qf[ks], b[0], b[1]);
      mma16816(s[2 * np + 1], qf[ks], b[2], b[3]);
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(128) attention_kernel(const AttnParams p) {
  using S = AttnShape<DH>;
  constexpr int DHP = S::kDHP;
  __shared__ __align__(16) __half sQ[S::kTile];
  __shared__ __align__(16) __half sK[2][S::kTile];
  __shared__ __align__(16) __half sV[2][S::kTile];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int2 wk = p.work[blockIdx.x];
  const int b = wk.x, q0 = wk.y * 64, h = blockIdx.y;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int ld = 3 * p.d;
  const __half* Qg = p.qkv + static_cast<size_t>(start) * ld + h * DH;
  const __half* Kg = Qg + p.d;
  const __half* Vg = Qg + 2 * p.d;

  zero_pad_cols<DH>(sQ, 1, tid, 128);
  zero_pad_cols<DH>(&sK[0][0], 2, tid, 128);
  zero_pad_cols<DH>(&sV[0][0], 2, tid, 128);
  __syncthreads();

  load_head_tile<DH>(sQ, Qg, q0, len, ld, tid, 128);
  load_head_tile<DH>(sK[0], Kg, 0, len, ld, tid, 128);
  load_head_tile<DH>(sV[0], Vg, 0, len, ld, tid, 128);
  cp_async_commit();

  const float sl2 = p.scale * kLog2e;
  const int nkv = (len + 63) / 64;
  float o[DHP / 8][4];
#pragma unroll
  for (int i = 0; i < DHP / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};
  uint32_t qf[DHP / 16][4];

  for (int j = 0; j < nkv; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkv) {
      load_head_tile<DH>(sK[buf ^ 1], Kg, (j + 1) * 64, len, ld, tid, 128);
      load_head_tile<DH>(sV[buf ^ 1], Vg, (j + 1) * 64, len, ld, tid, 128);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < DHP / 16; ++ks)
        ldmatrix_x4(qf[ks], sQ + (warp * 16 + (lane & 15)) * S::kStr + ks * 16 + (lane >> 4) * 8);
    }
    float s[8][4];
    qk_tile<DH>(s, qf, sK[buf], lane);

    const int kbase = j * 64;
    if (kbase + 64 > len) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int key = kbase + nt * 8 + (lane & 3) * 2;
        if (key >= len) s[nt][0] = s[nt][2] = -INFINITY;
        if (key + 1 >= len) s[nt][1] = s[nt][3] = -INFINITY;
      }
    }
    // Online softmax (fp32). Rows: r = 0 -> lane/4, r = 1 -> lane/4 + 8.
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * r], s[nt][2 * r + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run[r], mx);
      const float m_scaled = (m_new == -INFINITY) ? 0.0f : m_new * sl2;
      const float alpha = exp2f(m_run[r] * sl2 - m_scaled);
      float rs = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][2 * r] = exp2f(s[nt][2 * r] * sl2 - m_scaled);
        s[nt][2 * r + 1] = exp2f(s[nt][2 * r + 1] * sl2 - m_scaled);
        rs += s[nt][2 * r] + s[nt][2 * r + 1];
      }
      l_run[r] = l_run[r] * alpha + rs;
      m_run[r] = m_new;
#pragma unroll
      for (int i = 0; i < DHP / 8; ++i) {
        o[i][2 * r] *= alpha;
        o[i][2 * r + 1] *= alpha;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack_half2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_half2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nn = 0; nn < DHP / 16; ++nn) {
        uint32_t v[4];
        ldmatrix_x4_trans(v, sV[buf] + (kk * 16 + (lane & 15)) * S::kStr + nn * 16 + (lane >> 4) * 8);
        mma16816(o[2 * nn], a, v[0], v[1]);
        mma16816(o[2 * nn + 1], a, v[2], v[3]);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    float l = l_run[r];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int row = q0 + warp * 16 + (lane >> 2) + 8 * r;
    const float inv = 1.0f / l;
    if (row < len) {
      __half* dst = p.out + static_cast<size_t>(start + row) * p.d + h * DH;
#pragma unroll
      for (int i = 0; i < DHP / 8; ++i) {
        const int col = i * 8 + (lane & 3) * 2;
        if (col < DH) {
          *reinterpret_cast<__half2*>(dst + col) = __floats2half2_rn(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
        }
      }
      if (p.lse && (lane & 3) == 0) p.lse[static_cast<size_t>(h) * p.T + start + row] = m_run[r] * p.scale + logf(l);
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(128) contact_accumulate_kernel(const ContactParams p) {
  using S = AttnShape<DH>;
  constexpr int DHP = S::kDHP;
  __shared__ __align__(16) __half sQ[2][S::kTile];
  __shared__ __align__(16) __half sK[2][S::kTile];
  // With p.qk_lo, the fp16 rounding residues of the same query and key rows: the scores are then
  // Q K^T + Q_lo K^T + Q K_lo^T, as in the tcgen05 attention kernel whose log-sum-exp normalises
  // them here.
  constexpr bool kResidues = DH == 16 || DH == 24;  // the head sizes whose attention splits its scores
  constexpr int kLoTile = kResidues ? S::kTile : 8;
  __shared__ __align__(16) __half sQl[2][kLoTile];
  __shared__ __align__(16) __half sKl[2][kLoTile];
  const bool split = kResidues && p.qk_lo != nullptr;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 tl = p.tiles[blockIdx.x];
  const int b = tl.x, i0 = tl.y * 64, j0 = tl.z * 64;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int n = len - 2;
  const int ld = 3 * p.d;
  const float sl2 = p.scale * kLog2e;

  zero_pad_cols<DH>(&sQ[0][0], 2, tid, 128);
  zero_pad_cols<DH>(&sK[0][0], 2, tid, 128);
  if constexpr (kResidues) {
    if (split) {
      zero_pad_cols<DH>(&sQl[0][0], 2, tid, 128);
      zero_pad_cols<DH>(&sKl[0][0], 2, tid, 128);
    }
  }
  __syncthreads();
  const int ld_lo = 2 * p.d;
  // Queries and keys of head h (and their residues) for rows i0.. and j0.. into buffer `buf`.
  auto load_tiles = [&](int h, int buf) {
    const __half* Qg = p.qkv + static_cast<size_t>(start) * ld + h * DH;
    load_head_tile<DH>(sQ[buf], Qg, i0, len, ld, tid, 128);
    load_head_tile<DH>(sK[buf], Qg + p.d, j0, len, ld, tid, 128);
    if constexpr (kResidues) {
      if (split) {
        const __half* Lg = p.qk_lo + static_cast<size_t>(start) * ld_lo + h * DH;
        load_head_tile<DH>(sQl[buf], Lg, i0, len, ld_lo, tid, 128);
        load_head_tile<DH>(sKl[buf], Lg + p.d, j0, len, ld_lo, tid, 128);
      }
    }
    cp_async_commit();
  };

  // Heads that contribute (non-zero regression weight), up to 64; with several CTAs per tile
  // (gridDim.y = head groups, when a layer has too few tiles to fill the GPU) this CTA takes every
  // gridDim.y-th of them.
  int heads[64];
  int nh = 0, seen = 0;
  for (int h = 0; h < p.H && h < 64; ++h)
    if (p.w_layer[h] != 0.0f && seen++ % gridDim.y == blockIdx.y) heads[nh++] = h;

  float acc[8][4];
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;

  if (nh > 0) {
    load_tiles(heads[0], 0);
    const int g = lane >> 2;
    const int row_a = i0 + warp * 16 + g;  // token rows held by this thread (and row_a + 8)
    for (int t = 0; t < nh; ++t) {
      const int h = heads[t];
      const int buf = t & 1;
      if (t + 1 < nh) {
        load_tiles(heads[t + 1], buf ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      uint32_t qf[DHP / 16][4];
#pragma unroll
      for (int ks = 0; ks < DHP / 16; ++ks)
        ldmatrix_x4(qf[ks], sQ[buf] + (warp * 16 + (lane & 15)) * S::kStr + ks * 16 + (lane >> 4) * 8);
      float s[8][4];
      qk_tile<DH>(s, qf, sK[buf], lane);
      if constexpr (kResidues) {
        if (split) {
          qk_tile<DH, true>(s, qf, sKl[buf], lane);  // + Q K_lo^T
#pragma unroll
          for (int ks = 0; ks < DHP / 16; ++ks)
            ldmatrix_x4(qf[ks], sQl[buf] + (warp * 16 + (lane & 15)) * S::kStr + ks * 16 + (lane >> 4) * 8);
          qk_tile<DH, true>(s, qf, sK[buf], lane);  // + Q_lo K^T
        }
      }

      const float w = p.w_layer[h];
      const float* lse = p.lse + static_cast<size_t>(h) * p.T + start;
      const float l0 = (row_a < len) ? lse[row_a] * kLog2e : 0.0f;
      const float l1 = (row_a + 8 < len) ? lse[row_a + 8] * kLog2e : 0.0f;
      const bool inner0 = row_a >= 1 && row_a <= n;
      const bool inner1 = row_a + 8 >= 1 && row_a + 8 <= n;
      float rsum0 = 0.0f, rsum1 = 0.0f;
      float* rh = p.r + p.r_off[b] + static_cast<size_t>(p.head_base + h) * n;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = j0 + nt * 8 + (lane & 3) * 2;
        const bool cin0 = col >= 1 && col <= n;
        const bool cin1 = col + 1 >= 1 && col + 1 <= n;
        // Normalised probabilities of the inner block only (zero elsewhere).
        const float p00 = (inner0 && cin0) ? exp2f(s[nt][0] * sl2 - l0) : 0.0f;
        const float p01 = (inner0 && cin1) ? exp2f(s[nt][1] * sl2 - l0) : 0.0f;
        const float p10 = (inner1 && cin0) ? exp2f(s[nt][2] * sl2 - l1) : 0.0f;
        const float p11 = (inner1 && cin1) ? exp2f(s[nt][3] * sl2 - l1) : 0.0f;
        acc[nt][0] += w * p00;
        acc[nt][1] += w * p01;
        acc[nt][2] += w * p10;
        acc[nt][3] += w * p11;
        rsum0 += p00 + p01;
        rsum1 += p10 + p11;
        // Column sums over this warp's 16 rows: reduce across the 8 row groups (lane bits 2..4).
        float c0 = p00 + p10, c1 = p01 + p11;
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          c0 += __shfl_xor_sync(0xffffffffu, c0, o);
          c1 += __shfl_xor_sync(0xffffffffu, c1, o);
        }
        if (g == 0) {
          if (cin0 && c0 != 0.0f) atomicAdd(rh + (col - 1), c0);
          if (cin1 && c1 != 0.0f) atomicAdd(rh + (col + 1 - 1), c1);
        }
      }
      rsum0 += __shfl_xor_sync(0xffffffffu, rsum0, 1);
      rsum0 += __shfl_xor_sync(0xffffffffu, rsum0, 2);
      rsum1 += __shfl_xor_sync(0xffffffffu, rsum1, 1);
      rsum1 += __shfl_xor_sync(0xffffffffu, rsum1, 2);
      if ((lane & 3) == 0) {
        if (inner0) atomicAdd(rh + (row_a - 1), rsum0);
        if (inner1) atomicAdd(rh + (row_a + 8 - 1), rsum1);
      }
      __syncthreads();
    }
    // M[i-1, j-1] += acc over the inner block: a plain update when one CTA owns the tile, an
    // atomic one when the tile's heads are split over several CTAs.
    float* M = p.M + p.m_off[b];
    const bool shared_tile = gridDim.y > 1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = j0 + nt * 8 + (lane & 3) * 2;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = row_a + 8 * r;
        if (row < 1 || row > n) continue;
        float* mrow = M + static_cast<size_t>(row - 1) * n;
        if (shared_tile) {
          if (col >= 1 && col <= n) atomicAdd(mrow + col - 1, acc[nt][2 * r]);
          if (col + 1 >= 1 && col + 1 <= n) atomicAdd(mrow + col, acc[nt][2 * r + 1]);
        } else {
          if (col >= 1 && col <= n) mrow[col - 1] += acc[nt][2 * r];
          if (col + 1 >= 1 && col + 1 <= n) mrow[col] += acc[nt][2 * r + 1];
        }
      }
    }
  }
}

// a[b, hl] = w_hl / T_hl with T_hl = sum_i r[b, hl, i]; 0 when w == 0 or |T| <= 1e-12
// (the skip and the inv_total guard of accumulate_head_apc, src/lib.rs:5043-5045, 5061-5065).
__global__ void contact_head_scale_kernel(const float* r, const int64_t* r_off, const int32_t* cu, int n_heads_total,
                                          const float* w_all, float* a) {
  const int hl = blockIdx.x, b = blockIdx.y;
  const int n = cu[b + 1] - cu[b] - 2;
  float s = 0.0f;
  if (n > 0) {
    const float* rh = r + r_off[b] + static_cast<size_t>(hl) * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += rh[i];
  }
  __shared__ float red[8];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    const float wv = w_all[hl];
    a[static_cast<size_t>(b) * n_heads_total + hl] = (wv != 0.0f && fabsf(t) > 1e-12f) ? wv / t : 0.0f;
  }
}

// One CTA per 64x64 output tile of one sequence: APC correction as a K = n_heads_total rank
// update from shared-memory tiles, then the symmetrisation and the sigmoid.
__global__ void __launch_bounds__(256) contact_finalize_kernel(const float* M, const float* r, const int64_t* m_off,
                                                               const int64_t* r_off, const int32_t* cu,
                                                               int n_heads_total, const float* a, float bias,
                                                               float* out) {
  const int b = blockIdx.z;
  const int n = cu[b + 1] - cu[b] - 2;
  const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
  if (n <= 0 || i0 >= n || j0 >= n) return;
  __shared__ float Ri[32][65];
  __shared__ float Rj[32][65];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const float* rb = r + r_off[b];
  const float* ab = a + static_cast<size_t>(b) * n_heads_total;
  for (int k0 = 0; k0 < n_heads_total; k0 += 32) {
    for (int idx = threadIdx.x; idx < 32 * 64; idx += 256) {
      const int kk = idx >> 6, c = idx & 63;
      const int hl = k0 + kk;
      float vi = 0.0f, vj = 0.0f;
      if (hl < n_heads_total) {
        const float* rh = rb + static_cast<size_t>(hl) * n;
        if (i0 + c < n) vi = rh[i0 + c] * ab[hl];
        if (j0 + c < n) vj = rh[j0 + c];
      }
      Ri[kk][c] = vi;
      Rj[kk][c] = vj;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      float x[4], y[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        x[u] = Ri[kk][ty * 4 + u];
        y[u] = Rj[kk][tx * 4 + u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] += x[u] * y[v];
    }
    __syncthreads();
  }
  const float* Mb = M + m_off[b];
  float* ob = out + m_off[b];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty * 4 + u;
    if (i >= n) continue;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int jj = j0 + tx * 4 + v;
      if (jj >= n) continue;
      const float c = Mb[static_cast<size_t>(i) * n + jj] + Mb[static_cast<size_t>(jj) * n + i] - acc[u][v];
      ob[static_cast<size_t>(i) * n + jj] = 1.0f / (1.0f + expf(-(c + bias)));
    }
  }
}

template <int DH>
cudaError_t launch_attention_dh(const AttnParams& p, cudaStream_t s) {
  dim3 grid(p.n_work, p.H);
  attention_kernel<DH><<<grid, 128, 0, s>>>(p);
  return cudaGetLastError();
}

template <int DH>
cudaError_t launch_contact_dh(const ContactParams& p, cudaStream_t s) {
  const int groups = p.head_groups > 1 ? p.head_groups : 1;
  contact_accumulate_kernel<DH><<<dim3(p.n_tiles, groups), 128, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention(const AttnParams& p, cudaStream_t s) {
  if (p.n_work <= 0) return cudaSuccess;
  switch (p.dh) {
    case 16: return launch_attention_dh<16>(p, s);
    case 24: return launch_attention_dh<24>(p, s);
    case 32: return launch_attention_dh<32>(p, s);
    case 64: return launch_attention_dh<64>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_contact_accumulate(const ContactParams& p, cudaStream_t s) {
  if (p.n_tiles <= 0) return cudaSuccess;
  if (p.H > 64) return cudaErrorInvalidValue;
  switch (p.dh) {
    case 16: return launch_contact_dh<16>(p, s);
    case 24: return launch_contact_dh<24>(p, s);
    case 32: return launch_contact_dh<32>(p, s);
    case 64: return launch_contact_dh<64>(p, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_contact_finalize(const float* M, const float* r, const int64_t* m_off, const int64_t* r_off,
                                    const int32_t* cu_seqlens, int B, int max_n, int n_heads_total, const float* w_all,
                                    float bias, float* a_scratch, float* out, cudaStream_t s) {
  if (B <= 0 || max_n <= 0) return cudaSuccess;
  contact_head_scale_kernel<<<dim3(n_heads_total, B), 256, 0, s>>>(r, r_off, cu_seqlens, n_heads_total, w_all,
                                                                    a_scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int t = (max_n + 63) / 64;
  contact_finalize_kernel<<<dim3(t, t, B), 256, 0, s>>>(M, r, m_off, r_off, cu_seqlens, n_heads_total, a_scratch,
                                                        bias, out);
  return cudaGetLastError();
}

}  // namespace esm
