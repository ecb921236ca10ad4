// Host-side interface of the tcgen05 GEMM used for every projection of the encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace esm {

// What the epilogue does with acc = A[m,:] . B[n,:] (fp32, from TMEM) for output element (m, n).
enum GemmEpilogue : int {
  kEpiQkvRope = 0,  // out f16 = rope(acc + bias) for n < rope_cols, acc + bias otherwise
  kEpiGeluF16 = 1,  // out f16 = gelu(acc + bias)
  kEpiResidF32 = 2, // out f32 += acc + bias            (residual stream update)
  kEpiGeluF32 = 3,  // out f32 = gelu(acc + bias)
  kEpiStoreF32 = 4, // out f32 = acc + bias
  kEpiStoreF16 = 5, // out f16 = acc + bias (the V columns of the QKV epilogue)
};

struct GemmParams {
  int M, N, K;
  int num_m_blocks, num_n_blocks;
  const float* bias;    // [N], may be null
  void* out;            // row-major, `ldo` elements per row
  int ldo;
  const int* pos;       // [M] token position inside its sequence (kEpiQkvRope)
  const float2* rope;   // [max_pos, dh/2] (cos, sin) in f32 (kEpiQkvRope)
  int rope_cols;        // columns [0, rope_cols) are rotated (kEpiQkvRope)
  int* err;             // device error word
  // kEpiQkvRope with head_dim 16 / 24, optional: the rounding residue v - fp16(v) of every rotated
  // (query and key) column, as fp16, at lo[m * lo_ld + n] for n < rope_cols.
  __half* lo;
  int lo_ld;
};

// Encodes a 2-D fp16 tensor map over a row-major [rows, cols] matrix with `ld` elements per row,
// box = [box_rows, 64 columns], 128-byte swizzle, zero fill outside the matrix.
bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                   uint32_t box_rows);

// Same with an explicit box width (box_cols fp16 columns) and swizzle (64 or 128 bytes).
bool make_tmap_f16_box(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                       uint32_t box_rows, uint32_t box_cols, int swizzle_bytes);
// fp16 map over the heads of a [rows, ld] matrix whose columns are `heads` consecutive heads of
// head_dim (16 or 24) elements: a 3-D view [rows][heads][head_dim] with boxes of 32 x 1 x box_rows
// and 64-byte swizzle, so each row of a head lands in shared memory zero-padded to 32 elements
// (the elements past head_dim are outside the tensor and the TMA fills them with zeros).
bool make_tmap_f16_heads(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads, uint32_t head_dim,
                         uint64_t ld, uint32_t box_rows);

// Tensor map for the epilogue's bulk stores: a row-major [rows, cols] matrix of fp16 (elem_bytes 2)
// or fp32 (4), box = [32 rows, 64 bytes], 64-byte swizzle.
bool make_tmap_out(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols, uint64_t ld);

// Tile width that divides N (and is a multiple of `head_dim` when non-zero): the widest multiple of
// 64 among 256/192/128 when one fits, else 240 or 160.
int gemm_pick_bn(int N, int head_dim);
// Same, including the narrow widths (96..16) that only the kEpiStoreF32 epilogue supports.
int gemm_pick_bn_any(int N);

// C[M, N] = A[M, K] . B[N, K]^T with the requested epilogue; A and B are fp16 K-major behind the
// tensor maps (A box 128 rows, B box bn/2 rows). Persistent grid of at most num_sms CTAs; with
// cta_pair != 0 (and bn >= 128, M > 128) tiles of 256 rows run on CTA pairs (tcgen05 cta_group::2).
// `tout` (may be null) describes the output for the fp16 (kEpiQkvRope with head_dim 32 / 64,
// kEpiGeluF16) and residual (kEpiResidF32) epilogues: with it those epilogues stage each
// 32-row x 64-byte block in shared memory and write it with one bulk tensor store (or an L2
// reduce-add for the residual), instead of per-thread stores to 32 different rows.
cudaError_t gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, int bn, int epi,
                        int head_dim, GemmParams p, int num_sms, cudaStream_t stream, int cta_pair);

}  // namespace esm
