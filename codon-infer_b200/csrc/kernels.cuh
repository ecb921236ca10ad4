// Launchers of the memory-bound kernels around the GEMMs and of the attention kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace esm {

// Quantized matrices stay on the device in their on-disk CODQ layout: arrays of BlockQ8_0
// {f32 d; i8 qs[32]} (36 B) or BlockQ4_0 {f32 d; u8 qs[16]} (20 B, low nibble = element j, high
// nibble = element j + 16, value = (q - 8) * d), 32 elements per block along the input dimension
// (src/lib.rs:640-645, 1043-1051). Blocks are 4-byte aligned and read with 32-bit loads.
constexpr int kQ8BlockBytes = 36;
constexpr int kQ4BlockBytes = 20;

// One layer's weight matrices for the dequantizing conversion to fp16 (dtype = ESM_DTYPE_*):
// q, k, v, o, fc1, fc2 as fp32 arrays (dtype 0) or block arrays (dtype 1 / 2).
struct LayerSrc {
  int dtype[6];      // storage type of each matrix (a Q3_LUT model mixes Q4_0 and Q3_LUT)
  const void* w[6];
  int64_t elems[6];  // element count of each matrix
};

// Per-sequence bookkeeping: pos[t] (token index inside its sequence), seq_of[t], and the
// token-dropout embedding scale of each sequence (src/lib.rs:5115-5117).
cudaError_t launch_seq_setup(const int32_t* tokens, const int32_t* cu_seqlens, int B, int32_t* pos, int32_t* seq_of,
                             float* embed_scale, cudaStream_t s);

// x[t] = E[tok]*scale (0 for <mask>) in fp32, then xn = LN(x; ln_w, ln_b) in fp16.
// E is fp32 [V, d] (emb_f32 != null) or BlockQ8_0 blocks [V, d/32] (emb_q8). A token id outside
// [0, V) is never used as an index: its row is embedded as zeros and kDevBadToken is set in *err.
cudaError_t launch_embed_ln(const int32_t* tokens, const int32_t* seq_of, const float* embed_scale,
                            const float* emb_f32, const void* emb_q8, int V, int T, int d, const float* ln_w,
                            const float* ln_b, float* x, __half* xn, int* err, cudaStream_t s);

// out16 = LN(x) in fp16 (row stride ld16) and, when out32 != null, also in fp32 ([T, d]).
cudaError_t launch_layernorm(const float* x, int T, int d, const float* w, const float* b, __half* out16, int ld16,
                             float* out32, cudaStream_t s);

// Converts one layer's six weight matrices to fp16 (q|k|v stacked into wqkv).
cudaError_t launch_dequant_layer(const LayerSrc& src, __half* wqkv, __half* wo, __half* w1, __half* w2,
                                 cudaStream_t s);

// Generic converter of a whole matrix (fp32 or blocks) to fp16 / fp32 (load-time use).
cudaError_t launch_to_f16(int dtype, const void* src, int64_t elems, __half* dst, cudaStream_t s);
cudaError_t launch_to_f32(int dtype, const void* src, int64_t elems, float* dst, cudaStream_t s);

// Padded [B, Lmax] int32 tokens -> packed [T] following cu_seqlens.
cudaError_t launch_gather_tokens(const int32_t* padded, const int32_t* cu_seqlens, int B, int Lmax, int32_t* packed,
                                 cudaStream_t s);
// Packed per-sequence n_b x n_b maps -> padded [B, Lmax-2, Lmax-2] (zero outside each map).
cudaError_t launch_scatter_maps(const float* src, const int64_t* m_off, const int32_t* cu_seqlens, int B, int Lmax,
                                float* dst, cudaStream_t s);

// logits[t, :] = (do_ln ? LN(in[t]; ln_w, ln_b) : in[t]) . W^T + bias   (W fp32 [V, d], bias may be null)
cudaError_t launch_lm_decoder(const float* in, int T, int d, int do_ln, const float* ln_w, const float* ln_b,
                              const float* W, const float* bias, int V, float* logits, cudaStream_t s);

// Packed rows [T, C] -> padded [B, Lmax, C] (padding rows zeroed).
cudaError_t launch_scatter_rows(const float* src, const int32_t* cu_seqlens, int B, int Lmax, int C, float* dst,
                                cudaStream_t s);

// Masked-marginal scores of n variants (run_pipeline_dms_with_mode, src/pipeline.rs:111-174):
// for variant v, logits row tok_row[v] of the packed [*, V] logits -> log_softmax_canonical over
// ids 4..=23 (src/lib.rs:4426-4441), Shannon entropy, and deltas[v, c] = logP(aa_c) - logP(wt) in
// CANONICAL_AAS order (src/benchmark.rs:702-707), 0 for the wild type.
cudaError_t launch_dms_score(const float* logits, int V, const int32_t* tok_row, const int32_t* wt_tok, int n,
                             float* deltas, float* entropy, cudaStream_t s);

// One thread waits, with the kernels' bounded mbarrier wait and a limit of `limit_ns`, on a phase
// that nothing completes; on timeout it records kDevTimeoutProbe in *err and returns.
cudaError_t launch_wait_probe(int* err, uint64_t limit_ns, cudaStream_t s);

// ---- attention ------------------------------------------------------------------------------
struct AttnParams {
  const __half* qkv;       // [T, 3d]: q | k | v, head h at columns h*dh of each part
  __half* out;             // [T, d]
  float* lse;              // [H, T] natural-log row log-sum-exp of the scaled scores, or null
  const int32_t* cu_seqlens;
  const int2* work;        // (sequence, 64-row query tile) pairs
  int n_work;
  int T, d, H, dh;
  float scale;             // 1/sqrt(dh)
  int* err;                // device error word (bounded waits of the tcgen05 kernel)
  // tcgen05 kernel, exp_mode 3: a 32-key step whose row sum against the running max exceeds this
  // (>= 64) refreshes the max; it also bounds every P value, which must stay finite in fp16.
  float rescale_sum;
  // tcgen05 kernel: suspension hint (ns, 0 = spin) of the MMA issuers' waits, so that the issuers
  // take few issue slots from the softmax warps that share their sub-partitions.
  uint32_t wait_mma_ns;
};
// mma.sync attention (attention.cu): work items are (sequence, 64-row query tile); any head_dim
// that is a multiple of 8 up to 64.
cudaError_t launch_attention(const AttnParams& p, cudaStream_t s);
// BlockQ8_0 / BlockQ4_0 quantization of nblocks x 32 FP32 values on the device (quantize.cu);
// dtype 1 = Q8_0, 2 = Q4_0; src 16-byte aligned, dst 4-byte aligned.
cudaError_t launch_quantize(int dtype, const float* src, int64_t nblocks, uint8_t* dst, cudaStream_t s);
// Top-k ranking of contact pairs (contact_rank.cu): keys of the first k (<= 4096) candidate pairs
// (j >= i + min_sep) of the n x n map in the reference's order, into out_keys (ascending).
int64_t contact_rank_scratch_keys(int n, int k);
cudaError_t launch_contact_rank(const float* map, int n, int min_sep, int k, uint64_t* scratch, uint64_t* out_keys,
                                cudaStream_t s);
// tcgen05 attention for head_dim 64 or 32 (attention_tc3.cu): work items are (sequence, 256-row
// query block); two 128-row query tiles share every 32-key K/V tile and have two score buffers
// each. tm_q: qkv map with head_dim-column boxes of 128 rows; tm_kv32: the same with 32 rows
// (128- or 64-byte swizzle). poly_eighths (0..3) of the exponential pairs run on the FP32 pipe;
// exp_mode: 0 scalar FP32, 1 packed FP32 pairs, 2 fp16-pair exponentials, 3 packed FP32 pairs
// against the running max without a per-step row max (refreshed when the row sum says so).
// head_dim 16 / 24 (zero-padded to 32): tm_qlo / tm_klo map the fp16 rounding residues of the
// queries and keys ([rows][2 H][head_dim], 128- and 32-row boxes) for split-precision scores; for
// the other head sizes they are not read (pass tm_q / tm_kv32).
cudaError_t launch_attention_tc3(const CUtensorMap& tm_q, const CUtensorMap& tm_kv32, const CUtensorMap& tm_qlo,
                                 const CUtensorMap& tm_klo, const AttnParams& p, int poly_eighths, int exp_mode,
                                 cudaStream_t s);


// Contact mode of the attention (per layer): for each head with a non-zero regression weight w,
// recomputes P = softmax(q k^T * scale) tile by tile from the saved LSE, adds w * P into the
// per-sequence accumulator M[n, n] (inner block, <cls>/<eos> removed) and the head's row and column
// sums of P into r[head, n] (for APC). Nothing per-head is stored.
struct ContactParams {
  const __half* qkv;
  const float* lse;        // [H, T]
  const int32_t* cu_seqlens;
  const int4* tiles;       // (sequence, i-tile, j-tile, unused) over each sequence's L x L map
  int n_tiles;
  int T, d, H, dh;
  float scale;
  const float* w_layer;    // [H] regression weights of this layer
  const int64_t* m_off;    // [B] float offset of sequence b's M (and output map)
  float* M;                // sum over heads of w * P (inner block)
  const int64_t* r_off;    // [B] float offset of sequence b's r block ([n_heads_total, n_b])
  float* r;
  int head_base;           // layer * H
  int* err;                // device error word (bounded waits of the tensor-core kernel)
  int head_groups;         // mma.sync kernel: the contributing heads are split over this many CTAs per tile
  const __half* qk_lo;     // mma.sync kernel, optional: fp16 residues of the queries and keys ([T, 2d])
};
cudaError_t launch_contact_accumulate(const ContactParams& p, cudaStream_t s);

// Tensor-core contact accumulation for head_dim 64 (contact_tc.cu): tiles of 128 keys x 64
// queries, M accumulated transposed. contact_tc_tiles writes sequence b's tile list to `out` (if
// not null) and returns its length. tm_k128 / tm_q64: qkv [T, 3d] maps with 64-column boxes of 128
// and 64 rows.
int contact_tc_tiles(int len, int4* out, int b);
// Also launches the row-sum pass (contact_rowsum_kernel; seq_of [T] maps a token to its sequence).
cudaError_t launch_contact_tc(const CUtensorMap& tm_k128, const CUtensorMap& tm_q64, const ContactParams& p,
                              const int32_t* seq_of, cudaStream_t s);

// contacts = sigmoid(M + M^T - sum_h a_h r_h r_h^T + b) with a_h = w_h / T_h (APC), per sequence.
cudaError_t launch_contact_finalize(const float* M, const float* r, const int64_t* m_off, const int64_t* r_off,
                                    const int32_t* cu_seqlens, int B, int max_n, int n_heads_total, const float* w_all,
                                    float bias, float* a_scratch, float* out, cudaStream_t s);

}  // namespace esm
