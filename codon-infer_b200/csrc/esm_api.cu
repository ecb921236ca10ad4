// C ABI of the B200 ESM-2 encoder forward: context, weight upload, workspace, and the per-layer
// launch sequence that replaces codon-infer's forward_bidirectional* (src/lib.rs:5078-6147).
//
// Per layer (stream-ordered, no host synchronisation):
//   dequantize the layer's six matrices to fp16 (L2-resident scratch)
//   LN1 -> QKV GEMM (+bias, +RoPE) -> attention (-> contact accumulation) -> Wo GEMM (+bias, += x)
//   LN2 -> fc1 GEMM (+bias, GELU) -> fc2 GEMM (+bias, += x)
// then LN_f, the LM head (dense GEMM + GELU, LN + decoder) and, with contacts, the APC finalize.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/esm_b200.h"
#include "common.cuh"
#include "formats.h"
#include "gemm_tc.cuh"
#include "kernels.cuh"

using esm::CodqHeader;

struct esm_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 148;
  int cta_pair = 1;  // GEMM tiles on CTA pairs (cta_group::2); ESM_GEMM_CTA_PAIR=0 selects single CTAs
  // Attention kernel for head_dim 64 and 32 (ESM_ATTN_TC): 3 = tcgen05, two 128-row query tiles
  // per CTA sharing 32-key K/V tiles, two score buffers per tile (the default); 0 = the mma.sync
  // kernel (also the one for head_dim 16 and 24).
  int attn_tc = 3;
  // Eighths of the softmax exponentials on the FP32 pipe (ESM_ATTN_POLY, 0..3); -1 = the kernel's
  // measured best (2 with packed arithmetic, 0 otherwise).
  int attn_poly = -1;
  // Softmax arithmetic (ESM_ATTN_EXP): 0 scalar FP32, 1 packed FP32 pairs with a row max per
  // 32-key step, 2 fp16-pair exponentials, 3 packed FP32 pairs against the running max with the
  // max refreshed only when a step's row sum exceeds attn_rescale_sum (default, measured fastest:
  // about 4 % less attention time than 1 at c4).
  int attn_exp = 3;
  // exp_mode 3: the row-sum bound of a 32-key step above which the running max is refreshed
  // (ESM_ATTN_RESCALE_SUM, 64 .. 32768; small values exercise the refresh path in the tests).
  float attn_rescale_sum = 32768.0f;
  // Suspension hint (ns) of the tcgen05 attention kernel's MMA-issuer waits (ESM_ATTN_WAIT_MMA;
  // 0 = spin). 64 ns measured about 2 % less attention time than spinning at c4; 256 ns was slower.
  uint32_t attn_wait_mma = 64;
  int contact_tc = 1;  // tcgen05 contact accumulation for head_dim 64 (ESM_CONTACT_TC=0: mma.sync kernel)
  std::mutex mu;
  std::string err;
  int* d_err = nullptr;

  // ---- weights ----
  bool loaded = false;
  esm_config cfg{};
  int dtype = 0;
  std::vector<void*> w_allocs;
  void* w[ESM_NUM_TENSORS] = {};
  int64_t classifier_floats = 0;
  bool has_head = false;
  float* bqkv = nullptr;         // [nl, 3d]
  float* emb_f32 = nullptr;      // [V, d] fp32 embedding (dequantized copy for Q8 models)
  __half* dense16 = nullptr;     // LM-head dense weight in fp16 [d, d]
  // Per-layer fp16 weight scratch, two sets: layer l + 1 is dequantised into set (l + 1) & 1 on
  // the side stream while layer l computes with set l & 1.
  __half* wqkv16[2] = {};
  __half* wo16[2] = {};
  __half* w116[2] = {};
  __half* w216[2] = {};
  CUtensorMap tm_wqkv[2], tm_wo[2], tm_w1[2], tm_w2[2], tm_dense;
  // The side stream of the dequantisation and its events: ev_deq[b] = set b written, ev_read[b] =
  // the layer that read set b is done. ESM_DEQUANT_OVERLAP=0 dequantises in the forward's stream.
  int deq_overlap = 1;
  cudaStream_t side = nullptr;
  cudaEvent_t ev_start = nullptr, ev_deq[2] = {}, ev_read[2] = {};
  int bn_qkv = 0, bn_o = 0, bn_fc1 = 0, bn_fc2 = 0, bn_dense = 0;

  // ---- contact head ----
  bool has_ch = false;
  float ch_b = 0.0f;
  float* d_ch_w = nullptr;

  // ---- workspace ----
  int cap_tokens = 0, cap_seqs = 0, cap_len = 0;
  bool cap_contacts = false;
  int64_t cap_rows = 0, work_cap = 0, tiles_cap = 0, m_cap = 0, r_cap = 0;
  std::vector<void*> ws_allocs;
  float* x = nullptr;
  __half* xn = nullptr;
  __half* qkv = nullptr;
  // head_dim 16 / 24: fp16 rounding residues of the rotated queries and keys, [rows][2 d] (queries
  // then keys, per head as in qkv), for the attention's split-precision scores
  __half* qk_lo = nullptr;
  __half* ao = nullptr;
  __half* hb = nullptr;
  float* headf = nullptr;
  float* hidden = nullptr;
  float* logits = nullptr;
  float* lse = nullptr;
  float2* rope = nullptr;
  int32_t* pos = nullptr;
  int32_t* seq_of = nullptr;
  int32_t* tokens = nullptr;
  int32_t* cu = nullptr;
  float* escale = nullptr;
  int2* work = nullptr;
  int2* work256 = nullptr;
  int4* ctiles = nullptr;
  int64_t* m_off = nullptr;
  int64_t* r_off = nullptr;
  float* M = nullptr;
  float* r = nullptr;
  float* a_scr = nullptr;
  float* cmap = nullptr;
  CUtensorMap tm_xn, tm_ao, tm_hb;
  CUtensorMap tm_qkv_q, tm_qkv_kv;  // qkv [T, 3d] with 64-column boxes of 128 / 64 rows
  CUtensorMap tm_qkv_q32, tm_qkv_kv32;  // the same with 32-column boxes (head_dim 32)
  CUtensorMap tm_qkv_kv_r32;    // 64-column boxes of 32 rows (32-key K/V tiles, head_dim 64)
  CUtensorMap tm_qkv_kv32_r32;  // 32-column boxes of 32 rows, 64-byte swizzle (head_dim 32)
  // head_dim 16 / 24: 3-D views [rows][3 H][head_dim] with 32-wide boxes of 128 / 32 rows, which
  // zero-pad every head to 32 columns for the head_dim-32 attention tiles
  CUtensorMap tm_qkv_hq, tm_qkv_hkv;
  CUtensorMap tm_lo_q, tm_lo_k;  // the same views of qk_lo ([rows][2 H][head_dim])
  // pinned staging of the per-call plan, and the event that says it may be rewritten
  int32_t* h_cu = nullptr;
  int2* h_work = nullptr;
  int2* h_work256 = nullptr;
  int4* h_tiles = nullptr;
  int64_t* h_moff = nullptr;
  int64_t* h_roff = nullptr;
  cudaEvent_t plan_ev = nullptr;
  std::vector<int32_t> plan_key;
  int plan_work = 0, plan_work256 = 0, plan_tiles = 0;
  // instrumentation: CUDA event pairs around each launch while profiling is on
  struct ProfRec {
    cudaEvent_t a, b;
    int kind;
    double flops, bytes;
  };
  bool prof = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<ProfRec> prof_recs;
  // host-API staging (grows on demand)
  uint64_t* d_rank = nullptr;  // contact-pair ranking scratch (grown on demand)
  size_t rank_cap = 0;
  int32_t* d_padded_tokens = nullptr;
  size_t padded_tok_cap = 0;
  float* d_padded_out = nullptr;
  size_t padded_out_cap = 0;
  // per-layer residual states of esm_forward_ext (grows on demand)
  float* d_layers = nullptr;
  size_t layer_cap = 0;
  // mutational-scan staging (grows on demand): tok_row, wt_tok, deltas, entropy
  void* d_dms = nullptr;
  size_t dms_cap = 0;
};

namespace {

int fail(esm_ctx* c, int code, const std::string& msg) {
  if (c) c->err = msg;
  return code;
}

#define ESM_CUDA(call)                                                                          \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess)                                                                      \
      return fail(c, e_ == cudaErrorMemoryAllocation ? ESM_ENOMEM : ESM_ECUDA,                  \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                          \
  } while (0)

template <typename T>
int dev_alloc(esm_ctx* c, std::vector<void*>& list, T** out, size_t count) {
  void* p = nullptr;
  const size_t bytes = std::max<size_t>(count * sizeof(T), 256);
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(c, ESM_ENOMEM, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
  list.push_back(p);
  *out = static_cast<T*>(p);
  return ESM_OK;
}

void free_list(std::vector<void*>& list) {
  for (void* p : list) cudaFree(p);
  list.clear();
}

void free_pinned(esm_ctx* c) {
  for (void* p : {static_cast<void*>(c->h_cu), static_cast<void*>(c->h_work),
                  static_cast<void*>(c->h_work256),
                  static_cast<void*>(c->h_tiles), static_cast<void*>(c->h_moff), static_cast<void*>(c->h_roff)})
    if (p) cudaFreeHost(p);
  c->h_cu = nullptr;
  c->h_work = nullptr;
  c->h_work256 = nullptr;
  c->h_tiles = nullptr;
  c->h_moff = nullptr;
  c->h_roff = nullptr;
}

bool shape_supported(const esm_config& c, std::string* why) {
  const int d = c.dim, H = c.n_heads;
  if (d <= 0 || H <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.vocab_size <= 0) {
    *why = "non-positive dimension";
    return false;
  }
  if (d % 32 || c.hidden_dim % 32) {
    *why = "dim and hidden_dim must be multiples of 32 (Q-block size)";
    return false;
  }
  if (d % H) {
    *why = "dim must be divisible by n_heads";
    return false;
  }
  const int dh = d / H;
  if (dh != 16 && dh != 24 && dh != 32 && dh != 64) {
    *why = "head_dim must be 16, 24, 32 or 64 (the ESM-2 family)";
    return false;
  }
  if (d > 2560 || H > 64) {
    *why = "dim above 2560 or more than 64 heads";
    return false;
  }
  if (!esm::gemm_pick_bn(3 * d, dh) || !esm::gemm_pick_bn(d, 0) || !esm::gemm_pick_bn(c.hidden_dim, 0)) {
    *why = "no GEMM tile width divides the projection sizes";
    return false;
  }
  return true;
}

int build_weight_maps(esm_ctx* c) {
  const int d = c->cfg.dim, F = c->cfg.hidden_dim, dh = d / c->cfg.n_heads;
  c->bn_qkv = esm::gemm_pick_bn(3 * d, dh);
  c->bn_o = esm::gemm_pick_bn(d, 0);
  c->bn_fc1 = esm::gemm_pick_bn(F, 0);
  c->bn_fc2 = esm::gemm_pick_bn(d, 0);
  c->bn_dense = esm::gemm_pick_bn(d, 0);
  // Weight (B operand) maps load half tiles: bn/2 rows per box.
  bool ok = true;
  for (int b = 0; b < 2; ++b)
    ok = ok && esm::make_tmap_f16(&c->tm_wqkv[b], c->wqkv16[b], 3 * d, d, d, c->bn_qkv / 2) &&
         esm::make_tmap_f16(&c->tm_wo[b], c->wo16[b], d, d, d, c->bn_o / 2) &&
         esm::make_tmap_f16(&c->tm_w1[b], c->w116[b], F, d, d, c->bn_fc1 / 2) &&
         esm::make_tmap_f16(&c->tm_w2[b], c->w216[b], d, F, F, c->bn_fc2 / 2);
  if (ok && c->has_head) ok = esm::make_tmap_f16(&c->tm_dense, c->dense16, d, d, d, c->bn_dense / 2);
  return ok ? ESM_OK : fail(c, ESM_ECUDA, "cuTensorMapEncodeTiled failed for a weight matrix");
}

// Tensors of a Q8_0 / Q4_0 / Q3_LUT model quantized on the device while loading
// (EsmWeights::quantize_q8 / quantize_q4 / quantize_q3, src/lib.rs:559-633): the six matrices of
// every layer, for Q8_0 also the token embedding; for Q3_LUT only the four Q4_0 attention
// matrices (its Q3_LUT fc1 / fc2 are quantized on the host, see load_fp32_as).
uint32_t quantized_tensors(int dtype) {
  const uint32_t att = (1u << 3) | (1u << 5) | (1u << 7) | (1u << 9), fc = (1u << 13) | (1u << 15);
  if (dtype == ESM_DTYPE_Q8_0) return att | fc | 1u;
  if (dtype == ESM_DTYPE_Q4_0) return att | fc;
  if (dtype == ESM_DTYPE_Q3_LUT) return att;
  return 0u;
}

// Uploads a weight set. Tensor i with bit i of `quantize_mask` set is given as FP32 host data
// (sizes[i] = its FP32 byte size) and is quantized to `dtype` blocks on the device, straight into
// its device allocation; every other tensor is given in its `dtype` layout.
int load_host_impl(esm_ctx* c, const esm_config& cfg, int dtype, const void* const* tensors, const size_t* sizes,
                   uint32_t quantize_mask = 0) {
  std::string why;
  if (dtype < 0 || dtype > 3) return fail(c, ESM_EINVAL, "dtype must be FP32, Q8_0, Q4_0 or Q3_LUT");
  if (!shape_supported(cfg, &why)) return fail(c, ESM_EINVAL, "unsupported model shape: " + why);
  int64_t expect[ESM_NUM_TENSORS];
  esm::tensor_layout(cfg, dtype, expect);
  for (int i = 0; i < ESM_NUM_TENSORS; ++i) {
    if (tensors[i] == nullptr && !(i == 19 && sizes[i] == 0))
      return fail(c, ESM_EINVAL, "tensor " + std::to_string(i) + " is null");
    const bool q = (quantize_mask >> i) & 1u;
    const int64_t block_bytes = esm::matrix_dtype(dtype, i) == ESM_DTYPE_Q8_0 ? 36 : 20;
    const int64_t want = q ? expect[i] / block_bytes * 128 : expect[i];  // 32 floats per block
    if (i < 19 && static_cast<int64_t>(sizes[i]) != want)
      return fail(c, ESM_EFORMAT, "tensor " + std::to_string(i) + " has " + std::to_string(sizes[i]) +
                                      " bytes, expected " + std::to_string(want));
  }
  if (sizes[19] % 4) return fail(c, ESM_EFORMAT, "classifier byte size is not a multiple of 4");

  ESM_CUDA(cudaSetDevice(c->device));
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  free_list(c->w_allocs);
  const bool same_shape = c->cfg.dim == cfg.dim && c->cfg.hidden_dim == cfg.hidden_dim &&
                          c->cfg.n_heads == cfg.n_heads && c->cfg.n_layers == cfg.n_layers &&
                          c->cfg.vocab_size == cfg.vocab_size;
  if (!same_shape) {
    // The workspace is sized for the previous shape: drop it (esm_reserve is required again).
    free_list(c->ws_allocs);
    free_pinned(c);
    c->cap_tokens = 0;
    c->plan_key.clear();
  }
  c->loaded = false;
  c->cfg = cfg;
  c->dtype = dtype;
  const int64_t d = cfg.dim, F = cfg.hidden_dim, nl = cfg.n_layers, V = cfg.vocab_size;

  for (int i = 0; i < ESM_NUM_TENSORS; ++i) {
    const bool q = (quantize_mask >> i) & 1u;
    uint8_t* p = nullptr;
    int rc = dev_alloc(c, c->w_allocs, &p, std::max<size_t>(q ? expect[i] : sizes[i], 16));
    if (rc) return rc;
    if (q) {
      // FP32 staging on the device, quantized into place (load time only).
      std::vector<void*> tmp;
      float* f = nullptr;
      rc = dev_alloc(c, tmp, &f, sizes[i] / 4);
      if (rc) return rc;
      cudaError_t e = cudaMemcpyAsync(f, tensors[i], sizes[i], cudaMemcpyHostToDevice, c->stream);
      if (e == cudaSuccess)
        e = esm::launch_quantize(i == 0 ? dtype : esm::matrix_dtype(dtype, i), f, static_cast<int64_t>(sizes[i] / 128),
                                 p, c->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
      free_list(tmp);
      if (e != cudaSuccess) return fail(c, ESM_ECUDA, std::string("device quantization: ") + cudaGetErrorString(e));
    } else if (sizes[i]) {
      // On the context's stream, so the conversions enqueued below on that (non-blocking) stream
      // are ordered after the copy: a cudaMemcpy from pageable memory may return before its DMA
      // into device memory has finished.
      ESM_CUDA(cudaMemcpyAsync(p, tensors[i], sizes[i], cudaMemcpyHostToDevice, c->stream));
    }
    c->w[i] = p;
  }
  c->classifier_floats = static_cast<int64_t>(sizes[19] / 4);
  c->has_head = c->classifier_floats >= esm::lm_head_floats(cfg);

  // Stacked q|k|v bias per layer.
  {
    std::vector<float> hb(static_cast<size_t>(nl * 3 * d));
    const float* bq = static_cast<const float*>(tensors[4]);
    const float* bk = static_cast<const float*>(tensors[6]);
    const float* bv = static_cast<const float*>(tensors[8]);
    for (int64_t l = 0; l < nl; ++l) {
      std::memcpy(&hb[l * 3 * d], bq + l * d, d * 4);
      std::memcpy(&hb[l * 3 * d + d], bk + l * d, d * 4);
      std::memcpy(&hb[l * 3 * d + 2 * d], bv + l * d, d * 4);
    }
    int rc = dev_alloc(c, c->w_allocs, &c->bqkv, hb.size());
    if (rc) return rc;
    ESM_CUDA(cudaMemcpyAsync(c->bqkv, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice, c->stream));
    ESM_CUDA(cudaStreamSynchronize(c->stream));  // hb is a local staging vector
  }
  if (dtype == ESM_DTYPE_Q8_0) {
    int rc = dev_alloc(c, c->w_allocs, &c->emb_f32, static_cast<size_t>(V * d));
    if (rc) return rc;
    ESM_CUDA(esm::launch_to_f32(ESM_DTYPE_Q8_0, c->w[0], V * d, c->emb_f32, c->stream));
  } else {
    c->emb_f32 = static_cast<float*>(c->w[0]);
  }
  if (c->has_head) {
    int rc = dev_alloc(c, c->w_allocs, &c->dense16, static_cast<size_t>(d * d));
    if (rc) return rc;
    const float* dense_w = static_cast<const float*>(c->w[19]) + 2 * d;
    ESM_CUDA(esm::launch_to_f16(ESM_DTYPE_FP32, dense_w, d * d, c->dense16, c->stream));
  }
  int rc = ESM_OK;
  for (int b = 0; b < 2 && !rc; ++b) {
    rc = dev_alloc(c, c->w_allocs, &c->wqkv16[b], static_cast<size_t>(3 * d * d));
    if (!rc) rc = dev_alloc(c, c->w_allocs, &c->wo16[b], static_cast<size_t>(d * d));
    if (!rc) rc = dev_alloc(c, c->w_allocs, &c->w116[b], static_cast<size_t>(F * d));
    if (!rc) rc = dev_alloc(c, c->w_allocs, &c->w216[b], static_cast<size_t>(d * F));
  }
  if (rc) return rc;
  rc = build_weight_maps(c);
  if (rc) return rc;
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  c->loaded = true;
  // A previous contact head only fits if the shape is unchanged.
  if (c->has_ch) {
    cudaFree(c->d_ch_w);
    c->d_ch_w = nullptr;
    c->has_ch = false;
  }
  return ESM_OK;
}

// RoPE tables exactly as BidirectionalRunState::new (src/lib.rs:2510-2522), in f32 on the host.
std::vector<float2> rope_table(int max_len, int head_dim) {
  const int half = head_dim / 2;
  std::vector<float2> t(static_cast<size_t>(max_len) * half);
  for (int pos = 0; pos < max_len; ++pos) {
    for (int j = 0; j < half; ++j) {
      const float freq = 1.0f / std::pow(10000.0f, static_cast<float>(j * 2) / static_cast<float>(head_dim));
      const float val = static_cast<float>(pos) * freq;
      t[static_cast<size_t>(pos) * half + j] = make_float2(std::cos(val), std::sin(val));
    }
  }
  return t;
}

int reserve_impl(esm_ctx* c, int max_tokens, int max_seqs, int max_len, bool contacts) {
  if (!c->loaded) return fail(c, ESM_EINVAL, "load weights before reserving the workspace");
  if (max_tokens <= 0 || max_seqs <= 0 || max_len <= 0) return fail(c, ESM_EINVAL, "non-positive capacity");
  ESM_CUDA(cudaSetDevice(c->device));
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  free_list(c->ws_allocs);
  free_pinned(c);
  c->cap_tokens = 0;
  const esm_config& g = c->cfg;
  const int64_t d = g.dim, F = g.hidden_dim, H = g.n_heads, nl = g.n_layers;
  const int64_t rows = (static_cast<int64_t>(max_tokens) + 127) / 128 * 128;
  const int64_t full_seqs = max_tokens / max_len + 1;
  const int64_t t_per = (max_len + 63) / 64;
  const int64_t n_max = std::max(max_len - 2, 0);
  c->cap_rows = rows;
  c->work_cap = max_tokens / 64 + max_seqs + 1;
  c->tiles_cap = contacts ? std::min<int64_t>(full_seqs, max_seqs) * t_per * t_per + 1 : 1;
  c->m_cap = contacts ? std::min<int64_t>(full_seqs, max_seqs) * n_max * n_max + 1 : 1;
  c->r_cap = contacts ? nl * H * static_cast<int64_t>(max_tokens) + 1 : 1;

  int rc = ESM_OK;
  auto A = [&](auto** p, size_t n) {
    if (!rc) rc = dev_alloc(c, c->ws_allocs, p, n);
  };
  A(&c->x, rows * d);
  A(&c->xn, rows * d);
  A(&c->qkv, rows * 3 * d);
  const bool small_heads = d / H == 16 || d / H == 24;
  if (small_heads) A(&c->qk_lo, rows * 2 * d);
  A(&c->ao, rows * d);
  A(&c->hb, rows * F);
  A(&c->headf, rows * d);
  A(&c->hidden, rows * d);
  A(&c->logits, rows * g.vocab_size);
  A(&c->pos, rows);
  A(&c->seq_of, rows);
  A(&c->tokens, rows);
  A(&c->cu, max_seqs + 1);
  A(&c->escale, max_seqs);
  A(&c->work, c->work_cap);
  A(&c->work256, c->work_cap);
  A(&c->ctiles, c->tiles_cap);
  A(&c->m_off, max_seqs);
  A(&c->r_off, max_seqs);
  A(&c->rope, static_cast<size_t>(max_len) * (d / H / 2));
  if (contacts) {
    A(&c->lse, H * rows);
    A(&c->M, c->m_cap);
    A(&c->cmap, c->m_cap);
    A(&c->r, c->r_cap);
    A(&c->a_scr, static_cast<size_t>(max_seqs) * nl * H);
  }
  if (rc) return rc;
  // Stale rows past T are read by the GEMM A-loads of a partial last tile; keep them finite.
  // Everything the forward kernels read is written on the context's (non-blocking) stream, which
  // the legacy default stream of cudaMemset / cudaMemcpy does not order against.
  ESM_CUDA(cudaMemsetAsync(c->xn, 0, rows * d * 2, c->stream));
  ESM_CUDA(cudaMemsetAsync(c->ao, 0, rows * d * 2, c->stream));
  ESM_CUDA(cudaMemsetAsync(c->hb, 0, rows * F * 2, c->stream));
  if (small_heads) ESM_CUDA(cudaMemsetAsync(c->qk_lo, 0, rows * 2 * d * 2, c->stream));
  {
    std::vector<float2> rt = rope_table(max_len, static_cast<int>(d / H));
    ESM_CUDA(cudaMemcpyAsync(c->rope, rt.data(), rt.size() * sizeof(float2), cudaMemcpyHostToDevice, c->stream));
    ESM_CUDA(cudaStreamSynchronize(c->stream));  // rt is a local staging vector
  }
  ESM_CUDA(cudaMallocHost(&c->h_cu, sizeof(int32_t) * (max_seqs + 1)));
  ESM_CUDA(cudaMallocHost(&c->h_work, sizeof(int2) * c->work_cap));
  ESM_CUDA(cudaMallocHost(&c->h_work256, sizeof(int2) * c->work_cap));
  ESM_CUDA(cudaMallocHost(&c->h_tiles, sizeof(int4) * c->tiles_cap));
  ESM_CUDA(cudaMallocHost(&c->h_moff, sizeof(int64_t) * max_seqs));
  ESM_CUDA(cudaMallocHost(&c->h_roff, sizeof(int64_t) * max_seqs));
  bool ok = esm::make_tmap_f16(&c->tm_xn, c->xn, rows, d, d, 128) &&
            esm::make_tmap_f16(&c->tm_ao, c->ao, rows, d, d, 128) &&
            esm::make_tmap_f16(&c->tm_hb, c->hb, rows, F, F, 128) &&
            esm::make_tmap_f16(&c->tm_qkv_q, c->qkv, rows, 3 * d, 3 * d, 128) &&
            esm::make_tmap_f16(&c->tm_qkv_kv, c->qkv, rows, 3 * d, 3 * d, 64) &&
            esm::make_tmap_f16_box(&c->tm_qkv_q32, c->qkv, rows, 3 * d, 3 * d, 128, 32, 64) &&
            esm::make_tmap_f16_box(&c->tm_qkv_kv32, c->qkv, rows, 3 * d, 3 * d, 64, 32, 64) &&
            esm::make_tmap_f16(&c->tm_qkv_kv_r32, c->qkv, rows, 3 * d, 3 * d, 32) &&
            esm::make_tmap_f16_box(&c->tm_qkv_kv32_r32, c->qkv, rows, 3 * d, 3 * d, 32, 32, 64);
  const int64_t dh = d / H;
  if (ok && (dh == 16 || dh == 24))
    ok = esm::make_tmap_f16_heads(&c->tm_qkv_hq, c->qkv, rows, 3 * H, static_cast<uint32_t>(dh), 3 * d, 128) &&
         esm::make_tmap_f16_heads(&c->tm_qkv_hkv, c->qkv, rows, 3 * H, static_cast<uint32_t>(dh), 3 * d, 32) &&
         esm::make_tmap_f16_heads(&c->tm_lo_q, c->qk_lo, rows, 2 * H, static_cast<uint32_t>(dh), 2 * d, 128) &&
         esm::make_tmap_f16_heads(&c->tm_lo_k, c->qk_lo, rows, 2 * H, static_cast<uint32_t>(dh), 2 * d, 32);
  if (!ok) return fail(c, ESM_ECUDA, "cuTensorMapEncodeTiled failed for an activation buffer");
  c->cap_tokens = max_tokens;
  c->cap_seqs = max_seqs;
  c->cap_len = max_len;
  c->cap_contacts = contacts;
  c->plan_key.clear();
  return ESM_OK;
}

// Builds and uploads the per-call plan (cu_seqlens, attention work list, contact tiles and
// offsets). Identical consecutive plans are not re-uploaded.
// The tensor-core contact kernel serves head_dim 64 with up to 64 heads per layer.
bool use_contact_tc(const esm_ctx* c) {
  return c->contact_tc && c->cfg.n_heads > 0 && c->cfg.dim / c->cfg.n_heads == 64 && c->cfg.n_heads <= 64;
}

int upload_plan(esm_ctx* c, const int32_t* h_cu, int B, bool contacts, cudaStream_t s) {
  std::vector<int32_t> key(h_cu, h_cu + B + 1);
  const bool ct = contacts && use_contact_tc(c);
  key.push_back(contacts ? 1 : 0);
  key.push_back(ct ? 1 : 0);
  if (key == c->plan_key) return ESM_OK;
  const esm_config& g = c->cfg;
  const int64_t hl = static_cast<int64_t>(g.n_layers) * g.n_heads;
  // The previous plan's copies must have left the pinned staging before it is rewritten.
  if (c->plan_ev) ESM_CUDA(cudaEventSynchronize(c->plan_ev));
  int nw = 0, nw256 = 0, nt = 0;
  int64_t moff = 0, roff = 0;
  for (int b = 0; b <= B; ++b) c->h_cu[b] = h_cu[b];
  for (int b = 0; b < B; ++b) {
    const int len = h_cu[b + 1] - h_cu[b];
    const int qt = (len + 63) / 64;
    if (nw + qt > c->work_cap) return fail(c, ESM_ECAPACITY, "attention work list exceeds the reserved capacity");
    for (int t = 0; t < qt; ++t) c->h_work[nw++] = make_int2(b, t);
    for (int t = 0; t < (len + 255) / 256; ++t) c->h_work256[nw256++] = make_int2(b, t);
    if (contacts) {
      const int64_t n = std::max(len - 2, 0);
      c->h_moff[b] = moff;
      c->h_roff[b] = roff;
      moff += n * n;
      roff += hl * n;
      if (n > 0) {
        const int64_t tiles = ct ? esm::contact_tc_tiles(len, nullptr, b) : static_cast<int64_t>(qt) * qt;
        if (nt + tiles > c->tiles_cap) return fail(c, ESM_ECAPACITY, "contact tiles exceed the reserved capacity");
        if (ct) {
          esm::contact_tc_tiles(len, c->h_tiles + nt, b);
          nt += static_cast<int>(tiles);
        } else {
          for (int i = 0; i < qt; ++i)
            for (int j = 0; j < qt; ++j) c->h_tiles[nt++] = make_int4(b, i, j, 0);
        }
      }
    }
  }
  if (contacts && (moff > c->m_cap || roff > c->r_cap))
    return fail(c, ESM_ECAPACITY, "contact maps exceed the reserved capacity");
  ESM_CUDA(cudaMemcpyAsync(c->cu, c->h_cu, sizeof(int32_t) * (B + 1), cudaMemcpyHostToDevice, s));
  ESM_CUDA(cudaMemcpyAsync(c->work, c->h_work, sizeof(int2) * nw, cudaMemcpyHostToDevice, s));
  ESM_CUDA(cudaMemcpyAsync(c->work256, c->h_work256, sizeof(int2) * nw256, cudaMemcpyHostToDevice, s));
  if (contacts) {
    ESM_CUDA(cudaMemcpyAsync(c->m_off, c->h_moff, sizeof(int64_t) * B, cudaMemcpyHostToDevice, s));
    ESM_CUDA(cudaMemcpyAsync(c->r_off, c->h_roff, sizeof(int64_t) * B, cudaMemcpyHostToDevice, s));
    if (nt) ESM_CUDA(cudaMemcpyAsync(c->ctiles, c->h_tiles, sizeof(int4) * nt, cudaMemcpyHostToDevice, s));
  }
  if (!c->plan_ev) ESM_CUDA(cudaEventCreateWithFlags(&c->plan_ev, cudaEventDisableTiming));
  ESM_CUDA(cudaEventRecord(c->plan_ev, s));
  c->plan_key = key;
  c->plan_work = nw;
  c->plan_work256 = nw256;
  c->plan_tiles = nt;
  return ESM_OK;
}

int gemm(esm_ctx* c, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap* tout, int bn, int epi, int M,
         int N, int K, const float* bias, void* out, int ldo, cudaStream_t s, __half* lo = nullptr) {
  esm::GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.bias = bias;
  p.out = out;
  p.ldo = ldo;
  p.pos = c->pos;
  p.rope = c->rope;
  p.rope_cols = 2 * c->cfg.dim;
  p.err = c->d_err;
  p.lo = lo;
  p.lo_ld = 2 * c->cfg.dim;
  const int dh = c->cfg.dim / c->cfg.n_heads;
  ESM_CUDA(esm::gemm_launch(ta, tb, tout, bn, epi, epi == esm::kEpiQkvRope ? dh : 0, p, c->num_sms, s, c->cta_pair));
  return ESM_OK;
}

cudaEvent_t prof_event(esm_ctx* c) {
  if (c->ev_used == c->ev_pool.size()) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    c->ev_pool.push_back(e);
  }
  return c->ev_pool[c->ev_used++];
}

// Brackets one launch with events when profiling is on (no cost otherwise).
struct ProfScope {
  esm_ctx* c;
  cudaStream_t s;
  int kind;
  double flops, bytes;
  cudaEvent_t a = nullptr;
  ProfScope(esm_ctx* c_, cudaStream_t s_, int kind_, double flops_, double bytes_)
      : c(c_), s(s_), kind(kind_), flops(flops_), bytes(bytes_) {
    if (c->prof && (a = prof_event(c))) cudaEventRecord(a, s);
  }
  ~ProfScope() {
    if (!a) return;
    cudaEvent_t b = prof_event(c);
    if (!b) return;
    cudaEventRecord(b, s);
    c->prof_recs.push_back({a, b, kind, flops, bytes});
  }
};

// The forward over packed device tokens. Caller holds the context lock and validated shapes.
int forward_impl(esm_ctx* c, const int32_t* d_tokens, const int32_t* h_cu, int B, float* d_logits, float* d_hidden,
                 float* d_contacts, float* d_layer_hidden, cudaStream_t s) {
  const esm_config& g = c->cfg;
  const int d = g.dim, F = g.hidden_dim, H = g.n_heads, nl = g.n_layers, V = g.vocab_size;
  const int dh = d / H;
  const int T = h_cu[B];
  const bool contacts = d_contacts != nullptr;
  int rc = upload_plan(c, h_cu, B, contacts, s);
  if (rc) return rc;

  const float* ln1_w = static_cast<const float*>(c->w[1]);
  const float* ln1_b = static_cast<const float*>(c->w[2]);
  const float* bo = static_cast<const float*>(c->w[10]);
  const float* ln2_w = static_cast<const float*>(c->w[11]);
  const float* ln2_b = static_cast<const float*>(c->w[12]);
  const float* fc1_b = static_cast<const float*>(c->w[14]);
  const float* fc2_b = static_cast<const float*>(c->w[16]);
  const float* lnf_w = static_cast<const float*>(c->w[17]);
  const float* lnf_b = static_cast<const float*>(c->w[18]);
  const int64_t dd = static_cast<int64_t>(d) * d, fd = static_cast<int64_t>(F) * d;
  const int dt_mat = esm::matrix_dtype(c->dtype, 3), dt_fc = esm::matrix_dtype(c->dtype, 13);
  const int64_t mat_b = esm::matrix_bytes(dt_mat, dd), fc_b = esm::matrix_bytes(dt_fc, fd);

  ESM_CUDA(esm::launch_seq_setup(d_tokens, c->cu, B, c->pos, c->seq_of, c->escale, s));
  const double rowb = static_cast<double>(T) * d;
  {
  ProfScope ps(c, s, ESM_PROF_NORM, 0.0, rowb * 6.0);
  ESM_CUDA(esm::launch_embed_ln(d_tokens, c->seq_of, c->escale, c->dtype == ESM_DTYPE_Q8_0 ? nullptr : c->emb_f32,
                                c->w[0], g.vocab_size, T, d, ln1_w, ln1_b, c->x, c->xn, c->d_err, s));
  }
  int64_t attn_pairs = 0;
  for (int b = 0; b < B; ++b) attn_pairs += static_cast<int64_t>(h_cu[b + 1] - h_cu[b]) * (h_cu[b + 1] - h_cu[b]);
  int64_t m_total = 0, r_total = 0;
  if (contacts) {
    for (int b = 0; b < B; ++b) {
      const int64_t n = std::max(h_cu[b + 1] - h_cu[b] - 2, 0);
      m_total += n * n;
      r_total += static_cast<int64_t>(nl) * H * n;
    }
    ESM_CUDA(cudaMemsetAsync(c->M, 0, std::max<int64_t>(m_total, 1) * 4, s));
    ESM_CUDA(cudaMemsetAsync(c->r, 0, std::max<int64_t>(r_total, 1) * 4, s));
  }

  // Output maps of the bulk-store GEMM epilogues, over exactly this call's T rows (rows past T of a
  // 32-row block are clipped by the map, not written).
  CUtensorMap tm_out_qkv, tm_out_hb, tm_out_x;
  const bool out_maps = esm::make_tmap_out(&tm_out_qkv, c->qkv, 2, T, 3 * d, 3 * d) &&
                        esm::make_tmap_out(&tm_out_hb, c->hb, 2, T, F, F) &&
                        esm::make_tmap_out(&tm_out_x, c->x, 4, T, d, d);
  if (!out_maps) return fail(c, ESM_ECUDA, "cuTensorMapEncodeTiled failed for a GEMM output");
  const CUtensorMap* out_qkv = &tm_out_qkv;
  const CUtensorMap* out_hb = &tm_out_hb;
  const CUtensorMap* out_x = &tm_out_x;

  esm::AttnParams ap{};
  ap.qkv = c->qkv;
  ap.out = c->ao;
  ap.lse = contacts ? c->lse : nullptr;
  ap.cu_seqlens = c->cu;
  ap.work = c->work;
  ap.n_work = c->plan_work;
  ap.T = T;
  ap.d = d;
  ap.H = H;
  ap.dh = dh;
  ap.scale = 1.0f / std::sqrt(static_cast<float>(dh));
  ap.err = c->d_err;
  ap.rescale_sum = c->attn_rescale_sum;
  ap.wait_mma_ns = c->attn_wait_mma;
  // head_dim 64, 32, 24 and 16 run the tcgen05 kernel (attention_tc3.cu; 16 and 24 zero-padded to
  // 32 by the 3-D tensor maps) unless ESM_ATTN_TC=0, which selects the mma.sync kernel
  // (attention.cu).
  const bool attn_tc = (dh == 64 || dh == 32 || dh == 24 || dh == 16) && c->attn_tc != 0;
  const bool head_pad = dh == 16 || dh == 24;
  esm::AttnParams ap256 = ap;
  ap256.work = c->work256;
  ap256.n_work = c->plan_work256;

  // Weight dequantisation of layer l into fp16 set l & 1: on the side stream, one layer ahead of
  // the layer that uses it, after the layer that last read that set; the forward's stream waits
  // for it before the layer's first GEMM. The side stream starts after the work already queued on
  // the forward's stream and every side-stream launch is joined back into that stream.
  const bool overlap = c->deq_overlap != 0;
  cudaStream_t ds = overlap ? c->side : s;
  auto dequant = [&](int l) -> int {
    esm::LayerSrc src{};
    for (int m = 0; m < 6; ++m) src.dtype[m] = m < 4 ? dt_mat : dt_fc;
    src.w[0] = static_cast<const uint8_t*>(c->w[3]) + l * mat_b;
    src.w[1] = static_cast<const uint8_t*>(c->w[5]) + l * mat_b;
    src.w[2] = static_cast<const uint8_t*>(c->w[7]) + l * mat_b;
    src.w[3] = static_cast<const uint8_t*>(c->w[9]) + l * mat_b;
    src.w[4] = static_cast<const uint8_t*>(c->w[13]) + l * fc_b;
    src.w[5] = static_cast<const uint8_t*>(c->w[15]) + l * fc_b;
    src.elems[0] = src.elems[1] = src.elems[2] = src.elems[3] = dd;
    src.elems[4] = src.elems[5] = fd;
    const int b = l & 1;
    if (overlap) ESM_CUDA(cudaStreamWaitEvent(ds, c->ev_read[b], 0));
    {
      ProfScope ps(c, ds, ESM_PROF_DEQUANT, 0.0, static_cast<double>(4 * mat_b + 2 * fc_b) + 2.0 * (4 * dd + 2 * fd));
      ESM_CUDA(esm::launch_dequant_layer(src, c->wqkv16[b], c->wo16[b], c->w116[b], c->w216[b], ds));
    }
    if (overlap) ESM_CUDA(cudaEventRecord(c->ev_deq[b], ds));
    return ESM_OK;
  };
  if (overlap) {
    ESM_CUDA(cudaEventRecord(c->ev_start, s));
    ESM_CUDA(cudaStreamWaitEvent(ds, c->ev_start, 0));
    rc = dequant(0);
    if (rc) return rc;
  }
  for (int l = 0; l < nl; ++l) {
    const int wb = l & 1;
    if (overlap) {
      if (l + 1 < nl) {
        rc = dequant(l + 1);
        if (rc) return rc;
      }
      ESM_CUDA(cudaStreamWaitEvent(s, c->ev_deq[wb], 0));
    } else {
      rc = dequant(l);
      if (rc) return rc;
    }
    if (l > 0) {
      ProfScope ps(c, s, ESM_PROF_NORM, 0.0, rowb * 6.0);
      ESM_CUDA(esm::launch_layernorm(c->x, T, d, ln1_w + l * d, ln1_b + l * d, c->xn, d, nullptr, s));
    }
    {
      ProfScope ps(c, s, ESM_PROF_GEMM, 2.0 * T * 3.0 * d * d, 0.0);
      rc = gemm(c, c->tm_xn, c->tm_wqkv[wb], out_qkv, c->bn_qkv, esm::kEpiQkvRope, T, 3 * d, d,
                c->bqkv + static_cast<int64_t>(l) * 3 * d, c->qkv, 3 * d, s, c->qk_lo);
      if (rc) return rc;
    }
    {
      ProfScope ps(c, s, ESM_PROF_ATTENTION, 4.0 * static_cast<double>(attn_pairs) * d, 0.0);
      if (attn_tc) {
        const int poly = c->attn_poly >= 0 ? c->attn_poly : (c->attn_exp == 1 || c->attn_exp == 3 ? 2 : 0);
        const CUtensorMap& tq = head_pad ? c->tm_qkv_hq : (dh == 32 ? c->tm_qkv_q32 : c->tm_qkv_q);
        const CUtensorMap& tkv = head_pad ? c->tm_qkv_hkv : (dh == 32 ? c->tm_qkv_kv32_r32 : c->tm_qkv_kv_r32);
        ESM_CUDA(esm::launch_attention_tc3(tq, tkv, head_pad ? c->tm_lo_q : tq, head_pad ? c->tm_lo_k : tkv, ap256,
                                           poly, c->attn_exp, s));
      } else {
        ESM_CUDA(esm::launch_attention(ap, s));
      }
    }
    if (contacts) {
      ProfScope ps(c, s, ESM_PROF_CONTACT, 2.0 * static_cast<double>(attn_pairs) * d, 0.0);
      esm::ContactParams cp{};
      cp.qkv = c->qkv;
      cp.lse = c->lse;
      cp.cu_seqlens = c->cu;
      cp.tiles = c->ctiles;
      cp.n_tiles = c->plan_tiles;
      cp.T = T;
      cp.d = d;
      cp.H = H;
      cp.dh = dh;
      cp.scale = ap.scale;
      cp.qk_lo = (head_pad && attn_tc) ? c->qk_lo : nullptr;  // the scores the log-sum-exp came from
      cp.w_layer = c->d_ch_w + static_cast<int64_t>(l) * H;
      cp.m_off = c->m_off;
      cp.M = c->M;
      cp.r_off = c->r_off;
      cp.r = c->r;
      cp.head_base = l * H;
      cp.err = c->d_err;
      // The mma.sync kernel has one CTA per 64 x 64 tile; when a layer has fewer tiles than two
      // per SM (short sequences), the heads of each tile are split over more CTAs.
      cp.head_groups = std::max(1, std::min(H, (2 * c->num_sms + std::max(c->plan_tiles, 1) - 1) /
                                                   std::max(c->plan_tiles, 1)));
      if (use_contact_tc(c)) {
        ESM_CUDA(esm::launch_contact_tc(c->tm_qkv_q, c->tm_qkv_kv, cp, c->seq_of, s));
      } else {
        ESM_CUDA(esm::launch_contact_accumulate(cp, s));
      }
    }
    {
      ProfScope ps(c, s, ESM_PROF_GEMM, 2.0 * T * static_cast<double>(dd), 0.0);
      rc = gemm(c, c->tm_ao, c->tm_wo[wb], out_x, c->bn_o, esm::kEpiResidF32, T, d, d, bo + static_cast<int64_t>(l) * d, c->x, d,
                s);
      if (rc) return rc;
    }
    {
      ProfScope ps(c, s, ESM_PROF_NORM, 0.0, rowb * 6.0);
      ESM_CUDA(esm::launch_layernorm(c->x, T, d, ln2_w + l * d, ln2_b + l * d, c->xn, d, nullptr, s));
    }
    {
      ProfScope ps(c, s, ESM_PROF_GEMM, 2.0 * T * static_cast<double>(fd), 0.0);
      rc = gemm(c, c->tm_xn, c->tm_w1[wb], out_hb, c->bn_fc1, esm::kEpiGeluF16, T, F, d, fc1_b + static_cast<int64_t>(l) * F, c->hb,
                F, s);
      if (rc) return rc;
    }
    {
      ProfScope ps(c, s, ESM_PROF_GEMM, 2.0 * T * static_cast<double>(fd), 0.0);
      rc = gemm(c, c->tm_hb, c->tm_w2[wb], out_x, c->bn_fc2, esm::kEpiResidF32, T, d, F, fc2_b + static_cast<int64_t>(l) * d, c->x,
                d, s);
      if (rc) return rc;
    }
    if (overlap) ESM_CUDA(cudaEventRecord(c->ev_read[wb], s));
    if (d_layer_hidden)
      ESM_CUDA(cudaMemcpyAsync(d_layer_hidden + static_cast<int64_t>(l) * T * d, c->x, static_cast<size_t>(T) * d * 4,
                               cudaMemcpyDeviceToDevice, s));
  }

  if (contacts) {
    int max_n = 0;
    for (int b = 0; b < B; ++b) max_n = std::max(max_n, h_cu[b + 1] - h_cu[b] - 2);
    ProfScope ps(c, s, ESM_PROF_CONTACT, 0.0, 0.0);
    ESM_CUDA(esm::launch_contact_finalize(c->M, c->r, c->m_off, c->r_off, c->cu, B, max_n, nl * H, c->d_ch_w, c->ch_b,
                                          c->a_scr, d_contacts, s));
  }

  // Final LayerNorm (state.x after the call), then the LM head (src/lib.rs:5379-5439).
  float* hid32 = d_hidden ? d_hidden : (c->has_head ? nullptr : c->hidden);
  {
    ProfScope ps(c, s, ESM_PROF_NORM, 0.0, rowb * 6.0);
    ESM_CUDA(esm::launch_layernorm(c->x, T, d, lnf_w, lnf_b, c->xn, d, hid32, s));
  }
  if (c->has_head) {
    const float* cls = static_cast<const float*>(c->w[19]);
    const float* lm_ln_w = cls;
    const float* lm_ln_b = cls + d;
    const float* dense_b = cls + 2 * d + dd;
    const float* dec_w = cls + 3 * d + dd;
    const float* dec_b = dec_w + static_cast<int64_t>(V) * d;
    {
      ProfScope ps(c, s, ESM_PROF_GEMM, 2.0 * T * static_cast<double>(dd), 0.0);
      rc = gemm(c, c->tm_xn, c->tm_dense, nullptr, c->bn_dense, esm::kEpiGeluF32, T, d, d, dense_b, c->headf, d, s);
      if (rc) return rc;
    }
    ProfScope ps(c, s, ESM_PROF_HEAD, 2.0 * T * static_cast<double>(V) * d, rowb * 4.0);
    ESM_CUDA(esm::launch_lm_decoder(c->headf, T, d, 1, lm_ln_w, lm_ln_b, dec_w, dec_b, V, d_logits, s));
  } else {
    // Tied-embedding fallback: logits = x E^T with zero bias (src/lib.rs:5429-5439).
    ProfScope ps(c, s, ESM_PROF_HEAD, 2.0 * T * static_cast<double>(V) * d, rowb * 4.0);
    ESM_CUDA(esm::launch_lm_decoder(hid32, T, d, 0, nullptr, nullptr, c->emb_f32, nullptr, V, d_logits, s));
  }
  return ESM_OK;
}

int check_device_word(esm_ctx* c) {
  int h = 0;
  ESM_CUDA(cudaMemcpy(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (h != 0) {
    cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream);
    cudaStreamSynchronize(c->stream);
    if (h == esm::kDevBadToken)
      return fail(c, ESM_EINVAL, "a token id is outside [0, " + std::to_string(c->cfg.vocab_size) + ")");
    return fail(c, ESM_ETIMEOUT, "a device-side bounded wait gave up (code " + std::to_string(h) + ")");
  }
  return ESM_OK;
}

int validate_call(esm_ctx* c, const int32_t* h_cu, int B, bool contacts) {
  if (!c->loaded) return fail(c, ESM_EINVAL, "no weights loaded");
  if (c->cap_tokens == 0) return fail(c, ESM_EINVAL, "call esm_reserve before the first forward");
  if (B <= 0) return fail(c, ESM_EINVAL, "batch must hold at least one sequence");
  if (B > c->cap_seqs) return fail(c, ESM_ECAPACITY, "batch exceeds the reserved number of sequences");
  if (h_cu[0] != 0) return fail(c, ESM_EINVAL, "cu_seqlens must start at 0");
  for (int b = 0; b < B; ++b) {
    const int len = h_cu[b + 1] - h_cu[b];
    if (len <= 0) return fail(c, ESM_EINVAL, "sequence " + std::to_string(b) + " is empty");
    if (len > c->cap_len)
      return fail(c, ESM_ECAPACITY, "Sequence length " + std::to_string(len) + " exceeds max_len " +
                                        std::to_string(c->cap_len));
  }
  if (h_cu[B] > c->cap_tokens) return fail(c, ESM_ECAPACITY, "token count exceeds the reserved capacity");
  if (contacts && !c->cap_contacts) return fail(c, ESM_ECAPACITY, "workspace was reserved without contact maps");
  if (contacts && !c->has_ch) return fail(c, ESM_EINVAL, "contacts requested but no contact head was set");
  return ESM_OK;
}

bool read_exact(std::ifstream& f, void* dst, size_t n) {
  f.read(static_cast<char*>(dst), static_cast<std::streamsize>(n));
  return static_cast<size_t>(f.gcount()) == n;
}

bool path_hint(const std::string& p, const char* tag) { return p.find(tag) != std::string::npos; }

}  // namespace

extern "C" {

int esm_config_preset(int32_t arch, esm_config* out) {
  if (!out || !esm::config_preset(arch, out)) return ESM_EINVAL;
  return ESM_OK;
}

int esm_get_config(const esm_ctx* c, esm_config* out, int32_t* dtype) {
  if (!c || !out) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(const_cast<esm_ctx*>(c)->mu);
  if (!c->loaded) return ESM_EINVAL;
  *out = c->cfg;
  if (dtype) *dtype = c->dtype;
  return ESM_OK;
}

int esm_config_detect_file(const char* path, esm_config* out, int32_t* dtype) {
  if (!path || !out) return ESM_EINVAL;
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) return ESM_EIO;
  const uint64_t len = static_cast<uint64_t>(f.tellg());
  f.seekg(0);
  if (len >= 64) {
    CodqHeader h;
    if (read_exact(f, &h, 64) && std::memcmp(h.magic, "CODQ", 4) == 0) {
      if (!h.validate(nullptr).empty()) return ESM_EFORMAT;
      esm::config_preset(static_cast<int>(h.arch), out);
      if (dtype) *dtype = static_cast<int32_t>(h.dtype);
      return ESM_OK;
    }
  }
  if (!esm::detect_from_file_len(len, out)) return ESM_EFORMAT;
  if (dtype) *dtype = ESM_DTYPE_FP32;
  return ESM_OK;
}

int esm_quantize_q8(const float* src, int64_t n, void* dst) {
  if (!src || !dst || n < 0 || n % 32) return ESM_EINVAL;
  esm::quantize_q8(src, n, static_cast<uint8_t*>(dst));
  return ESM_OK;
}

int esm_quantize_q4(const float* src, int64_t n, void* dst) {
  if (!src || !dst || n < 0 || n % 32) return ESM_EINVAL;
  esm::quantize_q4(src, n, static_cast<uint8_t*>(dst));
  return ESM_OK;
}

int esm_quantize_q3(const float* src, int64_t n, void* dst) {
  if (!src || !dst || n < 0 || n % 32) return ESM_EINVAL;
  esm::quantize_q3(src, n, static_cast<uint8_t*>(dst));
  return ESM_OK;
}

int esm_tokenize(const char* seq, int32_t* out, int32_t cap, int32_t* n_out) {
  if (!seq || !n_out || (!out && cap > 0)) return ESM_EINVAL;
  return esm::tokenize(seq, out, cap, n_out);
}

int esm_ctx_create(int32_t device, esm_ctx** out) {
  if (!out) return ESM_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return ESM_ECUDA;
  if (device < 0 || device >= n) return ESM_EINVAL;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return ESM_ECUDA;
  if (prop.major != 10) return ESM_EINVAL;  // built for sm_100a only
  esm_ctx* c = new esm_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  if (const char* v = std::getenv("ESM_GEMM_CTA_PAIR")) c->cta_pair = std::atoi(v) != 0;
  if (const char* v = std::getenv("ESM_ATTN_TC")) c->attn_tc = std::atoi(v);
  if (const char* v = std::getenv("ESM_ATTN_POLY")) c->attn_poly = std::min(3, std::max(0, std::atoi(v)));
  if (const char* v = std::getenv("ESM_ATTN_EXP")) c->attn_exp = std::min(3, std::max(0, std::atoi(v)));
  if (const char* v = std::getenv("ESM_ATTN_WAIT_MMA"))
    c->attn_wait_mma = static_cast<uint32_t>(std::min(1000000, std::max(0, std::atoi(v))));
  if (const char* v = std::getenv("ESM_ATTN_RESCALE_SUM"))
    c->attn_rescale_sum = std::min(32768.0f, std::max(64.0f, static_cast<float>(std::atof(v))));
  if (const char* v = std::getenv("ESM_CONTACT_TC")) c->contact_tc = std::atoi(v) != 0;
  if (const char* v = std::getenv("ESM_DEQUANT_OVERLAP")) c->deq_overlap = std::atoi(v) != 0;
  bool events_ok = cudaSetDevice(device) == cudaSuccess &&
                   cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) == cudaSuccess &&
                   cudaEventCreateWithFlags(&c->ev_start, cudaEventDisableTiming) == cudaSuccess;
  for (int b = 0; b < 2 && events_ok; ++b)
    events_ok = cudaEventCreateWithFlags(&c->ev_deq[b], cudaEventDisableTiming) == cudaSuccess &&
                cudaEventCreateWithFlags(&c->ev_read[b], cudaEventDisableTiming) == cudaSuccess;
  if (!events_ok || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess ||
      cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream) != cudaSuccess ||
      cudaStreamSynchronize(c->stream) != cudaSuccess) {
    if (c->d_err) cudaFree(c->d_err);
    for (cudaStream_t st : {c->stream, c->side})
      if (st) cudaStreamDestroy(st);
    for (cudaEvent_t e : {c->ev_start, c->ev_deq[0], c->ev_deq[1], c->ev_read[0], c->ev_read[1]})
      if (e) cudaEventDestroy(e);
    delete c;
    return ESM_ECUDA;
  }
  *out = c;
  return ESM_OK;
}

int esm_ctx_destroy(esm_ctx* c) {
  if (!c) return ESM_EINVAL;
  {
    std::lock_guard<std::mutex> lk(c->mu);
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    free_list(c->w_allocs);
    free_list(c->ws_allocs);
    free_pinned(c);
    if (c->d_ch_w) cudaFree(c->d_ch_w);
    if (c->d_rank) cudaFree(c->d_rank);
    if (c->d_padded_tokens) cudaFree(c->d_padded_tokens);
    if (c->d_padded_out) cudaFree(c->d_padded_out);
    if (c->d_layers) cudaFree(c->d_layers);
    if (c->d_dms) cudaFree(c->d_dms);
    if (c->plan_ev) cudaEventDestroy(c->plan_ev);
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    if (c->d_err) cudaFree(c->d_err);
    if (c->side) {
      cudaStreamSynchronize(c->side);
      cudaStreamDestroy(c->side);
    }
    for (cudaEvent_t e : {c->ev_start, c->ev_deq[0], c->ev_deq[1], c->ev_read[0], c->ev_read[1]})
      if (e) cudaEventDestroy(e);
    cudaStreamDestroy(c->stream);
  }
  delete c;
  return ESM_OK;
}

const char* esm_last_error(const esm_ctx* c) { return c ? c->err.c_str() : "null context"; }

int esm_load_host(esm_ctx* c, const esm_config* cfg, int32_t dtype, const void* const* tensors, const size_t* sizes) {
  if (!c || !cfg || !tensors || !sizes) return fail(c, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  return load_host_impl(c, *cfg, dtype, tensors, sizes);
}

namespace {

// An FP32 weight set (host memory) loaded as a `dtype` model: the device quantizes what it can
// (Q8_0 / Q4_0 blocks); a Q3_LUT model's fc1 / fc2 go through the host quantizer first
// (BlockQ3_LUT's iterative fit is a load-time format conversion with no device version here).
int load_fp32_as(esm_ctx* c, const esm_config& cfg, int dtype, const void* const* tensors, const size_t* sizes) {
  if (dtype != ESM_DTYPE_Q3_LUT) return load_host_impl(c, cfg, dtype, tensors, sizes, quantized_tensors(dtype));
  const void* ptr[ESM_NUM_TENSORS];
  size_t sz[ESM_NUM_TENSORS];
  std::vector<uint8_t> q3[2];
  for (int i = 0; i < ESM_NUM_TENSORS; ++i) {
    ptr[i] = tensors[i];
    sz[i] = sizes[i];
  }
  for (int k = 0; k < 2; ++k) {
    const int i = k ? 15 : 13;
    if (!tensors[i] || sizes[i] % 128) return fail(c, ESM_EFORMAT, "tensor " + std::to_string(i) + " is not FP32 blocks");
    const int64_t n = static_cast<int64_t>(sizes[i] / 4);
    q3[k].resize(static_cast<size_t>(n / 32 * 14));
    esm::quantize_q3(static_cast<const float*>(tensors[i]), n, q3[k].data());
    ptr[i] = q3[k].data();
    sz[i] = q3[k].size();
  }
  return load_host_impl(c, cfg, dtype, ptr, sz, quantized_tensors(dtype));
}

// Reads a CODQ or header-less weight file into host memory and splits it into the 20 tensors
// (EsmWeights{,Q8,Q4}::from_file, src/lib.rs:310-547, 744-830, 1156-1242).
struct WeightFile {
  esm_config cfg{};
  int dtype = ESM_DTYPE_FP32;
  const void* ptr[ESM_NUM_TENSORS] = {};
  size_t sizes[ESM_NUM_TENSORS] = {};
  std::vector<uint8_t> buf;
  std::vector<float> reordered;
};

int read_weight_file(esm_ctx* c, const char* path, const esm_config* cfg_in, WeightFile& wf) {
  esm_config& cfg = wf.cfg;
  int& dtype = wf.dtype;
  const void** ptr = wf.ptr;
  size_t* sizes = wf.sizes;
  std::vector<uint8_t>& buf = wf.buf;
  std::vector<float>& reordered = wf.reordered;
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) return fail(c, ESM_EIO, std::string("cannot open ") + path);
  const uint64_t file_len = static_cast<uint64_t>(f.tellg());
  f.seekg(0);
  uint64_t start = 0;
  CodqHeader h{};
  const bool has_header = file_len >= 64 && read_exact(f, &h, 64) && std::memcmp(h.magic, "CODQ", 4) == 0;
  if (has_header) {
    const std::string why = h.validate(cfg_in);
    if (!why.empty()) return fail(c, ESM_EFORMAT, why);
    esm::config_preset(static_cast<int>(h.arch), &cfg);
    dtype = static_cast<int>(h.dtype);
    if (dtype > ESM_DTYPE_Q3_LUT) return fail(c, ESM_EFORMAT, "unsupported CODQ dtype " + std::to_string(dtype));
    start = 64;
  } else {
    if (cfg_in) {
      cfg = *cfg_in;
    } else if (!esm::detect_from_file_len(file_len, &cfg)) {
      esm::config_preset(0, &cfg);  // load_from_file falls back to the 8M config
    }
    // Header-less Q8_0/Q4_0 files are recognised by name, as load_or_convert does
    // (src/lib.rs:838-856, 1250-1274); everything else is FP32.
    const std::string p(path);
    if (path_hint(p, "q3")) dtype = ESM_DTYPE_Q3_LUT;  // load_model_weights checks q3 first (src/main.rs:190-200)
    else if (path_hint(p, "q4")) dtype = ESM_DTYPE_Q4_0;
    else if (path_hint(p, "q8")) dtype = ESM_DTYPE_Q8_0;
  }
  const uint64_t remaining = file_len - start;
  buf.resize(remaining);
  f.clear();
  f.seekg(static_cast<std::streamoff>(start));
  if (!read_exact(f, buf.data(), remaining)) return fail(c, ESM_EIO, "short read");

  int64_t sz[ESM_NUM_TENSORS];
  esm::tensor_layout(cfg, dtype, sz);
  if (dtype == ESM_DTYPE_FP32) {
    if (remaining % 4) return fail(c, ESM_EFORMAT, "Unaligned trailing bytes: not a multiple of 4");
    const int64_t floats = static_cast<int64_t>(remaining / 4);
    const int64_t d = cfg.dim, F = cfg.hidden_dim, nl = cfg.n_layers, V = cfg.vocab_size;
    if (floats == esm::grouped_canonical_floats(cfg)) {
      sz[19] = esm::lm_head_floats(cfg) * 4;
      uint64_t off = 0;
      for (int i = 0; i < ESM_NUM_TENSORS; ++i) {
        ptr[i] = buf.data() + off;
        sizes[i] = static_cast<size_t>(sz[i]);
        off += sz[i];
      }
    } else if (floats == esm::sequential_hf_floats(cfg)) {
      // Sequential HF / fair-esm dump (src/lib.rs:397-489): per-layer q,bq,k,bk,v,bv,o,bo,ln1 w/b,
      // fc1 w/b, fc2 w/b, ln2 w/b; then ln_f, contact head, lm bias, dense w/b, lm ln w/b, decoder.
      const float* s = reinterpret_cast<const float*>(buf.data());
      int64_t total = 0;
      for (int i = 0; i < 19; ++i) total += sz[i] / 4;
      total += esm::lm_head_floats(cfg);
      reordered.resize(static_cast<size_t>(total));
      int64_t off[ESM_NUM_TENSORS];
      int64_t o = 0;
      for (int i = 0; i < 19; ++i) {
        off[i] = o;
        o += sz[i] / 4;
      }
      off[19] = o;
      float* r = reordered.data();
      int64_t p = 0;
      auto take = [&](float* dst, int64_t n) {
        std::memcpy(dst, s + p, n * 4);
        p += n;
      };
      take(r + off[0], V * d);
      p += (d / cfg.n_heads) / 2;  // inv_freq
      for (int64_t l = 0; l < nl; ++l) {
        take(r + off[3] + l * d * d, d * d);
        take(r + off[4] + l * d, d);
        take(r + off[5] + l * d * d, d * d);
        take(r + off[6] + l * d, d);
        take(r + off[7] + l * d * d, d * d);
        take(r + off[8] + l * d, d);
        take(r + off[9] + l * d * d, d * d);
        take(r + off[10] + l * d, d);
        take(r + off[1] + l * d, d);
        take(r + off[2] + l * d, d);
        take(r + off[13] + l * F * d, F * d);
        take(r + off[14] + l * F, F);
        take(r + off[15] + l * d * F, d * F);
        take(r + off[16] + l * d, d);
        take(r + off[11] + l * d, d);
        take(r + off[12] + l * d, d);
      }
      take(r + off[17], d);
      take(r + off[18], d);
      p += nl * cfg.n_heads + 1;  // contact head
      float* cls = r + off[19];   // [lm_ln_w | lm_ln_b | dense_w | dense_b | dec_w | dec_b]
      take(cls + 3 * d + d * d + V * d, V);
      take(cls + 2 * d, d * d);
      take(cls + 2 * d + d * d, d);
      take(cls, d);
      take(cls + d, d);
      take(cls + 3 * d + d * d, V * d);
      sz[19] = esm::lm_head_floats(cfg) * 4;
      for (int i = 0; i < ESM_NUM_TENSORS; ++i) {
        ptr[i] = r + off[i];
        sizes[i] = static_cast<size_t>(sz[i]);
      }
    } else {
      return fail(c, ESM_EFORMAT,
                  "Invalid FP32 weights size: found " + std::to_string(remaining) + " bytes, expected " +
                      std::to_string(esm::grouped_canonical_floats(cfg) * 4) + " (grouped_canonical_v1) or " +
                      std::to_string(esm::sequential_hf_floats(cfg) * 4) + " (sequential_hf)");
    }
  } else {
    uint64_t off = 0;
    for (int i = 0; i < 19; ++i) {
      if (off + sz[i] > remaining) return fail(c, ESM_EIO, "weights file ends inside tensor " + std::to_string(i));
      ptr[i] = buf.data() + off;
      sizes[i] = static_cast<size_t>(sz[i]);
      off += sz[i];
    }
    const uint64_t rest = remaining - off;
    if (rest % 4) return fail(c, ESM_EFORMAT, "Unaligned trailing bytes: not a multiple of 4");
    ptr[19] = buf.data() + off;
    sizes[19] = static_cast<size_t>(rest);
  }
  return ESM_OK;
}

}  // namespace

int esm_load_file(esm_ctx* c, const char* path, const esm_config* cfg_in) {
  if (!c || !path) return fail(c, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  WeightFile wf;
  const int rc = read_weight_file(c, path, cfg_in, wf);
  if (rc) return rc;
  return load_host_impl(c, wf.cfg, wf.dtype, wf.ptr, wf.sizes);
}

int esm_load_file_quantized(esm_ctx* c, const char* path, const esm_config* cfg_in, int32_t dtype) {
  if (!c || !path) return fail(c, ESM_EINVAL, "null argument");
  if (dtype < ESM_DTYPE_Q8_0 || dtype > ESM_DTYPE_Q3_LUT) return fail(c, ESM_EINVAL, "dtype must be Q8_0, Q4_0 or Q3_LUT");
  std::lock_guard<std::mutex> lk(c->mu);
  WeightFile wf;
  const int rc = read_weight_file(c, path, cfg_in, wf);
  if (rc) return rc;
  // As in load_model_weights, the requested type applies to FP32 files; a quantized file loads as
  // it is stored.
  if (wf.dtype != ESM_DTYPE_FP32) return load_host_impl(c, wf.cfg, wf.dtype, wf.ptr, wf.sizes);
  return load_fp32_as(c, wf.cfg, dtype, wf.ptr, wf.sizes);
}

int esm_load_host_quantized(esm_ctx* c, const esm_config* cfg, int32_t dtype, const void* const* tensors,
                            const size_t* sizes) {
  if (!c || !cfg || !tensors || !sizes) return fail(c, ESM_EINVAL, "null argument");
  if (dtype < ESM_DTYPE_Q8_0 || dtype > ESM_DTYPE_Q3_LUT) return fail(c, ESM_EINVAL, "dtype must be Q8_0, Q4_0 or Q3_LUT");
  std::lock_guard<std::mutex> lk(c->mu);
  return load_fp32_as(c, *cfg, dtype, tensors, sizes);
}

namespace {

// The ranking of esm_contact_top_pairs on a device map; the caller holds the context lock.
int contact_rank_locked(esm_ctx* c, const float* d_map, int32_t n, const char* seq, int32_t min_separation,
                        int32_t max_k, float top_l_factor, int32_t* pos1, int32_t* pos2, float* score,
                        int32_t* n_out, float* cys_enrichment);

}  // namespace

int esm_contact_top_pairs(esm_ctx* c, const float* d_map, int32_t n, const char* seq, int32_t min_separation,
                          int32_t max_k, float top_l_factor, int32_t* pos1, int32_t* pos2, float* score,
                          int32_t* n_out, float* cys_enrichment) {
  if (!c || !d_map || !seq || !pos1 || !pos2 || !score || !n_out || !cys_enrichment)
    return fail(c, ESM_EINVAL, "null argument");
  // compute_pipeline_contacts_parallel asserts n >= 4 (src/pipeline.rs:421).
  if (n < 4) return fail(c, ESM_EINVAL, "Sequence too short for contact prediction");
  if (n > 65535) return fail(c, ESM_EINVAL, "n must be at most 65535 (32-bit pair index)");
  if (min_separation < 0) return fail(c, ESM_EINVAL, "min_separation must be >= 0");
  std::lock_guard<std::mutex> lk(c->mu);
  return contact_rank_locked(c, d_map, n, seq, min_separation, max_k, top_l_factor, pos1, pos2, score, n_out,
                             cys_enrichment);
}

int esm_contacts_pipeline(esm_ctx* c, const char* seq, int32_t min_separation, int32_t max_k, float top_l_factor,
                          float* logits, float* contact_probs, int32_t* pos1, int32_t* pos2, float* score,
                          int32_t* n_out, float* cys_enrichment) {
  if (!c || !seq || !pos1 || !pos2 || !score || !n_out || !cys_enrichment) return fail(c, ESM_EINVAL, "null argument");
  const int32_t n = static_cast<int32_t>(std::strlen(seq));
  if (n < 4) return fail(c, ESM_EINVAL, "Sequence too short for contact prediction");
  if (min_separation < 0) return fail(c, ESM_EINVAL, "min_separation must be >= 0");
  std::lock_guard<std::mutex> lk(c->mu);
  // Tokenizer::encode, then forward_bidirectional* with compute_contacts (src/pipeline.rs:423-445).
  std::vector<int32_t> toks(static_cast<size_t>(n) + 2);
  int32_t L = 0;
  if (esm::tokenize(seq, toks.data(), static_cast<int32_t>(toks.size()), &L) != ESM_OK)
    return fail(c, ESM_EINVAL, "tokenizer capacity");
  // The pipeline indexes the n x n map by byte position (src/pipeline.rs:420, 459-461), which
  // matches the map only when every byte is one token: "<mask>" or a multi-byte character would
  // make it read past the (L - 2)^2 entries the forward wrote.
  if (L - 2 != n) return fail(c, ESM_EINVAL, "the contacts pipeline needs one token per byte of the sequence");
  const int32_t cu[2] = {0, L};
  int rc = validate_call(c, cu, 1, true);
  if (rc) return rc;
  if (!c->has_ch) return fail(c, ESM_EINVAL, "the contact head is not set (esm_set_contact_head)");
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = c->stream;
  rc = upload_plan(c, cu, 1, true, s);
  if (rc) return rc;
  ESM_CUDA(cudaMemcpyAsync(c->tokens, toks.data(), static_cast<size_t>(L) * 4, cudaMemcpyHostToDevice, s));
  rc = forward_impl(c, c->tokens, cu, 1, c->logits, nullptr, c->cmap, nullptr, s);
  if (rc) return rc;
  if (logits)
    ESM_CUDA(cudaMemcpyAsync(logits, c->logits, static_cast<size_t>(L) * c->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, s));
  if (contact_probs)
    ESM_CUDA(cudaMemcpyAsync(contact_probs, c->cmap, static_cast<size_t>(n) * n * 4, cudaMemcpyDeviceToHost, s));
  rc = contact_rank_locked(c, c->cmap, n, seq, min_separation, max_k, top_l_factor, pos1, pos2, score, n_out,
                           cys_enrichment);
  if (rc) return rc;
  ESM_CUDA(cudaStreamSynchronize(s));
  return check_device_word(c);
}

namespace {

int contact_rank_locked(esm_ctx* c, const float* d_map, int32_t n, const char* seq, int32_t min_separation,
                        int32_t max_k, float top_l_factor, int32_t* pos1, int32_t* pos2, float* score,
                        int32_t* n_out, float* cys_enrichment) {
  // Candidate and Cys-Cys pair counts (src/pipeline.rs:454-477).
  int64_t total = 0;
  for (int64_t i = 0; i < n; ++i) total += std::max<int64_t>(0, n - (i + min_separation));
  std::vector<int32_t> cys;
  for (int32_t i = 0; i < n; ++i)
    if (seq[i] == 'C') cys.push_back(i);
  int64_t cys_pairs = 0;
  for (size_t a = 0; a < cys.size(); ++a)
    for (size_t b = a + 1; b < cys.size(); ++b)
      if (cys[b] >= cys[a] + min_separation) ++cys_pairs;
  // top_k (src/pipeline.rs:480-485): max_k, else round(n * top_l_factor) clamped to [5, 50].
  int64_t k;
  if (max_k >= 0) {
    k = std::min<int64_t>(max_k, total);
  } else {
    const float r = std::round(static_cast<float>(n) * top_l_factor);  // f32 product, half away from zero
    const int64_t rk = (r != r || r <= 0.0f) ? 0 : (r >= 9.2e18f ? INT64_MAX : static_cast<int64_t>(r));
    k = std::min<int64_t>(std::min<int64_t>(std::max<int64_t>(rk, 5), 50), total);
  }
  if (k > 4096) return fail(c, ESM_EINVAL, "at most 4096 top pairs are returned");
  int32_t top_cys = 0;
  if (k > 0) {
    const size_t need = static_cast<size_t>(esm::contact_rank_scratch_keys(n, static_cast<int>(k))) + 4096;
    ESM_CUDA(cudaSetDevice(c->device));
    if (need > c->rank_cap) {
      if (c->d_rank) cudaFree(c->d_rank);
      c->d_rank = nullptr;
      c->rank_cap = 0;
      ESM_CUDA(cudaMalloc(&c->d_rank, need * sizeof(uint64_t)));
      c->rank_cap = need;
    }
    uint64_t* out_keys = c->d_rank + (need - 4096);
    ESM_CUDA(esm::launch_contact_rank(d_map, n, min_separation, static_cast<int>(k), c->d_rank, out_keys, c->stream));
    std::vector<uint64_t> keys(static_cast<size_t>(k));
    ESM_CUDA(cudaMemcpyAsync(keys.data(), out_keys, keys.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost, c->stream));
    ESM_CUDA(cudaStreamSynchronize(c->stream));
    for (int64_t t = 0; t < k; ++t) {
      const uint32_t flat = static_cast<uint32_t>(keys[t]);
      const uint32_t asc = ~static_cast<uint32_t>(keys[t] >> 32);
      const uint32_t u = (asc & 0x80000000u) ? (asc & 0x7FFFFFFFu) : ~asc;
      pos1[t] = static_cast<int32_t>(flat / static_cast<uint32_t>(n));
      pos2[t] = static_cast<int32_t>(flat % static_cast<uint32_t>(n));
      std::memcpy(&score[t], &u, 4);
      if (seq[pos1[t]] == 'C' && seq[pos2[t]] == 'C') ++top_cys;
    }
  }
  *n_out = static_cast<int32_t>(k);
  // Enrichment in f32 as the reference computes it (src/pipeline.rs:487-503).
  const float top_density = k > 0 ? static_cast<float>(top_cys) / static_cast<float>(k) : 0.0f;
  const float bg_density = total > 0 ? static_cast<float>(cys_pairs) / static_cast<float>(total) : 0.05f;
  *cys_enrichment = bg_density > 0.0f ? top_density / bg_density : 1.0f;
  return ESM_OK;
}

}  // namespace

int esm_quantize_device(int32_t dtype, const float* d_src, int64_t n, void* d_dst, void* stream) {
  if (!d_src || !d_dst || n < 0 || n % 32) return ESM_EINVAL;
  if (dtype != ESM_DTYPE_Q8_0 && dtype != ESM_DTYPE_Q4_0) return ESM_EINVAL;
  if ((reinterpret_cast<uintptr_t>(d_src) & 15) || (reinterpret_cast<uintptr_t>(d_dst) & 3)) return ESM_EINVAL;
  const cudaError_t e = esm::launch_quantize(dtype, d_src, n / 32, static_cast<uint8_t*>(d_dst),
                                             static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? ESM_OK : ESM_ECUDA;
}

int esm_set_contact_head(esm_ctx* c, const float* w, int32_t nw, float b) {
  if (!c || !w) return fail(c, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  if (!c->loaded) return fail(c, ESM_EINVAL, "load weights before setting the contact head");
  if (nw != c->cfg.n_layers * c->cfg.n_heads)
    return fail(c, ESM_EINVAL, "contact head needs n_layers * n_heads = " +
                                   std::to_string(c->cfg.n_layers * c->cfg.n_heads) + " weights");
  ESM_CUDA(cudaSetDevice(c->device));
  if (!c->d_ch_w) ESM_CUDA(cudaMalloc(&c->d_ch_w, sizeof(float) * nw));
  ESM_CUDA(cudaMemcpyAsync(c->d_ch_w, w, sizeof(float) * nw, cudaMemcpyHostToDevice, c->stream));
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  c->ch_b = b;
  c->has_ch = true;
  return ESM_OK;
}

int esm_reserve(esm_ctx* c, int32_t max_tokens, int32_t max_seqs, int32_t max_len, int32_t contacts) {
  if (!c) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(c->mu);
  return reserve_impl(c, max_tokens, max_seqs, max_len, contacts != 0);
}

int esm_forward_device(esm_ctx* c, const int32_t* d_tokens, const int32_t* h_cu_seqlens, int32_t B, float* d_logits,
                       float* d_hidden, float* d_contacts, float* d_layer_hidden, void* stream, int32_t sync) {
  if (!c || !d_tokens || !h_cu_seqlens || !d_logits) return fail(c, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  int rc = validate_call(c, h_cu_seqlens, B, d_contacts != nullptr);
  if (rc) return rc;
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  rc = forward_impl(c, d_tokens, h_cu_seqlens, B, d_logits, d_hidden, d_contacts, d_layer_hidden, s);
  if (rc) return rc;
  if (sync) {
    ESM_CUDA(cudaStreamSynchronize(s));
    return check_device_word(c);
  }
  return ESM_OK;
}

namespace {

// esm_forward and esm_forward_ext: padded host batch in, padded host outputs out.
int forward_host(esm_ctx* c, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax, float* logits,
                 float* hidden, float* contacts, float* layer_hidden) {
  if (!c || !tokens || !lengths || !logits) return fail(c, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(c->mu);
  if (B <= 0 || Lmax <= 0) return fail(c, ESM_EINVAL, "empty batch");
  std::vector<int32_t> cu(B + 1, 0);
  for (int b = 0; b < B; ++b) {
    if (lengths[b] <= 0 || lengths[b] > Lmax) return fail(c, ESM_EINVAL, "length outside [1, Lmax]");
    cu[b + 1] = cu[b] + lengths[b];
  }
  int rc = validate_call(c, cu.data(), B, contacts != nullptr);
  if (rc) return rc;
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = c->stream;
  const esm_config& g = c->cfg;
  const size_t ntok = static_cast<size_t>(B) * Lmax;
  if (ntok > c->padded_tok_cap) {
    if (c->d_padded_tokens) cudaFree(c->d_padded_tokens);
    c->d_padded_tokens = nullptr;
    c->padded_tok_cap = 0;
    ESM_CUDA(cudaMalloc(&c->d_padded_tokens, ntok * sizeof(int32_t)));
    c->padded_tok_cap = ntok;
  }
  const size_t np = Lmax > 2 ? static_cast<size_t>(Lmax - 2) : 0;
  const size_t out_need = std::max({ntok * g.vocab_size, (hidden || layer_hidden) ? ntok * g.dim : 0,
                                     contacts ? B * np * np : 0});
  // The per-layer residual states [n_layers, T, dim] (packed) are kept only while asked for.
  const size_t layer_need = layer_hidden ? static_cast<size_t>(g.n_layers) * cu[B] * g.dim : 0;
  if (layer_need > c->layer_cap) {
    if (c->d_layers) cudaFree(c->d_layers);
    c->d_layers = nullptr;
    c->layer_cap = 0;
    ESM_CUDA(cudaMalloc(&c->d_layers, layer_need * sizeof(float)));
    c->layer_cap = layer_need;
  }
  if (out_need > c->padded_out_cap) {
    if (c->d_padded_out) cudaFree(c->d_padded_out);
    c->d_padded_out = nullptr;
    c->padded_out_cap = 0;
    ESM_CUDA(cudaMalloc(&c->d_padded_out, out_need * sizeof(float)));
    c->padded_out_cap = out_need;
  }
  // The plan (and with it cu_seqlens on the device) must be in place before the token gather.
  rc = upload_plan(c, cu.data(), B, contacts != nullptr, s);
  if (rc) return rc;
  ESM_CUDA(cudaMemcpyAsync(c->d_padded_tokens, tokens, ntok * sizeof(int32_t), cudaMemcpyHostToDevice, s));
  ESM_CUDA(esm::launch_gather_tokens(c->d_padded_tokens, c->cu, B, Lmax, c->tokens, s));
  rc = forward_impl(c, c->tokens, cu.data(), B, c->logits, hidden ? c->hidden : nullptr, contacts ? c->cmap : nullptr,
                    layer_hidden ? c->d_layers : nullptr, s);
  if (rc) return rc;
  for (int l = 0; layer_hidden && l < g.n_layers; ++l) {
    // Layer by layer through the padded staging buffer: [n_layers, B, Lmax, dim] on the host.
    ESM_CUDA(esm::launch_scatter_rows(c->d_layers + static_cast<size_t>(l) * cu[B] * g.dim, c->cu, B, Lmax, g.dim,
                                      c->d_padded_out, s));
    ESM_CUDA(cudaMemcpyAsync(layer_hidden + static_cast<size_t>(l) * ntok * g.dim, c->d_padded_out,
                             ntok * g.dim * sizeof(float), cudaMemcpyDeviceToHost, s));
  }
  ESM_CUDA(esm::launch_scatter_rows(c->logits, c->cu, B, Lmax, g.vocab_size, c->d_padded_out, s));
  ESM_CUDA(cudaMemcpyAsync(logits, c->d_padded_out, ntok * g.vocab_size * sizeof(float), cudaMemcpyDeviceToHost, s));
  if (hidden) {
    ESM_CUDA(esm::launch_scatter_rows(c->hidden, c->cu, B, Lmax, g.dim, c->d_padded_out, s));
    ESM_CUDA(cudaMemcpyAsync(hidden, c->d_padded_out, ntok * g.dim * sizeof(float), cudaMemcpyDeviceToHost, s));
  }
  if (contacts && np > 0) {
    ESM_CUDA(esm::launch_scatter_maps(c->cmap, c->m_off, c->cu, B, Lmax, c->d_padded_out, s));
    ESM_CUDA(cudaMemcpyAsync(contacts, c->d_padded_out, B * np * np * sizeof(float), cudaMemcpyDeviceToHost, s));
  }
  ESM_CUDA(cudaStreamSynchronize(s));
  return check_device_word(c);
}

}  // namespace

int esm_forward(esm_ctx* c, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax, float* logits,
                float* hidden, float* contacts) {
  return forward_host(c, tokens, lengths, B, Lmax, logits, hidden, contacts, nullptr);
}

int esm_forward_ext(esm_ctx* c, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax, float* logits,
                    float* hidden, float* contacts, float* layer_hidden) {
  return forward_host(c, tokens, lengths, B, Lmax, logits, hidden, contacts, layer_hidden);
}

int esm_dms_wildtype_marginal(esm_ctx* c, const int32_t* residues, int32_t n, int32_t window_size, int32_t stride,
                              float* deltas, float* entropy) {
  if (!c || !residues || !deltas || !entropy) return fail(c, ESM_EINVAL, "null argument");
  if (n <= 0) return fail(c, ESM_EINVAL, "Sequence cannot be empty");
  std::lock_guard<std::mutex> lk(c->mu);
  if (!c->loaded) return fail(c, ESM_EINVAL, "no weights loaded");
  for (int32_t i = 0; i < n; ++i)  // the wild-type ids index the logits rows
    if (residues[i] < 0 || residues[i] >= c->cfg.vocab_size) return fail(c, ESM_EINVAL, "residue token id out of range");
  if (c->cap_tokens == 0) return fail(c, ESM_EINVAL, "call esm_reserve before the first forward");
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = c->stream;
  const int max_len = c->cfg.max_seq_len;
  // Window arithmetic of run_pipeline_dms_with_mode (src/pipeline.rs:88-94, 176-291).
  const int W = (n <= window_size || window_size == 0) ? std::min(n, max_len) : std::min(window_size, max_len);
  if (W + 2 > c->cap_len)
    return fail(c, ESM_ECAPACITY, "window of " + std::to_string(W + 2) + " tokens exceeds max_len " +
                                      std::to_string(c->cap_len));
  if (W + 2 > c->cap_tokens) return fail(c, ESM_ECAPACITY, "window exceeds the reserved token capacity");
  // Windows [w_start, w_end) and the positions each one scores: one window when the sequence fits,
  // else windows `step` apart (stride when 0 < stride <= W, else W / 2), the last one ending at n;
  // every position is scored by the first window that covers it.
  struct Win { int start, end, first; };
  std::vector<Win> wins;
  if (n <= W) {
    wins.push_back({0, n, 0});
  } else {
    const int step = (stride > 0 && stride <= W) ? stride : std::max(W / 2, 1);
    int covered = 0, w_start = 0;
    while (covered < n) {
      const int w_end = std::min(w_start + W, n);
      wins.push_back({w_start, w_end, covered});
      covered = w_end;
      if (w_end >= n) break;
      w_start = std::min(w_start + step, n - W);
    }
  }
  // Staging: tok_row[n] | wt_tok[n] | deltas[20 n] | entropy[n]
  const size_t need = static_cast<size_t>(n) * (2 * 4 + 21 * 4);
  if (need > c->dms_cap) {
    if (c->d_dms) cudaFree(c->d_dms);
    c->d_dms = nullptr;
    c->dms_cap = 0;
    ESM_CUDA(cudaMalloc(&c->d_dms, need));
    c->dms_cap = need;
  }
  int32_t* d_row = static_cast<int32_t*>(c->d_dms);
  int32_t* d_wt = d_row + n;
  float* d_delta = reinterpret_cast<float*>(d_wt + n);
  float* d_ent = d_delta + static_cast<size_t>(20) * n;
  std::vector<int32_t> toks, cu{0}, rows, wts;
  int p0 = 0;  // first position scored by the current batch
  for (size_t w = 0; w <= wins.size(); ++w) {
    const bool flush = (w == wins.size()) || static_cast<int>(cu.size()) - 1 == c->cap_seqs ||
                       cu.back() + (wins[w].end - wins[w].start) + 2 > c->cap_tokens;
    if (flush && cu.size() > 1) {
      // One batch of windows through the forward, then score the rows of their positions.
      const int B = static_cast<int>(cu.size()) - 1;
      const int nr = static_cast<int>(rows.size());
      int rc = validate_call(c, cu.data(), B, false);
      if (rc) return rc;
      ESM_CUDA(cudaMemcpyAsync(c->tokens, toks.data(), toks.size() * 4, cudaMemcpyHostToDevice, s));
      ESM_CUDA(cudaMemcpyAsync(d_row + p0, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, s));
      ESM_CUDA(cudaMemcpyAsync(d_wt + p0, wts.data(), wts.size() * 4, cudaMemcpyHostToDevice, s));
      rc = forward_impl(c, c->tokens, cu.data(), B, c->logits, nullptr, nullptr, nullptr, s);
      if (rc) return rc;
      ESM_CUDA(esm::launch_dms_score(c->logits, c->cfg.vocab_size, d_row + p0, d_wt + p0, nr,
                                     d_delta + static_cast<size_t>(20) * p0, d_ent + p0, s));
      ESM_CUDA(cudaStreamSynchronize(s));  // the host vectors are reused by the next batch
      p0 += nr;
      toks.clear();
      rows.clear();
      wts.clear();
      cu.assign(1, 0);
    }
    if (w == wins.size()) break;
    const Win& wi = wins[w];
    const int base = cu.back();
    toks.push_back(0);
    for (int i = wi.start; i < wi.end; ++i) toks.push_back(residues[i]);
    toks.push_back(2);
    for (int p = wi.first; p < wi.end; ++p) {
      rows.push_back(base + (p - wi.start) + 1);
      wts.push_back(residues[p]);
    }
    cu.push_back(base + (wi.end - wi.start) + 2);
  }
  ESM_CUDA(cudaMemcpyAsync(deltas, d_delta, static_cast<size_t>(20) * n * 4, cudaMemcpyDeviceToHost, s));
  ESM_CUDA(cudaMemcpyAsync(entropy, d_ent, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, s));
  ESM_CUDA(cudaStreamSynchronize(s));
  return check_device_word(c);
}

namespace {

// Masked-marginal rows of positions [pb, pe) of the n-residue sequence into deltas[(pe - pb), 20]
// and entropy[pe - pb] (host).
int dms_masked_impl(esm_ctx* c, const int32_t* residues, int32_t n, int32_t window_size, int32_t pb, int32_t pe,
                    float* deltas, float* entropy) {
  if (!c || !residues || !deltas || !entropy) return fail(c, ESM_EINVAL, "null argument");
  if (n <= 0) return fail(c, ESM_EINVAL, "Sequence cannot be empty");
  if (pb < 0 || pe > n || pb >= pe) return fail(c, ESM_EINVAL, "position range must satisfy 0 <= begin < end <= n");
  std::lock_guard<std::mutex> lk(c->mu);
  if (!c->loaded) return fail(c, ESM_EINVAL, "no weights loaded");
  for (int32_t i = 0; i < n; ++i)  // the wild-type ids index the logits rows
    if (residues[i] < 0 || residues[i] >= c->cfg.vocab_size) return fail(c, ESM_EINVAL, "residue token id out of range");
  if (c->cap_tokens == 0) return fail(c, ESM_EINVAL, "call esm_reserve before the first forward");
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = c->stream;
  const int max_len = c->cfg.max_seq_len;
  // Window arithmetic of run_pipeline_dms_with_mode (src/pipeline.rs:88-94, 111-121).
  const int actual_window = (n <= window_size || window_size == 0) ? std::min(n, max_len) : std::min(window_size, max_len);
  const int half_w = actual_window / 2;
  if (actual_window + 2 > c->cap_len)
    return fail(c, ESM_ECAPACITY, "window of " + std::to_string(actual_window + 2) + " tokens exceeds max_len " +
                                      std::to_string(c->cap_len));
  // Staging: tok_row[m] | wt_tok[m] | deltas[20 m] | entropy[m] for the m = pe - pb positions.
  const int m = pe - pb;
  const size_t need = static_cast<size_t>(m) * (2 * 4 + 21 * 4);
  if (need > c->dms_cap) {
    if (c->d_dms) cudaFree(c->d_dms);
    c->d_dms = nullptr;
    c->dms_cap = 0;
    ESM_CUDA(cudaMalloc(&c->d_dms, need));
    c->dms_cap = need;
  }
  int32_t* d_row = static_cast<int32_t*>(c->d_dms);
  int32_t* d_wt = d_row + m;
  float* d_delta = reinterpret_cast<float*>(d_wt + m);
  float* d_ent = d_delta + static_cast<size_t>(20) * m;
  std::vector<int32_t> toks, cu{0}, rows, wts;
  int p0 = 0;  // first position of the current batch, relative to pb
  for (int p = pb; p <= pe; ++p) {
    const bool flush = (p == pe) || static_cast<int>(cu.size()) - 1 == c->cap_seqs ||
                       cu.back() + actual_window + 2 > c->cap_tokens;
    if (flush && cu.size() > 1) {
      // One batch of masked variants through the forward, then score their masked rows.
      const int B = static_cast<int>(cu.size()) - 1;
      int rc = validate_call(c, cu.data(), B, false);
      if (rc) return rc;
      ESM_CUDA(cudaMemcpyAsync(c->tokens, toks.data(), toks.size() * 4, cudaMemcpyHostToDevice, s));
      ESM_CUDA(cudaMemcpyAsync(d_row + p0, rows.data(), rows.size() * 4, cudaMemcpyHostToDevice, s));
      ESM_CUDA(cudaMemcpyAsync(d_wt + p0, wts.data(), wts.size() * 4, cudaMemcpyHostToDevice, s));
      rc = forward_impl(c, c->tokens, cu.data(), B, c->logits, nullptr, nullptr, nullptr, s);
      if (rc) return rc;
      ESM_CUDA(esm::launch_dms_score(c->logits, c->cfg.vocab_size, d_row + p0, d_wt + p0, B,
                                     d_delta + static_cast<size_t>(20) * p0, d_ent + p0, s));
      // The host vectors are reused by the next batch: wait for this batch's uploads.
      ESM_CUDA(cudaStreamSynchronize(s));
      toks.clear();
      rows.clear();
      wts.clear();
      cu.assign(1, 0);
      p0 = p - pb;
    }
    if (p == pe) break;
    int w_start;
    if (p < half_w) w_start = 0;
    else if (p + half_w > n) w_start = std::max(n - actual_window, 0);
    else w_start = p - half_w;
    const int w_end = std::min(w_start + actual_window, n);
    const int rel = p - w_start;
    const int base = cu.back();
    toks.push_back(0);
    for (int i = w_start; i < w_end; ++i) toks.push_back(residues[i]);
    toks.push_back(2);
    toks[base + rel + 1] = 32;
    rows.push_back(base + rel + 1);
    wts.push_back(residues[p]);
    cu.push_back(base + (w_end - w_start) + 2);
  }
  ESM_CUDA(cudaMemcpyAsync(deltas, d_delta, static_cast<size_t>(20) * m * 4, cudaMemcpyDeviceToHost, s));
  ESM_CUDA(cudaMemcpyAsync(entropy, d_ent, static_cast<size_t>(m) * 4, cudaMemcpyDeviceToHost, s));
  ESM_CUDA(cudaStreamSynchronize(s));
  return check_device_word(c);
}

}  // namespace

int esm_dms_masked_marginal(esm_ctx* c, const int32_t* residues, int32_t n, int32_t window_size, float* deltas,
                            float* entropy) {
  return dms_masked_impl(c, residues, n, window_size, 0, n, deltas, entropy);
}

int esm_dms_masked_marginal_range(esm_ctx* c, const int32_t* residues, int32_t n, int32_t window_size,
                                  int32_t pos_begin, int32_t pos_end, float* deltas, float* entropy) {
  return dms_masked_impl(c, residues, n, window_size, pos_begin, pos_end, deltas, entropy);
}

int esm_matmul_tiled(esm_ctx* c, int32_t dtype, const float* x, const void* w, const float* bias, int32_t in_dim,
                     int32_t out_dim, int32_t seq_len, float* out) {
  if (!c || !x || !w || !out) return fail(c, ESM_EINVAL, "null argument");
  if (dtype < 0 || dtype > 3) return fail(c, ESM_EINVAL, "dtype must be FP32, Q8_0, Q4_0 or Q3_LUT");
  if (in_dim <= 0 || in_dim % 32 || out_dim <= 0 || seq_len <= 0)
    return fail(c, ESM_EINVAL, "in_dim must be a positive multiple of 32; out_dim and seq_len positive");
  std::lock_guard<std::mutex> lk(c->mu);
  ESM_CUDA(cudaSetDevice(c->device));
  cudaStream_t s = c->stream;
  const int n_pad = (out_dim + 15) / 16 * 16;
  const int bn = esm::gemm_pick_bn_any(n_pad);
  const int64_t rows = (static_cast<int64_t>(seq_len) + 127) / 128 * 128;
  const int64_t wbytes = esm::matrix_bytes(dtype, static_cast<int64_t>(out_dim) * in_dim);
  std::vector<void*> tmp;
  float *x32 = nullptr, *b32 = nullptr, *o32 = nullptr;
  __half *x16 = nullptr, *w16 = nullptr;
  uint8_t* wd = nullptr;
  int rc = dev_alloc(c, tmp, &x32, static_cast<size_t>(seq_len) * in_dim);
  if (!rc) rc = dev_alloc(c, tmp, &x16, static_cast<size_t>(rows) * in_dim);
  if (!rc) rc = dev_alloc(c, tmp, &wd, static_cast<size_t>(wbytes));
  if (!rc) rc = dev_alloc(c, tmp, &w16, static_cast<size_t>(n_pad) * in_dim);
  if (!rc) rc = dev_alloc(c, tmp, &b32, static_cast<size_t>(n_pad));
  if (!rc) rc = dev_alloc(c, tmp, &o32, static_cast<size_t>(seq_len) * n_pad);
  auto done = [&](int code) {
    cudaStreamSynchronize(s);
    free_list(tmp);
    return code;
  };
  if (rc) return done(rc);
  CUtensorMap ta, tb;
  esm::GemmParams p{};
  cudaError_t e = cudaMemsetAsync(x16, 0, rows * in_dim * 2, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(w16, 0, static_cast<size_t>(n_pad) * in_dim * 2, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(b32, 0, static_cast<size_t>(n_pad) * 4, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(x32, x, static_cast<size_t>(seq_len) * in_dim * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(wd, w, static_cast<size_t>(wbytes), cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && bias) e = cudaMemcpyAsync(b32, bias, static_cast<size_t>(out_dim) * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = esm::launch_to_f16(ESM_DTYPE_FP32, x32, static_cast<int64_t>(seq_len) * in_dim, x16, s);
  if (e == cudaSuccess) e = esm::launch_to_f16(dtype, wd, static_cast<int64_t>(out_dim) * in_dim, w16, s);
  if (e != cudaSuccess) return done(fail(c, ESM_ECUDA, std::string("matmul_tiled setup: ") + cudaGetErrorString(e)));
  if (!esm::make_tmap_f16(&ta, x16, rows, in_dim, in_dim, 128) ||
      !esm::make_tmap_f16(&tb, w16, n_pad, in_dim, in_dim, bn / 2))
    return done(fail(c, ESM_ECUDA, "cuTensorMapEncodeTiled failed"));
  p.M = seq_len;
  p.N = n_pad;
  p.K = in_dim;
  p.bias = b32;
  p.out = o32;
  p.ldo = n_pad;
  p.err = c->d_err;
  e = esm::gemm_launch(ta, tb, nullptr, bn, esm::kEpiStoreF32, 0, p, c->num_sms, s, c->cta_pair);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(out, static_cast<size_t>(out_dim) * 4, o32, static_cast<size_t>(n_pad) * 4,
                          static_cast<size_t>(out_dim) * 4, seq_len, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return done(fail(c, ESM_ECUDA, std::string("matmul_tiled: ") + cudaGetErrorString(e)));
  return done(check_device_word(c));
}

int esm_profile_enable(esm_ctx* c, int32_t enable) {
  if (!c) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(c->mu);
  ESM_CUDA(cudaSetDevice(c->device));
  ESM_CUDA(cudaDeviceSynchronize());
  c->prof = enable != 0;
  c->prof_recs.clear();
  c->ev_used = 0;
  return ESM_OK;
}

int esm_profile_read(esm_ctx* c, int32_t kind, double* total_ms, int64_t* launches, double* flops, double* bytes) {
  if (!c || kind < 0 || kind >= ESM_PROF_KINDS) return fail(c, ESM_EINVAL, "bad profile kind");
  std::lock_guard<std::mutex> lk(c->mu);
  double ms = 0.0, fl = 0.0, by = 0.0;
  int64_t n = 0;
  for (const auto& r : c->prof_recs) {
    if (r.kind != kind) continue;
    ESM_CUDA(cudaEventSynchronize(r.b));
    float t = 0.0f;
    ESM_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
    ms += t;
    fl += r.flops;
    by += r.bytes;
    ++n;
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = n;
  if (flops) *flops = fl;
  if (bytes) *bytes = by;
  return ESM_OK;
}

int esm_probe_wait_timeout(esm_ctx* c, int32_t limit_ms) {
  if (!c || limit_ms <= 0 || limit_ms > 2000) return fail(c, ESM_EINVAL, "limit_ms must be in (0, 2000]");
  std::lock_guard<std::mutex> lk(c->mu);
  ESM_CUDA(cudaSetDevice(c->device));
  ESM_CUDA(esm::launch_wait_probe(c->d_err, static_cast<uint64_t>(limit_ms) * 1000000ull, c->stream));
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  return check_device_word(c);
}

int esm_check_device(esm_ctx* c) {
  if (!c) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(c->mu);
  ESM_CUDA(cudaSetDevice(c->device));
  ESM_CUDA(cudaStreamSynchronize(c->stream));
  return check_device_word(c);
}

}  // extern "C"
