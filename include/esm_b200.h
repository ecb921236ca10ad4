/*
 * esm_b200.h - C ABI of the B200 (sm_100a) ESM-2 bidirectional encoder forward.
 *
 * Drop-in for the hot path of codon-infer v1.12.0 (Rust crate, src/lib.rs): the
 * forward_bidirectional* family, its weight formats and its outputs. Plain C types only, so the
 * Rust host binds it with an `extern "C"` block. Every function returns an
 * ESM_* status code and never aborts; esm_last_error() gives the message of the last failure on a
 * context.
 *
 * Threading: one context per GPU. Calls on one context are serialised by an internal mutex;
 * contexts on different devices may be driven concurrently from different host threads.
 */
#ifndef ESM_B200_H_
#define ESM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (replace io::Result errors and assert!/index panics of the reference). */
enum {
  ESM_OK = 0,
  ESM_EINVAL = 1,    /* bad argument (null pointer, bad shape, unknown arch)             */
  ESM_EFORMAT = 2,   /* weight file/blob does not match the declared format (InvalidData) */
  ESM_ECAPACITY = 3, /* request exceeds the reserved workspace (reference: assert! panic)  */
  ESM_ECUDA = 4,     /* CUDA runtime error                                                 */
  ESM_ENCCL = 5,     /* reserved for collective failures                                   */
  ESM_ETIMEOUT = 6,  /* a device-side bounded wait gave up; the context stays usable       */
  ESM_ENOMEM = 7,    /* device or host allocation failed                                   */
  ESM_EIO = 8        /* file could not be opened/read (io::ErrorKind::NotFound, UnexpectedEof) */
};

/* Weight storage types: CODQ dtype ids, src/lib.rs:874-876. */
enum { ESM_DTYPE_FP32 = 0, ESM_DTYPE_Q8_0 = 1, ESM_DTYPE_Q4_0 = 2, ESM_DTYPE_Q3_LUT = 3 };

/* Architecture ids: CODQ arch ids, src/lib.rs:879-883. */
enum { ESM_ARCH_8M = 0, ESM_ARCH_35M = 1, ESM_ARCH_150M = 2, ESM_ARCH_650M = 3, ESM_ARCH_3B = 4 };

/* EsmConfig, src/lib.rs:76-84. */
typedef struct esm_config {
  int32_t dim;
  int32_t hidden_dim;
  int32_t n_layers;
  int32_t n_heads;
  int32_t vocab_size;
  int32_t max_seq_len;
  int32_t arch;
} esm_config;

typedef struct esm_ctx esm_ctx;

/* Number of tensors in the EsmWeights field order (src/lib.rs:299-307), which is also the
 * grouped_canonical_v1 / CODQ file order (src/lib.rs:369-389, 1175-1193):
 *  0 tok_emb  1 ln1_w  2 ln1_b  3 wq  4 bq  5 wk  6 bk  7 wv  8 bv  9 wo  10 bo
 * 11 ln2_w 12 ln2_b 13 fc1_w 14 fc1_b 15 fc2_w 16 fc2_b 17 lnf_w 18 lnf_b 19 classifier
 * Matrices are row-major [out, in] (src/lib.rs:2629-2634); for Q8_0/Q4_0 they are arrays of
 * BlockQ8_0 (36 B) / BlockQ4_0 (20 B) along `in`. tok_emb is Q8_0 blocks for Q8_0 models and
 * FP32 otherwise (src/lib.rs:744-746, docs/Q4_0_SPEC.md:88-92). */
#define ESM_NUM_TENSORS 20

/* ---- configuration ------------------------------------------------------------------------ */

/* EsmConfig::esm2_8m() .. esm2_3b(), src/lib.rs:87-150. */
int esm_config_preset(int32_t arch, esm_config* out);

/* EsmConfig::detect_from_file, src/lib.rs:277-297: CODQ header if present, otherwise the file
 * length table of detect_from_file_len (src/lib.rs:228-275). *dtype receives the storage type
 * (FP32 for header-less files). */
int esm_config_detect_file(const char* path, esm_config* out, int32_t* dtype);

/* The configuration and storage type of the weights loaded into ctx (ESM_EINVAL before a load);
 * with a CODQ header it is the header's, which may differ from the config a loader was given. */
int esm_get_config(const esm_ctx* ctx, esm_config* out, int32_t* dtype);

/* ---- quantizers (bit-exact with the reference) ---------------------------------------------- */

/* quantize_slice_to_q8 / BlockQ8_0::quantize, src/lib.rs:648-673: n % 32 == 0,
 * dst holds n/32 blocks of 36 bytes. */
int esm_quantize_q8(const float* src, int64_t n, void* dst);
/* quantize_slice_to_q4 / BlockQ4_0::quantize, src/lib.rs:1054-1088: dst holds n/32 x 20 bytes. */
int esm_quantize_q4(const float* src, int64_t n, void* dst);
/* quantize_slice_to_q3_lut / BlockQ3_LUT::quantize, src/lib.rs:1353-1458, 1511-1514: dst holds
 * n/32 x 14 bytes (32 sign bits, 32 two-bit level indices, the f16 scale of the reference's
 * truncating conversion). A Q3_LUT model (EsmWeights::quantize_q3, src/lib.rs:609-633) stores fc1
 * and fc2 this way and its attention matrices as Q4_0. */
int esm_quantize_q3(const float* src, int64_t n, void* dst);
/* The same two quantizers on device memory (dtype ESM_DTYPE_Q8_0 or ESM_DTYPE_Q4_0): d_src holds
 * n FP32 values (n % 32 == 0, 16-byte aligned), d_dst receives the n/32 blocks (4-byte aligned),
 * byte-identical to esm_quantize_q8/q4. Enqueued on `stream` (a cudaStream_t; NULL = the legacy
 * default stream); the caller synchronises. */
int esm_quantize_device(int32_t dtype, const float* d_src, int64_t n, void* d_dst, void* stream);

/* Tokenizer::encode, src/lib.rs:6511-6521: <cls> + ids + <eos>; returns ESM_ECAPACITY if the
 * sequence needs more than `cap` tokens. *n_out receives the token count. */
int esm_tokenize(const char* seq, int32_t* out, int32_t cap, int32_t* n_out);

/* ---- contact post-processing ------------------------------------------------------------ */

/* The pair ranking and Cys enrichment of compute_pipeline_contacts_parallel (src/pipeline.rs:410-512)
 * on a contact map in device memory (one sequence's n x n probabilities, row-major, e.g. its slice of
 * esm_forward_device's contacts; n = residues = L - 2 >= 4): the pairs (i, j) with
 * j >= i + min_separation, in descending probability with ties in (i, j) order (the reference's
 * stable sort), the first k of them into pos1/pos2/score (host arrays of k entries; *n_out = k),
 * where k = min(max_k, #candidates) for max_k >= 0, else round(n * top_l_factor) clamped to [5, 50]
 * and to #candidates; k may not exceed 4096, n not 65535. seq holds the n residue letters (host memory);
 * *cys_enrichment = (Cys-Cys share of the k pairs) / (Cys-Cys share of all candidates), computed in
 * f32 as the reference does. The map is not copied to the host. */
int esm_contact_top_pairs(esm_ctx* ctx, const float* d_map, int32_t n, const char* seq, int32_t min_separation,
                          int32_t max_k, float top_l_factor, int32_t* pos1, int32_t* pos2, float* score,
                          int32_t* n_out, float* cys_enrichment);

/* compute_pipeline_contacts_parallel (src/pipeline.rs:410-512) for one sequence in one call: seq is
 * the residue string (n >= 4 letters, tokenized as Tokenizer::encode, one token per byte: "<mask>"
 * or a multi-byte character is ESM_EINVAL, since the pipeline indexes the map by byte); the forward with contacts
 * (contact head set, workspace reserved for n + 2 tokens with contacts) and the ranking of
 * esm_contact_top_pairs run on the GPU, so the map crosses to the host only when contact_probs
 * ([n, n], host) is given; logits ([n + 2, vocab], host) is optional too. Outputs as in
 * esm_contact_top_pairs. */
int esm_contacts_pipeline(esm_ctx* ctx, const char* seq, int32_t min_separation, int32_t max_k, float top_l_factor,
                          float* logits, float* contact_probs, int32_t* pos1, int32_t* pos2, float* score,
                          int32_t* n_out, float* cys_enrichment);

/* ---- context ------------------------------------------------------------------------------ */

int esm_ctx_create(int32_t device, esm_ctx** out);
int esm_ctx_destroy(esm_ctx* ctx);
const char* esm_last_error(const esm_ctx* ctx);

/* EsmWeights{,Q8,Q4}::from_file, src/lib.rs:310-547, 744-830, 1156-1242. `cfg` may be NULL to
 * autodetect (EsmWeights*::load_from_file). Uploads to the context's device. */
int esm_load_file(esm_ctx* ctx, const char* path, const esm_config* cfg);

/* Upload weights from host memory: tensors[i] / sizes[i] (bytes) in the order above. */
int esm_load_host(esm_ctx* ctx, const esm_config* cfg, int32_t dtype, const void* const* tensors,
                  const size_t* sizes);

/* EsmWeights::quantize_q8 / quantize_q4 / quantize_q3 (src/lib.rs:559-633) done while uploading:
 * tensors / sizes are an FP32 weight set (the ESM_DTYPE_FP32 layout). For Q8_0 / Q4_0 the six
 * matrices of every layer (and for Q8_0 the token embedding) are quantized on the GPU; for Q3_LUT
 * the four attention matrices are quantized to Q4_0 on the GPU and fc1 / fc2 to Q3_LUT on the host.
 * Block for block identical to the host quantizers. */
int esm_load_host_quantized(esm_ctx* ctx, const esm_config* cfg, int32_t dtype, const void* const* tensors,
                            const size_t* sizes);

/* load_model_weights with QuantizationMode::Q8_0 / Q4_0 / Q3_LUT (src/main.rs:137-244): an FP32
 * weight file is quantized while loading (as esm_load_host_quantized); a quantized file loads as it
 * is stored. */
int esm_load_file_quantized(esm_ctx* ctx, const char* path, const esm_config* cfg, int32_t dtype);

/* Contact regression head (EsmConfig::contact_head_weights, src/lib.rs:154-177): w has
 * n_layers * n_heads entries (layer-major), b is the bias. Required before contacts are asked for. */
int esm_set_contact_head(esm_ctx* ctx, const float* w, int32_t nw, float b);

/* Workspace for up to `max_tokens` packed tokens in up to `max_seqs` sequences of at most
 * `max_len` tokens, with room for contact maps when `contacts` != 0 (BidirectionalRunState::new,
 * src/lib.rs:2510-2544). Calls that exceed it fail with ESM_ECAPACITY. */
int esm_reserve(esm_ctx* ctx, int32_t max_tokens, int32_t max_seqs, int32_t max_len, int32_t contacts);

/* ---- forward ------------------------------------------------------------------------------- */

/* Batched forward_bidirectional{_parallel,_q8,_q4} (src/lib.rs:5078-5095, 5442-5448, 5790-5798)
 * from HOST buffers. tokens: [B, Lmax] right-padded; lengths[b] tokens of row b are real (each
 * sequence is computed exactly as if run alone - key-padding mask). Outputs (host):
 *   logits   [B, Lmax, vocab]   (state.logits)                        required
 *   hidden   [B, Lmax, dim]     (state.x = LN_f(x) after the call)     or NULL
 *   contacts [B, Lmax-2, Lmax-2] sigmoid contact map, row-major over each sequence's own
 *            n = lengths[b]-2 rows/cols at the top-left (state.contact_probs)  or NULL
 * Padding positions of the outputs are set to 0. */
int esm_forward(esm_ctx* ctx, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax,
                float* logits, float* hidden, float* contacts);

/* esm_forward plus the residual stream after every layer, the values the on_layer hook of
 * forward_bidirectional_parallel_ext / _q4_ext / _q3_ext receives (src/lib.rs:5097-5103, 5368-5370,
 * 5800-5807, 6159-6165): layer_hidden [n_layers, B, Lmax, dim] (host, padding positions zero) or
 * NULL, which makes the call identical to esm_forward. The states are kept on the device only
 * while a call asks for them. */
int esm_forward_ext(esm_ctx* ctx, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax,
                    float* logits, float* hidden, float* contacts, float* layer_hidden);

/* Same forward on DEVICE buffers of the context's GPU, packed (varlen) layout:
 *   d_tokens [T] with T = sum of lengths; h_cu_seqlens [B+1] host prefix sums of the lengths.
 *   d_logits [T, vocab]; d_hidden [T, dim] or NULL; d_contacts packed per sequence (n_b*n_b
 *   floats each, n_b = len_b - 2, in sequence order) or NULL;
 *   d_layer_hidden [n_layers, T, dim] residual stream after each layer (the on_layer hook of
 *   forward_bidirectional_parallel_ext, src/lib.rs:5097-5103) or NULL.
 * Enqueued on `stream` (a cudaStream_t, NULL = the context's stream); returns after enqueueing
 * unless `sync` != 0. */
int esm_forward_device(esm_ctx* ctx, const int32_t* d_tokens, const int32_t* h_cu_seqlens, int32_t B,
                       float* d_logits, float* d_hidden, float* d_contacts, float* d_layer_hidden,
                       void* stream, int32_t sync);

/* In-silico deep mutational scan, masked-marginal mode (run_pipeline_dms_with_mode with
 * DmsScoringMode::MaskedMarginal, src/pipeline.rs:76-175): for every position p of the residue
 * tokens (ids 4..30, no <cls>/<eos>) the window around p (same centring rule and window_size
 * semantics as the reference; 0 = whole sequence) is encoded, position p is replaced by <mask>,
 * and the logits at p give log_softmax_canonical, the Shannon entropy entropy[p] and
 * deltas[p, c] = logP(aa_c) - logP(wt) for the 20 CANONICAL_AAS (A C D E F G H I K L M N P Q R S T
 * V W Y; 0 for the wild type). All n masked variants run as batches of independent sequences
 * through the forward, limited by the reserved workspace. Outputs are HOST buffers. */
int esm_dms_masked_marginal(esm_ctx* ctx, const int32_t* residues, int32_t n, int32_t window_size, float* deltas,
                            float* entropy);

/* The rows p in [pos_begin, pos_end) of esm_dms_masked_marginal on the same n-residue sequence
 * (same windows, same values): deltas [pos_end - pos_begin, 20] and entropy [pos_end - pos_begin],
 * HOST buffers. This is the per-position loop body of src/pipeline.rs:111-174 over a contiguous
 * block of positions: the unit by which a scan is split across GPUs. */
int esm_dms_masked_marginal_range(esm_ctx* ctx, const int32_t* residues, int32_t n, int32_t window_size,
                                  int32_t pos_begin, int32_t pos_end, float* deltas, float* entropy);

/* The same scan in wild-type-marginal mode (DmsScoringMode::WildtypeMarginal, src/pipeline.rs:176-291):
 * no masking; the whole sequence is one forward when it fits the window (window_size semantics as
 * above), otherwise windows of that size `stride` residues apart (stride in (0, window], else half a
 * window), the last one ending at the sequence end, and every position is scored from the first
 * window that covers it. deltas / entropy as above; all windows run as batches of independent
 * sequences. Outputs are HOST buffers. */
int esm_dms_wildtype_marginal(esm_ctx* ctx, const int32_t* residues, int32_t n, int32_t window_size, int32_t stride,
                              float* deltas, float* entropy);

/* matmul_tiled_{fp32,q8,q4}_parallel (src/lib.rs:4803-4827, 4870-4894, 4937-4961) on the GPU, from
 * HOST buffers: out[p, i] = sum_k W[i, k] * x[p, k] + bias[i] for p < seq_len, i < out_dim.
 * w is FP32 [out_dim, in_dim] or rows of BlockQ8_0 / BlockQ4_0 (dtype); x is FP32 [seq_len, in_dim];
 * bias [out_dim] or NULL (zero). Weights are dequantized (q*d) and both operands rounded to fp16
 * for the tensor cores; accumulation is fp32. in_dim must be a multiple of 32. */
int esm_matmul_tiled(esm_ctx* ctx, int32_t dtype, const float* x, const void* w, const float* bias, int32_t in_dim,
                     int32_t out_dim, int32_t seq_len, float* out);

/* No counterpart in the reference. The GEMM of esm_matmul_tiled for callers that cannot allocate
 * device memory (a process whose device memory is all reserved up front by its own allocator, a
 * latency-critical pipeline that cannot take cudaMalloc's device-wide synchronisation, a plugin
 * host that forbids allocation). Inputs and output are the caller's DEVICE buffers: d_x fp32
 * [seq_len, in_dim] and d_out fp32 [seq_len, out_dim] 16-byte aligned, d_w as in esm_matmul_tiled,
 * d_bias [out_dim] or NULL. Its only scratch is a static device array of ESM_NOALLOC_SCRATCH_BYTES
 * that holds the fp16 operand copies (2*(seq_len + out_dim)*in_dim bytes, 256-byte aligned each),
 * the bias padded to a multiple of 16 and, when out_dim % 16 != 0, a padded fp32 output; larger
 * problems return ESM_ECAPACITY. dtype may be any of the four storage types (Q3_LUT blocks need no
 * alignment). The array lives on every GPU where the library's device code is loaded until the
 * process exits. The first call on a device looks up the array's device address and loads the
 * kernels it uses, so make it before any stream capture. Calls on one device share its array:
 * calls that overlap on the same device race and must be serialised by the caller; calls on
 * different devices use each device's own copy. The stream and buffers must belong to the
 * calling thread's current device (otherwise ESM_EINVAL). The call is enqueued on `stream` (a
 * cudaStream_t, NULL = legacy default) and returns once the result is in d_out. */
#define ESM_NOALLOC_SCRATCH_BYTES (32u << 20)
int esm_matmul_tiled_noalloc(int32_t dtype, const float* d_x, const void* d_w, const float* d_bias, int32_t in_dim,
                             int32_t out_dim, int32_t seq_len, float* d_out, void* stream);

/* ---- several GPUs from one host process ------------------------------------------------------ */

/* The reference runs every sequence and every masked variant of a scan as its own forward, one
 * after another on the host (src/pipeline.rs:111-174, 427-444); these calls spread that same work
 * over several GPUs of one box. A group holds one context per listed device, each with a full
 * copy of the weights. A batch is split into contiguous blocks of sequences with balanced cost
 * (esm_partition), a scan into contiguous blocks of positions; one host thread per device runs its
 * block, and each device copies its rows straight into the caller's host arrays, so results are
 * bit for bit those of one context and no data moves between GPUs. */
typedef struct esm_group esm_group;

/* Contiguous blocks of sequences for `parts` devices: bounds[0..parts] (parts + 1 entries,
 * bounds[0] = 0, bounds[parts] = B); block r is [bounds[r], bounds[r+1]) and may be empty. The cost
 * of a sequence of L tokens is one layer's algorithmic FLOPs, 2L(4 dim^2 + 2 dim hidden_dim) for
 * the projections plus 4 L^2 dim for attention; block r ends at the first sequence whose cost
 * prefix reaches (r + 1) / parts of the total. Host-only. */
int esm_partition(const int32_t* lengths, int32_t B, int32_t dim, int32_t hidden_dim, int32_t parts,
                  int32_t* bounds);

/* One context per entry of devices[0..n_devices) (a device may be listed twice: two contexts on
 * one GPU). Members are destroyed by esm_group_destroy. */
int esm_group_create(const int32_t* devices, int32_t n_devices, esm_group** out);
int esm_group_destroy(esm_group* group);
const char* esm_group_last_error(const esm_group* group);
int esm_group_size(const esm_group* group, int32_t* n);
/* Member context i (owned by the group), for per-device calls such as esm_forward_device. */
int esm_group_ctx(esm_group* group, int32_t i, esm_ctx** out);
/* esm_load_host / esm_load_file / esm_set_contact_head / esm_reserve on every member (in
 * parallel). Capacities are per device: a device runs its block in chunks that fit them. */
int esm_group_load_host(esm_group* group, const esm_config* cfg, int32_t dtype, const void* const* tensors,
                        const size_t* sizes);
int esm_group_load_file(esm_group* group, const char* path, const esm_config* cfg);
int esm_group_set_contact_head(esm_group* group, const float* w, int32_t nw, float b);
int esm_group_reserve(esm_group* group, int32_t max_tokens, int32_t max_seqs, int32_t max_len, int32_t contacts);
/* esm_forward over the group: same arguments and outputs (HOST buffers, [B, Lmax, ...] padded). */
int esm_group_forward(esm_group* group, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax,
                      float* logits, float* hidden, float* contacts);
/* esm_dms_masked_marginal over the group: positions split into equal contiguous blocks, one per
 * device (esm_dms_masked_marginal_range); outputs as esm_dms_masked_marginal. */
int esm_group_dms_masked_marginal(esm_group* group, const int32_t* residues, int32_t n, int32_t window_size,
                                  float* deltas, float* entropy);

/* ---- instrumentation (no counterpart in the reference, which only times whole calls) ---------- */

/* Kernel classes reported by esm_profile_read. */
enum {
  ESM_PROF_DEQUANT = 0,   /* per-layer weight dequantization to fp16                 */
  ESM_PROF_NORM = 1,      /* embedding + LayerNorms                                  */
  ESM_PROF_GEMM = 2,      /* tcgen05 projection GEMMs (QKV, O, fc1, fc2, LM dense)   */
  ESM_PROF_ATTENTION = 3, /* attention                                               */
  ESM_PROF_CONTACT = 4,   /* contact-mode accumulation and APC finalize              */
  ESM_PROF_HEAD = 5,      /* LM-head LayerNorm + decoder                             */
  ESM_PROF_KINDS = 6
};

/* enable != 0: every kernel launched by later forwards is bracketed by CUDA events on its own
 * stream and counted per class, with its algorithmic FLOPs and bytes; counters are reset. */
int esm_profile_enable(esm_ctx* ctx, int32_t enable);
/* Totals for one class since the last enable (synchronizes with the recorded events). */
int esm_profile_read(esm_ctx* ctx, int32_t kind, double* total_ms, int64_t* launches, double* flops, double* bytes);

/* Self-test of the device failure path (no counterpart in the reference): one thread waits, with
 * the same bounded mbarrier wait the kernels use but a limit of limit_ms milliseconds, on a phase
 * that nothing completes. Returns ESM_ETIMEOUT when the wait gave up as designed, after which the
 * context is usable again. No trap, fault or unbounded loop is involved. */
int esm_probe_wait_timeout(esm_ctx* ctx, int32_t limit_ms);

/* Device error word check: ESM_ETIMEOUT if a kernel's bounded wait gave up since the last call. */
int esm_check_device(esm_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* ESM_B200_H_ */
