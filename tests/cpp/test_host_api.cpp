// Tests of the C++ host API (codon-infer_b200/host/codon_infer.hpp), written after codon-infer's own
// unit tests in src/lib.rs (mod tests, lines 6834-8459). Run by tests/test_host_cpp.py:
//
//   test_host_api cpu <scratch dir>                 known-answer tests that need no GPU
//   test_host_api forward <file> <fp32|q8|q4> <sequence> <out.bin> <contacts 0|1> <max_len>
//                                                   one forward_bidirectional* call; writes
//                                                   int32 L, vocab, n then logits [L, vocab],
//                                                   contacts [n, n], int32 n_layers and the _ext
//                                                   hook's states [n_layers, L, dim] (none for Q8)
//   test_host_api cosine <fp32 file> <q8 file> <q4 file> <sequence>
//                                                   FP32 vs Q8_0 / Q4_0 logit cosine similarity
//   test_host_api misuse <q4 file>                  the reference's panics and io errors
//   test_host_api pipelines <fp32 file> <sequence> <out.bin>
//                                                   load_model_weights(Q4_0), both DMS modes, the
//                                                   contacts pipeline, Q3_LUT blocks
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <memory>
#include <string>
#include <type_traits>
#include <vector>

#include "../../codon-infer_b200/host/codon_infer.hpp"

using namespace codon_infer;

static int g_failures = 0;
#define CHECK(cond)                                                        \
  do {                                                                     \
    if (!(cond)) {                                                         \
      std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
      ++g_failures;                                                        \
    }                                                                      \
  } while (0)

static std::vector<size_t> ids(std::initializer_list<size_t> l) { return std::vector<size_t>(l); }

// ---- known-answer tests (no GPU) -----------------------------------------------------------

static void test_q8_0_quantization_roundtrip() {  // src/lib.rs:6834-6849
  float src[32], dst[32];
  for (int i = 0; i < 32; ++i) src[i] = (static_cast<float>(i) / 31.0f) * 2.0f - 1.0f;
  BlockQ8_0::quantize(src).dequantize_to(dst);
  float mse = 0.0f;
  for (int i = 0; i < 32; ++i) mse += (src[i] - dst[i]) * (src[i] - dst[i]);
  CHECK(mse / 32.0f < 0.02f);
}

static void test_tokenizer_boundaries() {  // src/lib.rs:6871
  CHECK(Tokenizer::encode("LA") == ids({0, 4, 5, 2}));
}

static void test_mask_token_encoding_and_decoding() {  // src/lib.rs:6921-6926
  CHECK(Tokenizer::encode("M*C") == ids({0, 20, 32, 23, 2}));
  CHECK(Tokenizer::encode("M<mask_1>C") == ids({0, 20, 32, 23, 2}));
  CHECK(Tokenizer::decode(32) == '*');
  CHECK(Tokenizer::decode(4) == 'L' && Tokenizer::decode(30) == '-' && Tokenizer::decode(31) == '\0');
}

static void test_log_softmax_canonical() {  // src/lib.rs:6928-6937
  std::vector<float> logits(33, 1.0f);
  const std::vector<float> lp = log_softmax_canonical(logits.data());
  float s = 0.0f;
  for (int i = 4; i <= 23; ++i) s += std::exp(lp[i]);
  CHECK(std::fabs(s - 1.0f) < 1e-5f);
  CHECK(std::isinf(lp[0]) && lp[0] < 0 && std::isinf(lp[24]));
}

static void test_q4_0_roundtrip_quantize_dequantize_bound() {  // src/lib.rs:7440-7487
  std::vector<std::vector<float>> vecs;
  std::vector<float> v1(32);
  for (int i = 0; i < 32; ++i) v1[i] = -8.0f + static_cast<float>(i) * (15.0f / 31.0f);
  vecs.push_back(v1);
  const float scales[] = {0.05f, 1.0f, 2.5f, 10.0f};
  for (int sign = 0; sign < 2; ++sign) {
    for (float scale : scales) {
      std::vector<float> v(32);
      v[0] = (sign ? 8.0f : -8.0f) * scale;
      for (int i = 1; i < 32; ++i) {
        const float q = static_cast<float>(i % 16 - 8);
        const int mul = sign ? 7 : 11;
        const float noise = (static_cast<float>((i * mul) % 9) - 4.0f) / 10.0f * 0.45f * scale;
        v[i] = q * (sign ? -scale : scale) + noise;
      }
      vecs.push_back(v);
    }
  }
  for (const auto& src : vecs) {
    const BlockQ4_0 b = BlockQ4_0::quantize(src.data());
    float dst[32];
    b.dequantize_to(dst);
    const float bound = std::fabs(b.d) / 2.0f + 1e-5f;
    for (int i = 0; i < 32; ++i) CHECK(std::fabs(src[i] - dst[i]) <= bound);
  }
}

static void test_q4_0_exact_nibble_packing() {  // src/lib.rs:7490-7517
  float src[32], dst[32];
  for (int j = 0; j < 16; ++j) {
    src[j] = static_cast<float>(8 - j);
    src[j + 16] = static_cast<float>(j - 7);
  }
  const BlockQ4_0 b = BlockQ4_0::quantize(src);
  CHECK(b.d == -1.0f);
  for (int j = 0; j < 16; ++j) CHECK(b.qs[j] == static_cast<uint8_t>(j | ((15 - j) << 4)));
  b.dequantize_to(dst);
  for (int i = 0; i < 32; ++i) CHECK(dst[i] == src[i]);
}

static void test_q4_0_zero_block() {  // src/lib.rs:7520-7533
  float z[32] = {0}, dst[32];
  const BlockQ4_0 b = BlockQ4_0::quantize(z);
  CHECK(b.d == 0.0f);
  for (int j = 0; j < 16; ++j) CHECK(b.qs[j] == 0x88);
  for (float& x : dst) x = 999.0f;
  b.dequantize_to(dst);
  for (float x : dst) CHECK(x == 0.0f);
}

static void test_quantize_slice_rejects_ragged_length() {
  bool threw = false;
  try {
    quantize_slice_to_q4(std::vector<float>(33, 1.0f));
  } catch (const std::logic_error&) {
    threw = true;
  }
  CHECK(threw);
  CHECK(quantize_slice_to_q8(std::vector<float>(64, 1.0f)).size() == 2);
}

static void test_dms_row() {  // test_dms_row_and_csv_generation (src/export.rs:2603-2608), DmsPositionRow::new
  const float zeros[20] = {0};
  const DmsPositionRow row = DmsPositionRow::make(1, 'M', zeros, 2.5f);
  CHECK(row.pos == 1 && row.wt == 'M' && row.mean_delta_logp == 0.0f && row.entropy == 2.5f);
  CHECK(std::string(row.category) == "Tolerated Variable");
  // The mean is over the 19 non-zero deltas; the thresholds are -3.8 and -2.2 (src/export.rs:16-38).
  const std::pair<float, const char*> cases[] = {{-4.0f, "Catalytic / Strictly Intolerant"},
                                                 {-3.0f, "Conserved Structural Core"},
                                                 {-2.0f, "Tolerated Variable"}};
  for (const auto& [v, want] : cases) {
    float d[20];
    for (float& x : d) x = v;
    d[7] = 0.0f;  // the wild type
    const DmsPositionRow r = DmsPositionRow::make(2, 'A', d, 1.0f);
    CHECK(std::fabs(r.mean_delta_logp - v) < 1e-5f);
    CHECK(std::string(r.category) == want);
  }
}

static void test_config_presets() {  // src/lib.rs:87-150
  const EsmConfig c8 = EsmConfig::esm2_8m();
  CHECK(c8.dim == 320 && c8.hidden_dim == 1280 && c8.n_layers == 6 && c8.n_heads == 20 && c8.head_dim() == 16);
  const EsmConfig c650 = EsmConfig::esm2_650m();
  CHECK(c650.dim == 1280 && c650.n_layers == 33 && c650.head_dim() == 64 && c650.arch == EsmModelArch::Esm2_650M);
  const EsmConfig c3b = EsmConfig::esm2_3b();
  CHECK(c3b.dim == 2560 && c3b.hidden_dim == 10240 && c3b.n_layers == 36 && c3b.n_heads == 40);
}

static void test_detect_from_file_errors(const std::string& dir) {
  bool not_found = false;
  try {
    EsmConfig::detect_from_file(dir + "/does_not_exist.bin");
  } catch (const IoError& e) {
    not_found = e.kind() == ErrorKind::NotFound;
  }
  CHECK(not_found);
  const std::string junk = dir + "/junk.bin";
  { std::ofstream(junk, std::ios::binary) << "not a weights file"; }
  bool invalid = false;
  try {
    EsmConfig::detect_from_file(junk);
  } catch (const IoError& e) {
    invalid = e.kind() == ErrorKind::InvalidData;
  }
  CHECK(invalid);
}

// ---- GPU -------------------------------------------------------------------------------------

template <class W>
static void run_forward(const std::string& path, const std::string& seq, bool contacts, size_t max_len,
                        const std::string& out) {
  const EsmConfig cfg = EsmConfig::detect_from_file(path);
  std::unique_ptr<W> w = W::from_file(path, cfg);
  if (contacts) {
    std::vector<float> head(cfg.n_layers * cfg.n_heads);
    for (size_t i = 0; i < head.size(); ++i) head[i] = (i % 3 == 0) ? 0.0f : 0.05f * std::sin(0.7f * i);
    w->set_contact_head(head, -0.5f);
  }
  BidirectionalRunState state(cfg, max_len);
  state.compute_contacts = contacts;
  const std::vector<size_t> tokens = Tokenizer::encode(seq);
  if constexpr (std::is_same<W, EsmWeights>::value) forward_bidirectional(tokens, cfg, *w, state);
  else if constexpr (std::is_same<W, EsmWeightsQ8>::value) forward_bidirectional_q8(tokens, cfg, *w, state, 8);
  else forward_bidirectional_q4(tokens, cfg, *w, state, 8);

  const int32_t L = static_cast<int32_t>(tokens.size()), V = static_cast<int32_t>(cfg.vocab_size);
  const int32_t n = contacts ? L - 2 : 0;
  for (int32_t i = 0; i < L * V; ++i) CHECK(!std::isnan(state.logits[i]));
  // test_bidirectional_logits_entropy (src/lib.rs:6958-6985): a masked position keeps a spread
  // distribution over the 20 canonical residues.
  for (int32_t p = 0; p < L; ++p) {
    if (tokens[p] != 32) continue;
    const std::vector<float> lp = log_softmax_canonical(&state.logits[static_cast<size_t>(p) * V]);
    float h = 0.0f;
    for (int i = 4; i <= 23; ++i) {
      const float pr = std::exp(lp[i]);
      if (pr > 1e-12f) h -= pr * lp[i];
    }
    CHECK(h > 0.1f);
  }
  // The _ext forms (FP32 and Q4_0 have one): the same outputs, and on_layer once per layer, in
  // order, with the residual stream after that layer.
  std::vector<float> layers;
  int32_t nl_out = 0;
  if constexpr (!std::is_same<W, EsmWeightsQ8>::value) {
    BidirectionalRunState st2(cfg, max_len);
    st2.compute_contacts = contacts;
    size_t next = 0;
    const OnLayer hook = [&](size_t l, const float* x, size_t count) {
      CHECK(l == next++ && count == tokens.size() * cfg.dim);
      layers.insert(layers.end(), x, x + count);
    };
    if constexpr (std::is_same<W, EsmWeights>::value) forward_bidirectional_parallel_ext(tokens, cfg, *w, st2, 8, hook);
    else forward_bidirectional_q4_ext(tokens, cfg, *w, st2, 8, hook);
    CHECK(next == cfg.n_layers);
    CHECK(std::equal(st2.logits.begin(), st2.logits.begin() + L * V, state.logits.begin()));
    CHECK(std::equal(st2.x.begin(), st2.x.begin() + static_cast<size_t>(L) * cfg.dim, state.x.begin()));
    nl_out = static_cast<int32_t>(cfg.n_layers);
  }
  std::ofstream f(out, std::ios::binary);
  f.write(reinterpret_cast<const char*>(&L), 4);
  f.write(reinterpret_cast<const char*>(&V), 4);
  f.write(reinterpret_cast<const char*>(&n), 4);
  f.write(reinterpret_cast<const char*>(state.logits.data()), static_cast<std::streamsize>(L) * V * 4);
  if (n > 0) f.write(reinterpret_cast<const char*>(state.contact_probs.data()), static_cast<std::streamsize>(n) * n * 4);
  f.write(reinterpret_cast<const char*>(&nl_out), 4);
  f.write(reinterpret_cast<const char*>(layers.data()), static_cast<std::streamsize>(layers.size() * 4));
}

static float cosine_canonical(const std::vector<float>& a, const std::vector<float>& b, size_t L, size_t V) {
  double dot = 0, na = 0, nb = 0;
  for (size_t p = 0; p < L; ++p)
    for (size_t i = 4; i <= 23; ++i) {
      const double x = a[p * V + i], y = b[p * V + i];
      dot += x * y;
      na += x * x;
      nb += y * y;
    }
  return static_cast<float>(dot / (std::sqrt(na) * std::sqrt(nb)));
}

// test_forward_q8_cosine_similarity_8m / test_forward_q4_cosine_similarity_8m
// (src/lib.rs:7273-7353): logits of the quantized models stay close to FP32's on the canonical
// residue columns (> 0.995 for Q8_0, > 0.850 for Q4_0).
static void run_cosine(const std::string& f32, const std::string& q8, const std::string& q4, const std::string& seq) {
  const EsmConfig cfg = EsmConfig::detect_from_file(f32);
  const std::vector<size_t> tokens = Tokenizer::encode(seq);
  BidirectionalRunState s32(cfg, tokens.size()), s8(cfg, tokens.size()), s4(cfg, tokens.size());
  s32.compute_contacts = s8.compute_contacts = s4.compute_contacts = false;
  {
    auto w = EsmWeights::from_file(f32, cfg);
    forward_bidirectional_parallel(tokens, cfg, *w, s32, 4);
  }
  {
    auto w = EsmWeightsQ8::from_file(q8, cfg);
    forward_bidirectional_q8(tokens, cfg, *w, s8, 4);
  }
  {
    auto w = EsmWeightsQ4::from_file(q4, cfg);
    forward_bidirectional_q4(tokens, cfg, *w, s4, 4);
  }
  const float c8 = cosine_canonical(s32.logits, s8.logits, tokens.size(), cfg.vocab_size);
  const float c4 = cosine_canonical(s32.logits, s4.logits, tokens.size(), cfg.vocab_size);
  std::printf("cosine fp32/q8 %.5f fp32/q4 %.5f\n", c8, c4);
  CHECK(c8 > 0.995f);
  CHECK(c4 > 0.850f);
}

// The reference panics on a sequence longer than the run state (assert!, src/lib.rs:5106) and
// returns io errors from its loaders; here the panic is std::logic_error and the weights stay
// usable after it.
static void run_misuse(const std::string& q4) {
  const EsmConfig cfg = EsmConfig::detect_from_file(q4);
  auto w = EsmWeightsQ4::from_file(q4, cfg);
  BidirectionalRunState small(cfg, 8);
  small.compute_contacts = false;
  bool panicked = false;
  try {
    forward_bidirectional_q4(Tokenizer::encode("MKTAYIAKQRQ"), cfg, *w, small, 1);
  } catch (const std::logic_error&) {
    panicked = true;
  }
  CHECK(panicked);
  forward_bidirectional_q4(Tokenizer::encode("MKTAY*"), cfg, *w, small, 1);
  for (size_t i = 0; i < 8 * cfg.vocab_size; ++i) CHECK(std::isfinite(small.logits[i]));

  bool not_found = false;
  try {
    EsmWeightsQ4::from_file(q4 + ".missing", cfg);
  } catch (const IoError& e) {
    not_found = e.kind() == ErrorKind::NotFound;
  }
  CHECK(not_found);
  // A Q4_0 file opened as Q8_0 weights is InvalidData.
  bool wrong_type = false;
  try {
    EsmWeightsQ8::from_file(q4, cfg);
  } catch (const IoError& e) {
    wrong_type = e.kind() == ErrorKind::InvalidData;
  }
  CHECK(wrong_type);
  // A truncated CODQ file is rejected.
  const std::string cut = q4 + ".cut";
  {
    std::ifstream in(q4, std::ios::binary);
    std::vector<char> buf(4096);
    in.read(buf.data(), static_cast<std::streamsize>(buf.size()));
    std::ofstream(cut, std::ios::binary).write(buf.data(), in.gcount());
  }
  bool truncated = false;
  try {
    EsmWeightsQ4::from_file(cut, cfg);
  } catch (const IoError&) {
    truncated = true;
  }
  CHECK(truncated);
}

// The pipelines on an FP32 file quantized to Q4_0 while loading (load_model_weights with
// QuantizationMode::Q4_0): both mutational-scan modes and the contacts pipeline. Their outputs go
// to `out` for the Python side to compare with the oracle; the row bookkeeping is checked here.
static void run_pipelines(const std::string& f32, const std::string& seq, const std::string& out) {
  LoadedWeights lw = load_model_weights(f32, QuantizationMode::Q4_0);
  CHECK(lw.mode == QuantizationMode::Q4_0);
  const EsmConfig& cfg = lw.config;
  DeviceWeights& w = *lw.weights;
  std::vector<float> head(cfg.n_layers * cfg.n_heads);
  for (size_t i = 0; i < head.size(); ++i) head[i] = (i % 3 == 0) ? 0.0f : 0.05f * std::sin(0.7f * i);
  w.set_contact_head(head, -0.5f);
  const FastaRecord rec{"test", "test protein", seq};
  const DmsPipelineResult mm = run_pipeline_dms_with_mode(rec, 0, 0, cfg, w, 8, DmsScoringMode::MaskedMarginal);
  const DmsPipelineResult wt = run_pipeline_dms_with_mode(rec, 16, 5, cfg, w, 8, DmsScoringMode::WildtypeMarginal);
  {
    // The convenience form is the masked-marginal mode.
    const DmsPipelineResult again = run_pipeline_dms_parallel(rec, 0, 0, cfg, w, 8);
    CHECK(again.rows.size() == mm.rows.size() && again.scoring_mode == DmsScoringMode::MaskedMarginal);
    for (size_t p = 0; p < again.rows.size() && p < mm.rows.size(); ++p) CHECK(again.rows[p].deltas == mm.rows[p].deltas);
  }
  const size_t n = seq.size();
  for (const DmsPipelineResult* r : {&mm, &wt}) {
    CHECK(r->rows.size() == n);
    size_t catalytic = 0;
    for (size_t p = 0; p < n; ++p) {
      const DmsPositionRow& row = r->rows[p];
      CHECK(row.pos == p + 1 && row.wt == seq[p]);
      float sum = 0.0f;
      for (float d : row.deltas) sum += (d != 0.0f) ? d : 0.0f;
      CHECK(row.mean_delta_logp == sum / 19.0f);
      catalytic += row.mean_delta_logp <= -3.8f;
    }
    CHECK(r->catalytic_sites_detected == catalytic);
    CHECK(r->muts_per_sec > 0.0);
  }
  const ContactsPipelineResult cp = compute_pipeline_contacts_parallel(rec, 6, 1.0f, std::nullopt, cfg, w, 8);
  CHECK(cp.sequence_length == n && cp.contact_probs.size() == n * n);
  for (const ContactPair& c : cp.top_contacts) CHECK(c.pos2 >= c.pos1 + 6 && c.res1 == seq[c.pos1]);
  // "<mask>" makes the byte count differ from the token count: refused, not misindexed.
  bool threw = false;
  try {
    compute_pipeline_contacts_parallel(FastaRecord{"m", "", "MKT<mask>AYIAKQRQ"}, 6, 1.0f, std::nullopt, cfg, w, 8);
  } catch (const std::exception&) {
    threw = true;
  }
  CHECK(threw);
  // Q3_LUT blocks through the C++ types: a block decodes to the reference's LUT values.
  std::vector<float> src(64);
  for (size_t i = 0; i < src.size(); ++i) src[i] = std::sin(0.37f * static_cast<float>(i));
  const std::vector<BlockQ3_LUT> q3 = quantize_slice_to_q3_lut(src);
  CHECK(q3.size() == 2);
  float dq[64];
  q3[0].dequantize_to(dq);
  q3[1].dequantize_to(dq + 32);
  for (int i = 0; i < 64; ++i) CHECK(std::isfinite(dq[i]) && (src[i] == 0.0f || (dq[i] < 0.0f) == (src[i] < 0.0f)));

  std::ofstream f(out, std::ios::binary);
  const int32_t hdr[2] = {static_cast<int32_t>(n), static_cast<int32_t>(cp.top_contacts.size())};
  f.write(reinterpret_cast<const char*>(hdr), 8);
  for (const DmsPipelineResult* r : {&mm, &wt}) {
    for (const DmsPositionRow& row : r->rows) f.write(reinterpret_cast<const char*>(row.deltas.data()), 80);
    for (const DmsPositionRow& row : r->rows) f.write(reinterpret_cast<const char*>(&row.entropy), 4);
  }
  for (const ContactPair& c : cp.top_contacts) {
    const int32_t ij[2] = {static_cast<int32_t>(c.pos1), static_cast<int32_t>(c.pos2)};
    f.write(reinterpret_cast<const char*>(ij), 8);
    f.write(reinterpret_cast<const char*>(&c.apc_score), 4);
  }
  f.write(reinterpret_cast<const char*>(&cp.cys_enrichment_ratio), 4);
  f.write(reinterpret_cast<const char*>(cp.contact_probs.data()), static_cast<std::streamsize>(n * n * 4));
  f.write(reinterpret_cast<const char*>(q3.data()), 28);
  f.write(reinterpret_cast<const char*>(dq), sizeof(dq));

}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const std::string cmd = argv[1];
  try {
    if (cmd == "cpu" && argc == 3) {
      test_q8_0_quantization_roundtrip();
      test_tokenizer_boundaries();
      test_mask_token_encoding_and_decoding();
      test_log_softmax_canonical();
      test_q4_0_roundtrip_quantize_dequantize_bound();
      test_q4_0_exact_nibble_packing();
      test_q4_0_zero_block();
      test_quantize_slice_rejects_ragged_length();
      test_config_presets();
      test_dms_row();
      test_detect_from_file_errors(argv[2]);
    } else if (cmd == "forward" && argc == 8) {
      const std::string kind = argv[3];
      const bool contacts = std::atoi(argv[6]) != 0;
      const size_t max_len = static_cast<size_t>(std::atol(argv[7]));
      if (kind == "fp32") run_forward<EsmWeights>(argv[2], argv[4], contacts, max_len, argv[5]);
      else if (kind == "q8") run_forward<EsmWeightsQ8>(argv[2], argv[4], contacts, max_len, argv[5]);
      else run_forward<EsmWeightsQ4>(argv[2], argv[4], contacts, max_len, argv[5]);
    } else if (cmd == "cosine" && argc == 6) {
      run_cosine(argv[2], argv[3], argv[4], argv[5]);
    } else if (cmd == "misuse" && argc == 3) {
      run_misuse(argv[2]);
    } else if (cmd == "pipelines" && argc == 5) {
      run_pipelines(argv[2], argv[3], argv[4]);
    } else {
      return 2;
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "uncaught exception: %s\n", e.what());
    return 1;
  }
  if (g_failures) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failures);
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
