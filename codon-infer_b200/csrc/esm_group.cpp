// Several GPUs driven from one host process: one esm_ctx per device, a batch split into
// contiguous cost-balanced blocks of sequences (a scan into contiguous blocks of positions), one
// host thread per device. Every device writes its rows straight into the caller's host output
// arrays, so the gather of the results is each device's own device-to-host copy and nothing else
// crosses between GPUs. Each sequence's outputs do not depend on which other sequences share its
// batch, so a group's results are the single-context results bit for bit.
//
// The reference runs its sequences and masked variants one forward at a time on the host
// (src/pipeline.rs:111-174 for the scan); this is the same work spread over the box's GPUs.
#include <algorithm>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/esm_b200.h"

struct esm_group {
  std::vector<int32_t> devices;
  std::vector<esm_ctx*> ctx;
  std::mutex mu;
  std::string err;
  int32_t cap_tokens = 0, cap_seqs = 0, cap_len = 0;
  bool cap_contacts = false;
  bool loaded = false;
  esm_config cfg{};
};

namespace {

int gfail(esm_group* g, int code, const std::string& msg) {
  if (g) g->err = msg;
  return code;
}

// Runs fn(i) for every member on its own host thread; returns the first failure, its message
// prefixed with the device.
template <typename Fn>
int run_all(esm_group* g, Fn fn) {
  const size_t n = g->ctx.size();
  std::vector<int> rc(n, ESM_OK);
  std::vector<std::thread> th;
  th.reserve(n);
  for (size_t i = 0; i < n; ++i) th.emplace_back([&, i] { rc[i] = fn(static_cast<int>(i)); });
  for (auto& t : th) t.join();
  for (size_t i = 0; i < n; ++i)
    if (rc[i] != ESM_OK) {
      const char* m = esm_last_error(g->ctx[i]);
      return gfail(g, rc[i], "device " + std::to_string(g->devices[i]) + ": " + (m ? m : ""));
    }
  return ESM_OK;
}

double seq_cost(int32_t L, int32_t d, int32_t F) {
  const double l = L;
  return 2.0 * l * (4.0 * d * d + 2.0 * d * F) + 4.0 * l * l * d;
}

}  // namespace

extern "C" {

int esm_partition(const int32_t* lengths, int32_t B, int32_t dim, int32_t hidden_dim, int32_t parts,
                  int32_t* bounds) {
  if (!lengths || !bounds || B < 0 || parts <= 0 || dim <= 0 || hidden_dim <= 0) return ESM_EINVAL;
  std::vector<double> csum(static_cast<size_t>(B) + 1, 0.0);
  for (int32_t i = 0; i < B; ++i) {
    if (lengths[i] < 0) return ESM_EINVAL;
    csum[i + 1] = csum[i] + seq_cost(lengths[i], dim, hidden_dim);
  }
  const double total = csum[B];
  bounds[0] = 0;
  for (int32_t r = 1; r < parts; ++r) {
    const double target = total * r / parts;
    // The first prefix that reaches the target, never before the previous bound.
    int32_t idx = static_cast<int32_t>(std::lower_bound(csum.begin(), csum.end(), target) - csum.begin());
    idx = std::min(std::max(idx, bounds[r - 1]), B);
    bounds[r] = idx;
  }
  bounds[parts] = B;
  return ESM_OK;
}

int esm_group_create(const int32_t* devices, int32_t n_devices, esm_group** out) {
  if (!devices || n_devices <= 0 || !out) return ESM_EINVAL;
  *out = nullptr;
  auto* g = new esm_group();
  for (int32_t i = 0; i < n_devices; ++i) {
    esm_ctx* c = nullptr;
    const int rc = esm_ctx_create(devices[i], &c);
    if (rc != ESM_OK) {
      for (esm_ctx* x : g->ctx) esm_ctx_destroy(x);
      delete g;
      return rc;
    }
    g->devices.push_back(devices[i]);
    g->ctx.push_back(c);
  }
  *out = g;
  return ESM_OK;
}

int esm_group_destroy(esm_group* g) {
  if (!g) return ESM_EINVAL;
  for (esm_ctx* c : g->ctx) esm_ctx_destroy(c);
  delete g;
  return ESM_OK;
}

const char* esm_group_last_error(const esm_group* g) { return g ? g->err.c_str() : "null group"; }

int esm_group_size(const esm_group* g, int32_t* n) {
  if (!g || !n) return ESM_EINVAL;
  *n = static_cast<int32_t>(g->ctx.size());
  return ESM_OK;
}

int esm_group_ctx(esm_group* g, int32_t i, esm_ctx** out) {
  if (!g || !out || i < 0 || i >= static_cast<int32_t>(g->ctx.size())) return ESM_EINVAL;
  *out = g->ctx[i];
  return ESM_OK;
}

int esm_group_load_host(esm_group* g, const esm_config* cfg, int32_t dtype, const void* const* tensors,
                        const size_t* sizes) {
  if (!g) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(g->mu);
  g->loaded = false;
  int rc = run_all(g, [&](int i) { return esm_load_host(g->ctx[i], cfg, dtype, tensors, sizes); });
  if (rc != ESM_OK) return rc;
  int32_t dt = 0;
  esm_get_config(g->ctx[0], &g->cfg, &dt);
  g->loaded = true;
  return ESM_OK;
}

int esm_group_load_file(esm_group* g, const char* path, const esm_config* cfg) {
  if (!g) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(g->mu);
  g->loaded = false;
  int rc = run_all(g, [&](int i) { return esm_load_file(g->ctx[i], path, cfg); });
  if (rc != ESM_OK) return rc;
  int32_t dt = 0;
  esm_get_config(g->ctx[0], &g->cfg, &dt);
  g->loaded = true;
  return ESM_OK;
}

int esm_group_set_contact_head(esm_group* g, const float* w, int32_t nw, float b) {
  if (!g) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(g->mu);
  return run_all(g, [&](int i) { return esm_set_contact_head(g->ctx[i], w, nw, b); });
}

int esm_group_reserve(esm_group* g, int32_t max_tokens, int32_t max_seqs, int32_t max_len, int32_t contacts) {
  if (!g) return ESM_EINVAL;
  std::lock_guard<std::mutex> lk(g->mu);
  int rc = run_all(g, [&](int i) { return esm_reserve(g->ctx[i], max_tokens, max_seqs, max_len, contacts); });
  if (rc != ESM_OK) return rc;
  g->cap_tokens = max_tokens;
  g->cap_seqs = max_seqs;
  g->cap_len = max_len;
  g->cap_contacts = contacts != 0;
  return ESM_OK;
}

int esm_group_forward(esm_group* g, const int32_t* tokens, const int32_t* lengths, int32_t B, int32_t Lmax,
                      float* logits, float* hidden, float* contacts) {
  if (!g || !tokens || !lengths || !logits) return gfail(g, ESM_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(g->mu);
  if (!g->loaded) return gfail(g, ESM_EINVAL, "no weights loaded");
  if (g->cap_tokens == 0) return gfail(g, ESM_EINVAL, "call esm_group_reserve before the first forward");
  if (B <= 0 || Lmax <= 0) return gfail(g, ESM_EINVAL, "empty batch");
  for (int32_t b = 0; b < B; ++b) {
    if (lengths[b] <= 0 || lengths[b] > Lmax) return gfail(g, ESM_EINVAL, "length outside [1, Lmax]");
    if (lengths[b] > g->cap_len || lengths[b] > g->cap_tokens)
      return gfail(g, ESM_ECAPACITY, "sequence of " + std::to_string(lengths[b]) + " tokens exceeds the reserved max_len");
  }
  if (contacts && !g->cap_contacts) return gfail(g, ESM_ECAPACITY, "contacts were not reserved");
  const int32_t n_dev = static_cast<int32_t>(g->ctx.size());
  std::vector<int32_t> bounds(n_dev + 1);
  esm_partition(lengths, B, g->cfg.dim, g->cfg.hidden_dim, n_dev, bounds.data());
  const size_t V = g->cfg.vocab_size, d = g->cfg.dim;
  const size_t np = Lmax > 2 ? static_cast<size_t>(Lmax - 2) : 0;
  return run_all(g, [&](int i) {
    // This device's block, in chunks that fit its workspace.
    int32_t b = bounds[i];
    while (b < bounds[i + 1]) {
      int32_t e = b, tok = 0;
      while (e < bounds[i + 1] && e - b < g->cap_seqs && tok + lengths[e] <= g->cap_tokens) tok += lengths[e++];
      if (e == b) return static_cast<int>(ESM_ECAPACITY);  // not reached: lengths were checked above
      const size_t row = static_cast<size_t>(b) * Lmax;
      const int rc = esm_forward(g->ctx[i], tokens + row, lengths + b, e - b, Lmax, logits + row * V,
                                 hidden ? hidden + row * d : nullptr, contacts ? contacts + b * np * np : nullptr);
      if (rc != ESM_OK) return rc;
      b = e;
    }
    return static_cast<int>(ESM_OK);
  });
}

int esm_group_dms_masked_marginal(esm_group* g, const int32_t* residues, int32_t n, int32_t window_size,
                                  float* deltas, float* entropy) {
  if (!g || !residues || !deltas || !entropy) return gfail(g, ESM_EINVAL, "null argument");
  if (n <= 0) return gfail(g, ESM_EINVAL, "Sequence cannot be empty");
  std::lock_guard<std::mutex> lk(g->mu);
  const int32_t n_dev = static_cast<int32_t>(g->ctx.size());
  // Every variant is one window of the same length, so equal blocks of positions balance the cost.
  return run_all(g, [&](int i) {
    const int32_t pb = static_cast<int32_t>(static_cast<int64_t>(n) * i / n_dev);
    const int32_t pe = static_cast<int32_t>(static_cast<int64_t>(n) * (i + 1) / n_dev);
    if (pb == pe) return static_cast<int>(ESM_OK);
    return esm_dms_masked_marginal_range(g->ctx[i], residues, n, window_size, pb, pe,
                                         deltas + static_cast<size_t>(pb) * 20, entropy + pb);
  });
}

}  // extern "C"
