"""Contact-pair ranking on the device (esm_contact_top_pairs) against a restatement of
compute_pipeline_contacts_parallel's ranking (src/pipeline.rs:454-503): candidates (i, j) with
j >= i + min_separation in row-major order, a stable sort on descending probability, the first k
(max_k, else round(n * top_l_factor) clamped to [5, 50]), and the Cys enrichment in f32. Pairs and
scores must match exactly, ties included."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

AAS = "ACDEFGHIKLMNPQRSTVWY"


def reference_ranking(m, seq, min_sep, max_k, factor):
    n = m.shape[0]
    ii, jj = np.triu_indices(n, k=min_sep)          # row-major (i, then j)
    s = m[ii, jj]
    order = np.argsort(-s, kind="stable")
    total = ii.size
    if max_k is not None:
        k = min(max_k, total)
    else:
        x = np.float32(n) * np.float32(factor)
        r = np.sign(x) * np.floor(np.abs(x) + np.float32(0.5))  # Rust f32::round: half away from zero
        k = min(min(max(int(r) if r > 0 else 0, 5), 50), total)
    top = order[:k]
    is_c = np.array([ch == "C" for ch in seq])
    cc_all = int(np.sum(is_c[ii] & is_c[jj]))
    cc_top = int(np.sum(is_c[ii[top]] & is_c[jj[top]]))
    top_d = np.float32(cc_top) / np.float32(k) if k else np.float32(0.0)
    bg_d = np.float32(cc_all) / np.float32(total) if total else np.float32(0.05)
    enr = top_d / bg_d if bg_d > 0 else np.float32(1.0)
    return ii[top], jj[top], s[top], np.float32(enr)


@pytest.mark.parametrize("n,min_sep,max_k,factor,levels", [
    (4, 6, None, 1.0, 16),      # no candidates
    (50, 6, None, 1.0, 16),     # k = 50 by the clamp
    (91, 6, None, 0.25, 8),     # k = round(22.75) = 23
    (300, 6, 7, 1.0, 4),        # heavy ties
    (300, 24, 4096, 1.0, 1000), # k = 4096
    (1200, 6, None, 1.0, 0),    # continuous values, three selection rounds
])
def test_ranking_matches_reference(esm, n, min_sep, max_k, factor, levels):
    import torch

    rng = np.random.default_rng(n + min_sep)
    m = rng.random((n, n), dtype=np.float32)
    if levels:
        m = np.floor(m * levels).astype(np.float32) / np.float32(levels)
    m[0, 7 % n] = -0.0  # -0 ties +0 in the reference's comparison
    seq = "".join(rng.choice(list(AAS + "CCCC"), n))
    d = torch.from_numpy(m).cuda()
    mdl = esm.Model(0)
    got = mdl.contact_top_pairs(d.data_ptr(), n, seq, min_sep, max_k, factor)
    mdl.close()
    p1, p2, sc, enr = reference_ranking(m, seq, min_sep, max_k, factor)
    np.testing.assert_array_equal(got["pos1"], p1)
    np.testing.assert_array_equal(got["pos2"], p2)
    np.testing.assert_array_equal(got["score"], sc)
    assert np.float32(got["cys_enrichment"]) == enr


def test_ranking_of_a_forward_contact_map(esm):
    # The map of a real forward (8M shape with its contact head), ranked without leaving the GPU.
    import torch

    cfg = esm.esm2_8m()
    t32 = esm.synth_fp32_tensors(cfg, seed=3)
    m = esm.Model(0)
    m.load_tensors(cfg, esm.DTYPE_FP32, t32)
    rng = np.random.default_rng(4)
    m.set_contact_head((rng.standard_normal(cfg.n_layers * cfg.n_heads) * 0.1).astype(np.float32), -0.5)
    seq = "".join(rng.choice(list(AAS + "CC"), 180))
    toks = esm.tokenize(seq)
    L, n = len(toks), len(seq)
    m.reserve(L, 1, L, contacts=True)
    d_tok = torch.from_numpy(toks.astype(np.int32)).cuda()
    d_logits = torch.empty(L, cfg.vocab_size, dtype=torch.float32, device="cuda")
    d_con = torch.empty(n * n, dtype=torch.float32, device="cuda")
    m.forward_device(d_tok, np.array([0, L], dtype=np.int32), d_logits, d_contacts=d_con, sync=True)
    got = m.contact_top_pairs(d_con.data_ptr(), n, seq, 6, None, 1.0)
    p1, p2, sc, enr = reference_ranking(d_con.cpu().numpy().reshape(n, n), seq, 6, None, 1.0)
    m.close()
    np.testing.assert_array_equal(got["pos1"], p1)
    np.testing.assert_array_equal(got["pos2"], p2)
    np.testing.assert_array_equal(got["score"], sc)
    assert np.float32(got["cys_enrichment"]) == enr


def test_contacts_pipeline_one_call(esm):
    # esm_contacts_pipeline (tokenize, forward with contacts, ranking) gives what the separate calls
    # give on the same map, and refuses a sequence whose bytes are not one token each.
    cfg = esm.esm2_8m()
    m = esm.Model(0)
    m.load_tensors(cfg, esm.DTYPE_FP32, esm.synth_fp32_tensors(cfg, seed=5))
    rng = np.random.default_rng(6)
    m.set_contact_head((rng.standard_normal(cfg.n_layers * cfg.n_heads) * 0.1).astype(np.float32), -0.5)
    seq = "".join(rng.choice(list(AAS + "CC"), 150))
    n = len(seq)
    m.reserve(n + 2, 1, n + 2, contacts=True)
    one = m.contacts_pipeline(seq, 6, None, 1.0, want_map=True, want_logits=True)
    fwd = m.forward([esm.tokenize(seq)], want_contacts=True)
    # Logits are bitwise reproducible; contact maps to float rounding (the APC row sums are
    # accumulated across tiles with float atomics, in an order that varies between runs).
    np.testing.assert_array_equal(one["logits"], fwd["logits"][0])
    assert np.abs(one["contact_probs"] - fwd["contacts"][0]).max() <= 1e-6
    p1, p2, sc, enr = reference_ranking(one["contact_probs"], seq, 6, None, 1.0)
    np.testing.assert_array_equal(one["pos1"], p1)
    np.testing.assert_array_equal(one["pos2"], p2)
    np.testing.assert_array_equal(one["score"], sc)
    assert np.float32(one["cys_enrichment"]) == enr
    with pytest.raises(esm.EsmError) as e:
        m.contacts_pipeline("MKT<mask>AYIAKQRQISFVK")
    assert e.value.code == esm.ESM_EINVAL
    m.close()
