"""GPU masked-marginal mutational scan (esm_dms_masked_marginal) against the oracle's restatement of
run_pipeline_dms_with_mode / DmsScoringMode::MaskedMarginal (codon-infer src/pipeline.rs:76-175):
one oracle forward per masked variant, log_softmax_canonical at the masked row, entropy, and the
20 CANONICAL_AAS deltas.

Tolerance: logits agree within 2e-2, so each log-probability within 2 * 2e-2 (logit plus
log-sum-exp) and each delta (a difference of two log-probabilities) within 8e-2; entropy within
5e-2.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _oracle_scan(orc, esm, cfg, dtype, t, residues, window_size):
    n = len(residues)
    max_len = 1024
    aw = min(n, max_len) if (n <= window_size or window_size == 0) else min(window_size, max_len)
    half = aw // 2
    deltas = np.zeros((n, 20), np.float32)
    ent = np.zeros(n, np.float32)
    for p in range(n):
        if p < half:
            ws = 0
        elif p + half > n:
            ws = max(n - aw, 0)
        else:
            ws = p - half
        we = min(ws + aw, n)
        toks = np.concatenate([[0], residues[ws:we], [2]]).astype(np.int32)
        pos = p - ws + 1
        wt = int(toks[pos])
        toks[pos] = 32
        lg = orc.forward(cfg, dtype, t, toks)["logits"][pos]
        lp = orc.log_softmax_canonical(lg)
        pa = np.exp(lp[4:24].astype(np.float64))
        ent[p] = -(pa * lp[4:24]).sum()
        for c, aa in enumerate(esm.CANONICAL_IDS):
            deltas[p, c] = 0.0 if aa == wt else lp[aa] - lp[wt]
    return deltas, ent


@pytest.mark.parametrize("window_size", [0, 16])
def test_dms_matches_oracle(esm, orc, window_size):
    cfg = esm.esm2_8m()
    t = esm.synth_fp32_tensors(cfg, seed=21, std=0.05, bias_std=0.02, ln_jitter=0.1)
    m = esm.Model(0)
    m.load_tensors(cfg, esm.DTYPE_FP32, t)
    n = 40
    residues = esm.random_sequences(1, n + 2, seed=22)[0][1:-1]
    # Room for only 16 variants per batch, so the scan runs in several batches.
    m.reserve(16 * (n + 2), 16, n + 2)
    got_d, got_e = m.dms_masked_marginal(residues, window_size)
    ref_d, ref_e = _oracle_scan(orc, esm, cfg, esm.DTYPE_FP32, t, residues, window_size)
    assert np.isfinite(got_d).all() and np.isfinite(got_e).all()
    assert np.abs(got_d - ref_d).max() <= 8e-2
    assert np.abs(got_e - ref_e).max() <= 5e-2
    wt_cols = [esm.CANONICAL_IDS.index(int(r)) for r in residues]
    assert (got_d[np.arange(n), wt_cols] == 0).all()
    m.close()


def test_dms_rejects_window_beyond_capacity(esm):
    cfg = esm.EsmConfig(320, 1280, 1, 20, arch=0)
    m = esm.Model(0)
    m.load_tensors(cfg, esm.DTYPE_FP32, esm.synth_fp32_tensors(cfg, seed=1))
    m.reserve(64, 2, 32)
    with pytest.raises(esm.EsmError) as e:
        m.dms_masked_marginal(np.full(40, 5, np.int32))
    assert e.value.code == esm.ESM_ECAPACITY
    m.close()


def _oracle_wt_scan(orc, esm, cfg, dtype, t, residues, window_size, stride):
    # run_pipeline_dms_with_mode / DmsScoringMode::WildtypeMarginal (src/pipeline.rs:176-291): one
    # forward per window, each position scored from the first window that covers it.
    n = len(residues)
    max_len = 1024
    aw = min(n, max_len) if (n <= window_size or window_size == 0) else min(window_size, max_len)
    wins = []
    if n <= aw:
        wins.append((0, n, 0))
    else:
        step = stride if 0 < stride <= aw else max(aw // 2, 1)
        covered, ws = 0, 0
        while covered < n:
            we = min(ws + aw, n)
            wins.append((ws, we, covered))
            covered = we
            if we >= n:
                break
            ws = min(ws + step, n - aw)
    deltas = np.zeros((n, 20), np.float32)
    ent = np.zeros(n, np.float32)
    for ws, we, first in wins:
        toks = np.concatenate([[0], residues[ws:we], [2]]).astype(np.int32)
        lg = orc.forward(cfg, dtype, t, toks)["logits"]
        for p in range(first, we):
            pos = p - ws + 1
            wt = int(toks[pos])
            lp = orc.log_softmax_canonical(lg[pos])
            pa = np.exp(lp[4:24].astype(np.float64))
            ent[p] = -(pa * lp[4:24]).sum()
            for c, aa in enumerate(esm.CANONICAL_IDS):
                deltas[p, c] = 0.0 if aa == wt else lp[aa] - lp[wt]
    return deltas, ent


@pytest.mark.parametrize("window_size,stride", [(0, 0), (16, 0), (16, 5), (16, 16)])
def test_wildtype_marginal_matches_oracle(esm, orc, window_size, stride):
    cfg = esm.esm2_8m()
    t = esm.synth_fp32_tensors(cfg, seed=23, std=0.05, bias_std=0.02, ln_jitter=0.1)
    m = esm.Model(0)
    m.load_tensors(cfg, esm.DTYPE_FP32, t)
    n = 45
    residues = esm.random_sequences(1, n + 2, seed=24)[0][1:-1]
    # Room for only two windows per batch, so the windowed scans run in several batches.
    m.reserve(2 * (n + 2), 2, n + 2)
    got_d, got_e = m.dms_wildtype_marginal(residues, window_size, stride)
    ref_d, ref_e = _oracle_wt_scan(orc, esm, cfg, esm.DTYPE_FP32, t, residues, window_size, stride)
    assert np.isfinite(got_d).all() and np.isfinite(got_e).all()
    assert np.abs(got_d - ref_d).max() <= 8e-2
    assert np.abs(got_e - ref_e).max() <= 5e-2
    wt_cols = [esm.CANONICAL_IDS.index(int(r)) for r in residues]
    assert (got_d[np.arange(n), wt_cols] == 0).all()
    m.close()
