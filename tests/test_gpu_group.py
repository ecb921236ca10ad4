"""Several GPUs from one host process (esm_group_*): the batch split into cost-balanced contiguous
blocks, one context and host thread per device, rows written straight into the caller's arrays.
Every sequence's outputs are independent of its batch, so the group must return exactly what one
context returns. Runs on two GPUs when the machine has them, else on two contexts of GPU 0 (the
same host logic; the contexts' kernels never wait on one another)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _devices():
    import torch
    return [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]


def _model(esm, cfg, dtype, t, cw):
    m = esm.Model(0)
    m.load_tensors(cfg, dtype, t)
    m.set_contact_head(cw, -0.2)
    return m


def test_group_forward_equals_one_context(esm):
    base = esm.esm2_650m()
    cfg = esm.EsmConfig(base.dim, base.hidden_dim, 2, base.n_heads, arch=base.arch)
    t = esm.quantize_tensors(esm.synth_fp32_tensors(cfg, seed=31, bias_std=0.02, ln_jitter=0.1), esm.DTYPE_Q4_0)
    cw = (np.random.default_rng(32).standard_normal(cfg.n_layers * cfg.n_heads) * 0.1).astype(np.float32)
    lens = [300, 41, 129, 257, 3, 64, 511, 90, 200]
    seqs = esm.random_sequences(len(lens), lens, seed=33)
    one = _model(esm, cfg, esm.DTYPE_Q4_0, t, cw)
    one.reserve(sum(lens), len(lens), max(lens), contacts=True)
    ref = one.forward(seqs, want_hidden=True, want_contacts=True)
    one.close()
    g = esm.Group(_devices())
    g.load_tensors(cfg, esm.DTYPE_Q4_0, t)
    g.set_contact_head(cw, -0.2)
    # Per-device room for fewer tokens than a block holds: each device runs its block in chunks.
    g.reserve(700, 3, 511, contacts=True)
    out = g.forward(seqs, want_hidden=True, want_contacts=True)
    np.testing.assert_array_equal(out["logits"], ref["logits"])
    np.testing.assert_array_equal(out["hidden"], ref["hidden"])
    # APC row sums are accumulated with float atomics: maps agree to rounding.
    np.testing.assert_allclose(out["contacts"], ref["contacts"], rtol=0, atol=1e-6)
    # A sequence longer than the per-device max_len is refused, and the group stays usable.
    with pytest.raises(esm.EsmError) as e:
        g.forward(esm.random_sequences(1, 600, seed=34))
    assert e.value.code == esm.ESM_ECAPACITY
    np.testing.assert_array_equal(g.forward(seqs[:2])["logits"], ref["logits"][:2, :300])
    g.close()


def test_group_scan_equals_one_context(esm):
    cfg = esm.esm2_8m()
    t = esm.synth_fp32_tensors(cfg, seed=35, std=0.05, bias_std=0.02, ln_jitter=0.1)
    residues = esm.random_sequences(1, 62, seed=36)[0][1:-1]
    one = esm.Model(0)
    one.load_tensors(cfg, esm.DTYPE_FP32, t)
    one.reserve(8 * 62, 8, 62)
    d1, e1 = one.dms_masked_marginal(residues)
    # The range form returns the same rows as the whole scan.
    d2, e2 = one.dms_masked_marginal_range(residues, 17, 45)
    np.testing.assert_array_equal(d2, d1[17:45])
    np.testing.assert_array_equal(e2, e1[17:45])
    with pytest.raises(esm.EsmError) as e:
        one.dms_masked_marginal_range(residues, 30, 30)
    assert e.value.code == esm.ESM_EINVAL
    one.close()
    g = esm.Group(_devices())
    g.load_tensors(cfg, esm.DTYPE_FP32, t)
    g.reserve(5 * 62, 5, 62)
    dg, eg = g.dms_masked_marginal(residues)
    np.testing.assert_array_equal(dg, d1)
    np.testing.assert_array_equal(eg, e1)
    g.close()
