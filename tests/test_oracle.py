"""Pins the CPU oracle before it is trusted as the parity checker.

1. The reference's own known-answer tests for this path (codon-infer src/lib.rs tests), restated.
2. Golden vectors from an independent implementation (HF transformers EsmForMaskedLM) on the
   reference's bundled real ESM-2 8M weights (tests/golden/esm2_8m_hf.npz, made by
   tests/golden/make_golden.py); the reference documents cos >= 0.999999 against HF for FP32.
"""
import numpy as np
import pytest
from types import SimpleNamespace

from conftest import REF_WEIGHTS_8M, ROOT

CFG_8M = SimpleNamespace(dim=320, hidden_dim=1280, n_layers=6, n_heads=20, vocab_size=33)


# ---- quantizer known answers ------------------------------------------------------------------

def test_q4_exact_nibble_packing(orc):
    # test_q4_0_exact_nibble_packing, src/lib.rs:7490-7517
    src = np.zeros(32, dtype=np.float32)
    for j in range(16):
        src[j] = 8 - j
        src[j + 16] = j - 7
    blk = orc.quantize_q4(src)
    d = blk[:4].view(np.float32)[0]
    assert d == -1.0
    expect = np.array([j | ((15 - j) << 4) for j in range(16)], dtype=np.uint8)
    np.testing.assert_array_equal(blk[4:20], expect)
    np.testing.assert_array_equal(orc.dequantize_q4(blk), src)


def test_q4_zero_block(orc):
    # test_q4_0_zero_block, src/lib.rs:7520-7531
    blk = orc.quantize_q4(np.zeros(32, dtype=np.float32))
    assert blk[:4].view(np.float32)[0] == 0.0
    assert (blk[4:] == 0x88).all()
    assert (orc.dequantize_q4(blk) == 0.0).all()


def _q4_roundtrip_vectors():
    # test_q4_0_roundtrip_quantize_dequantize_bound, src/lib.rs:7440-7487
    vecs = [np.array([-8.0 + i * (15.0 / 31.0) for i in range(32)], dtype=np.float32)]
    for scale in (0.05, 1.0, 2.5, 10.0):
        v = np.zeros(32, dtype=np.float32)
        v[0] = -8.0 * scale
        for i in range(1, 32):
            v[i] = np.float32((i % 16) - 8) * np.float32(scale) + \
                np.float32((((i * 11) % 9) - 4.0) / 10.0 * 0.45 * scale)
        vecs.append(v)
    for scale in (0.05, 1.0, 2.5, 10.0):
        v = np.zeros(32, dtype=np.float32)
        v[0] = 8.0 * scale
        for i in range(1, 32):
            v[i] = np.float32((i % 16) - 8) * np.float32(-scale) + \
                np.float32((((i * 7) % 9) - 4.0) / 10.0 * 0.45 * scale)
        vecs.append(v)
    return vecs


def test_q4_roundtrip_bound(orc):
    for src in _q4_roundtrip_vectors():
        blk = orc.quantize_q4(src)
        d = abs(float(blk[:4].view(np.float32)[0]))
        err = np.abs(orc.dequantize_q4(blk) - src)
        assert (err <= d / 2 + 1e-5).all()


def test_q8_roundtrip_mse(orc):
    # test_q8_0_quantization_roundtrip, src/lib.rs:6834-6849
    src = np.array([(i / 31.0) * 2.0 - 1.0 for i in range(32)], dtype=np.float32)
    mse = float(np.mean((orc.dequantize_q8(orc.quantize_q8(src)) - src) ** 2))
    assert mse < 0.02


# ---- kernels ----------------------------------------------------------------------------------

def test_tiled_gemm_matches_gemv(orc):
    # test_tiled_gemm_and_contact_head_v1_7_0, src/lib.rs:8473-8515: tiled GEMM vs per-token GEMV
    # at seq_len 7 and 12, (320 -> 64); FP32 within 1e-4, Q8/Q4 within 1e-3.
    in_dim, out_dim = 320, 64
    for seq_len in (7, 12):
        x = np.sin(np.arange(seq_len * in_dim, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
        w = (np.cos(np.arange(out_dim * in_dim, dtype=np.float32) * np.float32(0.007)) * 0.5).astype(np.float32)
        b = (np.arange(out_dim, dtype=np.float32) * np.float32(0.01) - np.float32(0.2)).astype(np.float32)
        X = x.reshape(seq_len, in_dim).astype(np.float64)
        for dt, wq, deq, tol in ((0, w, lambda a: a, 1e-4),
                                 (1, orc.quantize_q8(w), orc.dequantize_q8, 1e-3),
                                 (2, orc.quantize_q4(w), orc.dequantize_q4, 1e-3)):
            got = orc.tiled_gemm(dt, x, wq, b, in_dim, out_dim, n_threads=2)
            gemv = X @ deq(wq).reshape(out_dim, in_dim).astype(np.float64).T + b
            assert np.abs(got - gemv).max() < tol


def test_tiled_gemm_thread_count_invariant(orc):
    # test_q4_thread_determinism (bit-identical for 1/2/4/8 threads), src/lib.rs:7803-7828
    rng = np.random.default_rng(3)
    x = rng.standard_normal(9 * 1280, dtype=np.float32)
    w = orc.quantize_q4(rng.standard_normal(320 * 1280, dtype=np.float32) * 0.02)
    b = rng.standard_normal(320, dtype=np.float32)
    ref = orc.tiled_gemm(2, x, w, b, 1280, 320, n_threads=1)
    for t in (2, 4, 8):
        assert np.array_equal(ref, orc.tiled_gemm(2, x, w, b, 1280, 320, n_threads=t))


def test_softmax_and_log_softmax(orc):
    # test_softmax_sum_to_one (src/lib.rs:6868-6870), test_log_softmax_canonical (6928-6936)
    assert abs(orc.softmax([1.0, 2.0, 3.0]).sum() - 1.0) < 1e-6
    lp = orc.log_softmax_canonical(np.ones(33, dtype=np.float32))
    assert abs(np.exp(lp[4:24]).sum() - 1.0) < 1e-5
    assert np.isneginf(lp[:4]).all() and np.isneginf(lp[24:]).all()


def test_layer_norm_stability(orc):
    # test_layer_norm_stability, src/lib.rs:6865-6867
    out = orc.layer_norm([1.0, 2.0, 3.0, 4.0], np.ones(4), np.zeros(4))
    assert np.isfinite(out).all()


def test_gelu_matches_exact_erf(orc):
    import math
    for x in np.linspace(-6, 6, 97):
        exact = 0.5 * x * (1 + math.erf(x / math.sqrt(2)))
        assert abs(orc.gelu(x) - exact) < 2e-6 * max(1.0, abs(x))


def test_apc_row_sum_beyond_1024(orc):
    # The reference's accumulate_head_apc has a fixed [f32; 1024] row-sum buffer; the oracle's is
    # dynamic. On a symmetric, row-stochastic map APC is the identity minus a uniform term.
    L = 1100
    n = L - 2
    att = np.full((L, L), 1.0 / L, dtype=np.float32)
    acc = np.zeros((n, n), dtype=np.float32)
    orc.accumulate_head_apc(att, acc, L, n, 1.0)
    np.testing.assert_allclose(acc, 0.0, atol=1e-6)


# ---- independent golden vectors ---------------------------------------------------------------

def _read_grouped_8m():
    import make_golden
    return make_golden.read_grouped(REF_WEIGHTS_8M)


@pytest.mark.skipif(not REF_WEIGHTS_8M.exists(), reason="reference 8M weights not mounted")
@pytest.mark.parametrize("name", ["peptidase", "masked", "chl"])
def test_oracle_matches_hf_on_real_8m(orc, name):
    g = np.load(ROOT / "tests" / "golden" / "esm2_8m_hf.npz")
    t = _read_grouped_8m()
    out = orc.forward(CFG_8M, 0, t, g[f"{name}_tokens"], contact_w=g["contact_w"], contact_b=float(g["contact_b"]),
                      want_hidden=True)
    lg, ref = out["logits"].astype(np.float64), g[f"{name}_logits"].astype(np.float64)
    cos = (lg * ref).sum() / np.linalg.norm(lg) / np.linalg.norm(ref)
    assert cos >= 0.999999
    assert np.abs(lg - ref).max() < 1e-3
    assert (lg.argmax(1) == ref.argmax(1)).all()
    assert np.abs(out["hidden"] - g[f"{name}_hidden"]).max() < 1e-4
    assert np.abs(out["contacts"] - g[f"{name}_contacts"]).max() < 1e-4


@pytest.mark.skipif(not REF_WEIGHTS_8M.exists(), reason="reference 8M weights not mounted")
def test_masked_logit_entropy_on_real_8m(orc):
    # test_bidirectional_logits_entropy, src/lib.rs:6958-6983: "MCMP*TTD", mask row 5, H > 0.1
    g = np.load(ROOT / "tests" / "golden" / "esm2_8m_hf.npz")
    toks = g["masked_tokens"]
    assert list(toks) == [0, 20, 23, 20, 14, 32, 11, 11, 13, 2]
    out = orc.forward(CFG_8M, 0, _read_grouped_8m(), toks)
    lp = orc.log_softmax_canonical(out["logits"][5])
    p = np.exp(lp[4:24])
    assert -(p * lp[4:24]).sum() > 0.1


def test_quantized_forward_thread_invariant(orc, esm):
    cfg = esm.EsmConfig(dim=64, hidden_dim=256, n_layers=2, n_heads=4)
    t = esm.quantize_tensors(esm.synth_fp32_tensors(cfg, seed=5, bias_std=0.02, ln_jitter=0.1), esm.DTYPE_Q4_0)
    toks = esm.random_sequences(1, 40, seed=1)[0]
    a = orc.forward(cfg, 2, t, toks, n_threads=1)["logits"]
    b = orc.forward(cfg, 2, t, toks, n_threads=8)["logits"]
    assert np.array_equal(a, b)
