"""Host-side checks of the product library (no GPU): C-ABI exports, bit-exact quantizers,
tokenizer, presets, file-format detection and the error contract."""
import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_functions():
    text = (ROOT / "include" / "esm_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(esm_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol(esm):
    names = _declared_functions()
    assert len(names) >= 15
    L = esm.lib()
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/esm_b200.h but not exported"


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_quantizers_bit_exact_with_oracle(esm, orc, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(32 * 4096) * rng.choice([1e-3, 0.02, 1.0, 50.0], 32 * 4096)).astype(np.float32)
    # Edge cases: all-zero block, ties at .5 of the step, negative and positive extremes.
    x[:32] = 0.0
    x[32:64] = np.arange(32, dtype=np.float32) - 16.0
    x[64:96] = np.linspace(-8.0, 8.0, 32, dtype=np.float32)
    x[96:128] = -np.arange(32, dtype=np.float32) * 0.5
    assert np.array_equal(esm.quantize_q8(x), orc.quantize_q8(x))
    assert np.array_equal(esm.quantize_q4(x), orc.quantize_q4(x))


def test_quantizer_known_answers(esm):
    src = np.zeros(32, dtype=np.float32)
    for j in range(16):
        src[j] = 8 - j
        src[j + 16] = j - 7
    blk = esm.quantize_q4(src)
    assert blk[:4].view(np.float32)[0] == -1.0
    assert list(blk[4:]) == [j | ((15 - j) << 4) for j in range(16)]
    z = esm.quantize_q4(np.zeros(32, dtype=np.float32))
    assert (z[4:] == 0x88).all() and z[:4].view(np.float32)[0] == 0.0


def test_quantizer_rejects_ragged_length(esm):
    with pytest.raises(esm.EsmError):
        esm.quantize_q8(np.zeros(33, dtype=np.float32))


def test_tokenizer(esm):
    # test_tokenizer_boundaries (src/lib.rs:6871), test_mask_token_encoding_and_decoding (6921-6925)
    assert list(esm.tokenize("LA")) == [0, 4, 5, 2]
    assert list(esm.tokenize("M*C")) == [0, 20, 32, 23, 2]
    assert list(esm.tokenize("M<mask_1>C")) == [0, 20, 32, 23, 2]
    assert list(esm.tokenize("M<mask>C")) == [0, 20, 32, 23, 2]
    assert list(esm.tokenize("")) == [0, 2]
    assert list(esm.tokenize("J1é")) == [0, 3, 3, 3, 2]
    assert list(esm.tokenize("XBUZO.-")) == [0, 24, 25, 26, 27, 28, 29, 30, 2]


def test_presets(esm):
    # EsmConfig::esm2_8m .. esm2_3b, src/lib.rs:87-150
    exp = [(320, 1280, 6, 20), (480, 1920, 12, 20), (640, 2560, 30, 20), (1280, 5120, 33, 20), (2560, 10240, 36, 40)]
    for arch, (d, F, nl, H) in enumerate(exp):
        c = esm.EsmConfig.preset(arch)
        assert (c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.vocab_size, c.max_seq_len) == (d, F, nl, H, 33, 1024)


def test_grouped_size_autodetect(esm, tmp_path):
    # detect_from_file_len exact sizes (src/lib.rs:228-236); a sparse file of the 8M grouped size.
    p = tmp_path / "w.bin"
    with open(p, "wb") as f:
        f.truncate(30_091_652)
    cfg, dt = esm.detect_file(str(p))
    assert (cfg.dim, cfg.n_layers, dt) == (320, 6, esm.DTYPE_FP32)


def test_codq_header_detect_and_corruption(esm, tmp_path):
    cfg = esm.esm2_8m()
    t = esm.quantize_tensors(esm.synth_fp32_tensors(cfg, seed=0), esm.DTYPE_Q4_0)
    p = tmp_path / "m.q4"
    esm.write_codq(str(p), cfg, esm.DTYPE_Q4_0, t)
    got, dt = esm.detect_file(str(p))
    assert got.arch == esm.ARCH_8M and dt == esm.DTYPE_Q4_0
    raw = bytearray(p.read_bytes())
    raw[4:8] = (7).to_bytes(4, "little")  # bad version
    p.write_bytes(bytes(raw))
    with pytest.raises(esm.EsmError) as e:
        esm.detect_file(str(p))
    assert e.value.code == esm.ESM_EFORMAT


def test_missing_file_is_eio(esm, tmp_path):
    with pytest.raises(esm.EsmError) as e:
        esm.detect_file(str(tmp_path / "nope.bin"))
    assert e.value.code == esm.ESM_EIO


def test_context_without_gpu_fails_cleanly(esm):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = ctypes.c_void_p()
    rc = esm.lib().esm_ctx_create(0, ctypes.byref(ctx))
    assert rc == esm.ESM_ECUDA and not ctx.value


def test_synthetic_weights_are_seeded(esm):
    cfg = esm.EsmConfig(dim=64, hidden_dim=256, n_layers=2, n_heads=4)
    a = esm.synth_fp32_tensors(cfg, seed=7)
    b = esm.synth_fp32_tensors(cfg, seed=7)
    for n in esm.TENSOR_NAMES:
        assert np.array_equal(a[n], b[n])
    assert a["classifier"].size == cfg.lm_head_floats()
    d, V = cfg.dim, cfg.vocab_size
    dec = a["classifier"][3 * d + d * d: 3 * d + d * d + V * d]
    assert np.array_equal(dec, a["tok_emb"])  # tied LM decoder


def test_synthetic_presets_match_the_library(esm):
    # The numpy-only presets that the CPU baseline and the fixture generators use are the
    # library's EsmConfig presets.
    import synth
    for arch in range(5):
        a, b = synth.preset(arch), esm.EsmConfig.preset(arch)
        assert (a.dim, a.hidden_dim, a.n_layers, a.n_heads, a.vocab_size, a.arch) == \
               (b.dim, b.hidden_dim, b.n_layers, b.n_heads, b.vocab_size, b.arch)
