"""The C++ host API (codon-infer_b200/host/codon_infer.hpp) driven by tests/cpp/test_host_api.cpp,
a C++ restatement of codon-infer's own unit tests (src/lib.rs mod tests). The known-answer part
needs no GPU; the forward part writes weight files in the reference's formats, runs
forward_bidirectional / _q8 / _q4 through EsmWeights*::from_file and compares the outputs with
the CPU oracle (logits max-abs <= 2e-2, contacts max-abs <= 1e-2).
"""
import shutil
import subprocess

import numpy as np
import pytest

from conftest import ROOT

LOGIT_TOL = 2e-2
CONTACT_TOL = 1e-2
SEQ = "MKTAYIAKQRQISFVKSHFSRQLEERLGLIEVQAPILSRVGDGTQDNLSGAEKAVQVKVKALPDAQFEVVHSLAKWKRQTLGQHDFSAGEG*YTHMK"


@pytest.fixture(scope="module")
def driver(esm, tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = tmp_path_factory.mktemp("hostcpp") / "test_host_api"
    libdir = ROOT / "codon-infer_b200"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-o", str(out),
                    str(ROOT / "tests" / "cpp" / "test_host_api.cpp"), f"-L{libdir}", "-lesm_b200",
                    f"-Wl,-rpath,{libdir}"], check=True)
    return out


def run(driver, *args):
    r = subprocess.run([str(driver), *map(str, args)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def test_known_answers(driver, tmp_path):
    assert "ok" in run(driver, "cpu", tmp_path)


def _files(esm, tmp_path, seed=31):
    cfg = esm.esm2_8m()
    t = esm.synth_fp32_tensors(cfg, seed=seed, std=0.05, bias_std=0.02, ln_jitter=0.1)
    f32 = tmp_path / "esm2_8m_weights.bin"  # header-less grouped_canonical_v1 FP32
    with open(f32, "wb") as f:
        for n in esm.TENSOR_NAMES:
            f.write(np.ascontiguousarray(t[n], np.float32).tobytes())
    paths = {"fp32": f32}
    for name, dt in (("q8", esm.DTYPE_Q8_0), ("q4", esm.DTYPE_Q4_0)):
        paths[name] = tmp_path / f"esm2_8m_{name}.codq"
        esm.write_codq(str(paths[name]), cfg, dt, esm.quantize_tensors(t, dt))
    return cfg, t, paths


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["fp32", "q8", "q4"])
def test_forward_matches_oracle(esm, orc, driver, tmp_path, kind):
    cfg, t, paths = _files(esm, tmp_path)
    dtype = {"fp32": esm.DTYPE_FP32, "q8": esm.DTYPE_Q8_0, "q4": esm.DTYPE_Q4_0}[kind]
    out = tmp_path / "out.bin"
    run(driver, "forward", paths[kind], kind, SEQ, out, 1, 128)
    raw = np.fromfile(out, np.int32)
    L, V, n = raw[:3]
    vals = raw[3:].view(np.float32)
    logits = vals[: L * V].reshape(L, V)
    contacts = vals[L * V: L * V + n * n].reshape(n, n)
    nl = raw[3 + L * V + n * n]
    layers = raw[4 + L * V + n * n:].view(np.float32).reshape(nl, L, cfg.dim)
    assert nl == (0 if kind == "q8" else cfg.n_layers)  # the reference has no _q8_ext
    i = np.arange(cfg.n_layers * cfg.n_heads)
    head = np.where(i % 3 == 0, 0.0, 0.05 * np.sin(0.7 * i.astype(np.float32))).astype(np.float32)
    toks = esm.tokenize(SEQ)
    states = []
    ref = orc.forward(cfg, dtype, esm.quantize_tensors(t, dtype), toks, contact_w=head, contact_b=-0.5,
                      on_layer=lambda l, x: states.append(x))
    assert np.abs(logits - ref["logits"]).max() <= LOGIT_TOL
    assert (logits.argmax(1) == ref["logits"].argmax(1)).mean() >= 0.99
    assert np.abs(contacts - ref["contacts"]).max() <= CONTACT_TOL
    for l in range(nl):  # on_layer of the _ext forwards
        assert np.abs(layers[l] - states[l]).max() <= 1e-2 * max(np.abs(states[l]).max(), 1.0)


@pytest.mark.gpu
def test_quantized_cosine_similarity(esm, driver, tmp_path):
    _, _, paths = _files(esm, tmp_path)
    run(driver, "cosine", paths["fp32"], paths["q8"], paths["q4"], SEQ)


@pytest.mark.gpu
def test_panics_and_io_errors(esm, driver, tmp_path):
    _, _, paths = _files(esm, tmp_path)
    run(driver, "misuse", paths["q4"])


PIPE_SEQ = "MKTCAYIAKQRQCISFVKSHFSRQLEERLGCLIEVQAPILSC"


@pytest.mark.gpu
def test_pipelines_match_oracle(esm, orc, driver, tmp_path):
    # load_model_weights(QuantizationMode::Q4_0) on an FP32 file, then run_pipeline_dms_with_mode
    # in both modes and compute_pipeline_contacts_parallel (min separation 6, k = n clamped to
    # [5, 50]); every output checked against the oracle run on the same Q4_0 blocks.
    from test_gpu_contact_rank import reference_ranking
    from test_gpu_dms import _oracle_scan, _oracle_wt_scan

    cfg, t, paths = _files(esm, tmp_path)
    out = tmp_path / "pipelines.bin"
    run(driver, "pipelines", paths["fp32"], PIPE_SEQ, out)
    raw = np.fromfile(out, np.uint8)
    n, k = raw[:8].view(np.int32)
    assert n == len(PIPE_SEQ)
    off = 8

    def take(count, dtype=np.float32):
        nonlocal off
        size = count * np.dtype(dtype).itemsize
        a = raw[off:off + size].view(dtype)
        off += size
        return a

    scans = []
    for _ in range(2):
        d = take(n * 20).reshape(n, 20)
        e = take(n)
        scans.append((d, e))
    pairs = take(3 * k, np.int32).reshape(k, 3)
    enr = take(1)[0]
    cmap = take(n * n).reshape(n, n)
    q3 = raw[off:off + 28]
    off += 28
    q3_dq = take(64)
    assert off == raw.size

    tq = esm.quantize_tensors(t, esm.DTYPE_Q4_0)
    residues = esm.tokenize(PIPE_SEQ)[1:-1].astype(np.int32)
    for (got_d, got_e), (window, stride, scan) in zip(
            scans, [(0, 0, _oracle_scan), (16, 5, _oracle_wt_scan)]):
        args = (window,) if scan is _oracle_scan else (window, stride)
        ref_d, ref_e = scan(orc, esm, cfg, esm.DTYPE_Q4_0, tq, residues, *args)
        assert np.abs(got_d - ref_d).max() <= 8e-2
        assert np.abs(got_e - ref_e).max() <= 5e-2

    i = np.arange(cfg.n_layers * cfg.n_heads)
    head = np.where(i % 3 == 0, 0.0, 0.05 * np.sin(0.7 * i.astype(np.float32))).astype(np.float32)
    ref = orc.forward(cfg, esm.DTYPE_Q4_0, tq, esm.tokenize(PIPE_SEQ), contact_w=head, contact_b=-0.5)
    assert np.abs(cmap - ref["contacts"]).max() <= CONTACT_TOL
    # The ranking of the map the pipeline returned is exact, ties and Cys enrichment included.
    ri, rj, rs, renr = reference_ranking(cmap, PIPE_SEQ, 6, None, 1.0)
    assert k == ri.size
    np.testing.assert_array_equal(pairs[:, 0], ri)
    np.testing.assert_array_equal(pairs[:, 1], rj)
    np.testing.assert_array_equal(pairs[:, 2].view(np.float32), rs)
    assert enr == renr

    src = np.sin(np.float32(0.37) * np.arange(64, dtype=np.float32)).astype(np.float32)
    np.testing.assert_array_equal(q3, esm.quantize_q3(src))
    np.testing.assert_array_equal(q3_dq, orc.dequantize_q3(esm.quantize_q3(src)))
