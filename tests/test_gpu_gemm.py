"""GPU parity of the tcgen05 projection GEMM through the C ABI (esm_matmul_tiled) against the
oracle's restatement of matmul_tiled_{fp32,q8,q4,q3}_parallel.

Tolerance: the tensor cores see fp16 operands (x and the dequantized weight q*d each rounded once,
relative error <= 2^-11) and accumulate in fp32, so element (p, i) may differ from the fp32
reference by at most ~2 * 2^-11 * sum_k |x[p,k] * w[i,k]|; the test allows 3 * 2^-11 of that sum
plus 1e-5.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

U16 = 2.0 ** -11


@pytest.fixture(scope="module")
def model(esm):
    m = esm.Model(0)
    yield m
    m.close()


def _bound(x, wdeq, in_dim):
    X = np.abs(x.reshape(-1, in_dim)).astype(np.float64)
    W = np.abs(wdeq.reshape(-1, in_dim)).astype(np.float64)
    return 3 * U16 * (X @ W.T) + 1e-5


def _check(model, orc, dt, x, w_f32, bias, in_dim, out_dim):
    if dt == 0:
        wq, deq = w_f32, w_f32
    elif dt == 1:
        wq = orc.quantize_q8(w_f32)
        deq = orc.dequantize_q8(wq)
    elif dt == 2:
        wq = orc.quantize_q4(w_f32)
        deq = orc.dequantize_q4(wq)
    else:
        wq = orc.quantize_q3(w_f32)
        deq = orc.dequantize_q3(wq)
    got = model.matmul_tiled(dt, x, wq, bias, in_dim, out_dim)
    ref = orc.tiled_gemm(dt, x, wq, bias if bias is not None else np.zeros(out_dim, np.float32), in_dim, out_dim,
                         n_threads=8)
    err = np.abs(got.astype(np.float64) - ref)
    bound = _bound(x, deq, in_dim)
    assert np.isfinite(got).all()
    assert (err <= bound).all(), f"max err {err.max():.3e}, worst excess {(err - bound).max():.3e}"


@pytest.mark.parametrize("dt", [0, 1, 2, 3])
@pytest.mark.parametrize("seq_len", [7, 12])
def test_reference_tiled_vs_gemv_case(model, orc, dt, seq_len):
    # The reference's tiled-GEMM test inputs (src/lib.rs:8473-8515): (320 -> 64), seq 7 and 12.
    in_dim, out_dim = 320, 64
    x = np.sin(np.arange(seq_len * in_dim, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    w = (np.cos(np.arange(out_dim * in_dim, dtype=np.float32) * np.float32(0.007)) * 0.5).astype(np.float32)
    b = (np.arange(out_dim, dtype=np.float32) * np.float32(0.01) - np.float32(0.2)).astype(np.float32)
    _check(model, orc, dt, x, w, b, in_dim, out_dim)


@pytest.mark.parametrize("dt", [0, 1, 2, 3])
@pytest.mark.parametrize("shape", [
    (1280, 5120, 300),   # 650M fc1
    (5120, 1280, 257),   # 650M fc2, ragged M
    (1280, 3840, 129),   # 650M fused QKV width
    (480, 1440, 77),     # 35M QKV: K not a multiple of 64, N = 6 x 240
    (640, 2560, 130),    # 150M fc1
    (320, 33, 50),       # decoder width, N padded to 48
    (2560, 10240, 64),   # 3B fc1
])
def test_esm_shapes(model, orc, dt, shape):
    in_dim, out_dim, seq_len = shape
    rng = np.random.default_rng(in_dim + out_dim + seq_len + dt)
    x = rng.standard_normal(seq_len * in_dim, dtype=np.float32)
    w = (rng.standard_normal(out_dim * in_dim, dtype=np.float32) * 0.02).astype(np.float32)
    b = (rng.standard_normal(out_dim, dtype=np.float32) * 0.1).astype(np.float32)
    _check(model, orc, dt, x, w, b, in_dim, out_dim)


def test_zero_weights_give_bias(model, orc):
    # test_q4_zero_weights_zero_x (bias exactly), src/lib.rs:7860-7888
    in_dim, out_dim = 1280, 320
    x = np.zeros(5 * in_dim, dtype=np.float32)
    w = np.zeros(out_dim * in_dim, dtype=np.float32)
    b = np.linspace(-1, 1, out_dim, dtype=np.float32)
    got = model.matmul_tiled(2, x, orc.quantize_q4(w), b, in_dim, out_dim)
    assert np.array_equal(got, np.broadcast_to(b, got.shape))


def test_rejects_bad_in_dim(model, esm):
    with pytest.raises(esm.EsmError) as e:
        model.matmul_tiled(0, np.zeros(33, np.float32), np.zeros(33, np.float32), None, 33, 1)
    assert e.value.code == esm.ESM_EINVAL
