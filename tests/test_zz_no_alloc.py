"""The allocation-free GEMM entry point, for callers that cannot call cudaMalloc (device memory
reserved up front by their own allocator, no tolerance for cudaMalloc's implicit synchronisation,
or a host that forbids its plugins any allocation).

esm_matmul_tiled_noalloc keeps its fp16 operand copies in one static device array shared by all
calls, so two calls in a row with different shapes (the second on top of the first call's leftover
bytes) must each agree with the allocating entry point esm_matmul_tiled, within the GEMM tolerance
of the other GPU tests: 3 * 2^-11 * sum_k |x w| + 1e-5 per element (fp16 operands, fp32
accumulation). This file is collected last so a failure here cannot stop the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

U16 = 2.0 ** -11


def _noalloc(esm):
    fn = esm.lib().esm_matmul_tiled_noalloc
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    fn.argtypes = [i32, vp, vp, vp, i32, i32, i32, vp, vp]
    fn.restype = ctypes.c_int
    return fn


def test_noalloc_matches_allocating_entry_point_twice(esm, orc):
    import torch

    fn = _noalloc(esm)
    model = esm.Model(0)
    dev = torch.device("cuda:0")
    stream = torch.cuda.Stream(dev)
    # First a larger problem, then a smaller one with a ragged output width over its leftovers,
    # then Q3_LUT blocks (14 bytes, so rows start at any byte).
    cases = [(esm.DTYPE_Q4_0, 1280, 640, 300), (esm.DTYPE_Q8_0, 480, 33, 77), (esm.DTYPE_Q3_LUT, 640, 100, 50)]
    for call, (dt, in_dim, out_dim, seq_len) in enumerate(cases):
        rng = np.random.default_rng(100 + call)
        x = rng.standard_normal(seq_len * in_dim, dtype=np.float32)
        w32 = (rng.standard_normal(out_dim * in_dim, dtype=np.float32) * 0.02).astype(np.float32)
        b = (rng.standard_normal(out_dim, dtype=np.float32) * 0.1).astype(np.float32)
        quant = {esm.DTYPE_Q4_0: (esm.quantize_q4, orc.dequantize_q4), esm.DTYPE_Q8_0: (esm.quantize_q8, orc.dequantize_q8),
                 esm.DTYPE_Q3_LUT: (esm.quantize_q3, orc.dequantize_q3)}[dt]
        wq = quant[0](w32)
        deq = quant[1](wq)

        expect = model.matmul_tiled(dt, x, wq, b, in_dim, out_dim)

        d_x = torch.from_numpy(x).to(dev)
        d_w = torch.from_numpy(wq).to(dev)
        d_b = torch.from_numpy(b).to(dev)
        d_out = torch.full((seq_len, out_dim), float("nan"), device=dev)
        torch.cuda.synchronize(dev)
        rc = fn(dt, d_x.data_ptr(), d_w.data_ptr(), d_b.data_ptr(), in_dim, out_dim, seq_len, d_out.data_ptr(),
                stream.cuda_stream)
        assert rc == esm.ESM_OK, f"call {call}: status {rc}"
        got = d_out.cpu().numpy()

        bound = 3 * U16 * (np.abs(x.reshape(seq_len, in_dim)).astype(np.float64)
                           @ np.abs(deq.reshape(out_dim, in_dim)).astype(np.float64).T) + 1e-5
        assert np.isfinite(got).all()
        assert (np.abs(got.astype(np.float64) - expect) <= bound).all(), f"call {call} differs"
    model.close()


def test_noalloc_rejects_problems_beyond_its_scratch(esm):
    import torch

    fn = _noalloc(esm)
    limit = 32 << 20                       # ESM_NOALLOC_SCRATCH_BYTES in include/esm_b200.h
    in_dim, out_dim = 4096, 4096           # fp16 weight copy alone is 32 MiB
    seq_len = 16
    assert 2 * (seq_len + out_dim) * in_dim > limit
    d_x = torch.zeros(seq_len * in_dim, device="cuda:0")
    d_w = torch.zeros(out_dim * in_dim, device="cuda:0")
    d_out = torch.zeros(seq_len * out_dim, device="cuda:0")
    rc = fn(esm.DTYPE_FP32, d_x.data_ptr(), d_w.data_ptr(), None, in_dim, out_dim, seq_len, d_out.data_ptr(), None)
    assert rc == esm.ESM_ECAPACITY
