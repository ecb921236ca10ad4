"""ctypes front end of the CPU restatement oracle (``oracle/esm_oracle.cpp``).

TEST INFRASTRUCTURE ONLY: the parity checker for the B200 library. Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this module; the
product package never does.

The restated reference functions are listed, with their codon-infer file:line, at the top of
``esm_oracle.cpp``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libesm_oracle.so"

DT_FP32, DT_Q8, DT_Q4, DT_Q3 = 0, 1, 2, 3
Q8_BLOCK_BYTES = 36  # BlockQ8_0 {f32 d; i8 qs[32]}, src/lib.rs:640-645
Q4_BLOCK_BYTES = 20  # BlockQ4_0 {f32 d; u8 qs[16]}, src/lib.rs:1043-1051

# EsmWeights field order, src/lib.rs:299-307 (also the grouped_canonical_v1 file order).
TENSOR_NAMES = (
    "tok_emb", "ln1_w", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
    "ln2_w", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "lnf_w", "lnf_b", "classifier",
)

_lib = None
_LAYER_CB = ctypes.CFUNCTYPE(None, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_void_p)


def build() -> Path:
    """Compile the oracle with its Makefile (g++ only; no CUDA)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "esm_oracle.cpp").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i64, f32p = ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_float)
        L.orc_quantize_q8.argtypes = [vp, i64, vp]
        L.orc_quantize_q4.argtypes = [vp, i64, vp]
        L.orc_dequantize_q8.argtypes = [vp, i64, vp]
        L.orc_dequantize_q4.argtypes = [vp, i64, vp]
        L.orc_quantize_q3.argtypes = [vp, i64, vp]
        L.orc_dequantize_q3.argtypes = [vp, i64, vp]
        L.orc_tiled_gemm.argtypes = [ctypes.c_int, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_layer_norm.argtypes = [vp, vp, vp, vp, ctypes.c_int]
        L.orc_gelu.argtypes = [ctypes.c_float]
        L.orc_gelu.restype = ctypes.c_float
        L.orc_softmax.argtypes = [vp, ctypes.c_int]
        L.orc_log_softmax_canonical.argtypes = [vp, vp]
        L.orc_rope_tables.argtypes = [ctypes.c_int, ctypes.c_int, vp, vp]
        L.orc_accumulate_head_apc.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_forward.argtypes = [
            vp, ctypes.c_int, ctypes.POINTER(vp), i64, vp, ctypes.c_int, ctypes.c_int, vp, ctypes.c_float,
            vp, vp, vp, _LAYER_CB, vp,
        ]
        L.orc_forward.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def quantize_q8(x) -> np.ndarray:
    """BlockQ8_0 blocks (raw bytes, 36 per block) of a float32 array whose size is a multiple of 32."""
    x = _f32(x).ravel()
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * Q8_BLOCK_BYTES, dtype=np.uint8)
    lib().orc_quantize_q8(_ptr(x), x.size, _ptr(out))
    return out


def quantize_q4(x) -> np.ndarray:
    """BlockQ4_0 blocks (raw bytes, 20 per block) of a float32 array whose size is a multiple of 32."""
    x = _f32(x).ravel()
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * Q4_BLOCK_BYTES, dtype=np.uint8)
    lib().orc_quantize_q4(_ptr(x), x.size, _ptr(out))
    return out


def quantize_tensors(t: dict, dtype: int) -> dict:
    """EsmWeights::quantize_q8 / quantize_q4 / quantize_q3 (src/lib.rs:558-633) with the oracle's
    quantizers: the six matrices become blocks; Q8_0 also quantizes the token embedding (Q4_0
    keeps it FP32); Q3_LUT stores the attention matrices as Q4_0 and fc1 / fc2 as Q3_LUT."""
    out = dict(t)
    if dtype == DT_FP32:
        return out
    mats = ("wq", "wk", "wv", "wo", "fc1_w", "fc2_w")
    for m in mats:
        if dtype == DT_Q3:
            out[m] = quantize_q3(t[m]) if m in ("fc1_w", "fc2_w") else quantize_q4(t[m])
        else:
            out[m] = quantize_q8(t[m]) if dtype == DT_Q8 else quantize_q4(t[m])
    if dtype == DT_Q8:
        out["tok_emb"] = quantize_q8(t["tok_emb"])
    return out


def dequantize_q8(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // Q8_BLOCK_BYTES * 32
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize_q8(_ptr(blocks), n, _ptr(out))
    return out


def dequantize_q4(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // Q4_BLOCK_BYTES * 32
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize_q4(_ptr(blocks), n, _ptr(out))
    return out


def quantize_q3(x) -> np.ndarray:
    """BlockQ3_LUT blocks (raw bytes, 14 per block) of a float32 array whose size is a multiple of 32."""
    x = _f32(x).ravel()
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * 14, dtype=np.uint8)
    lib().orc_quantize_q3(_ptr(x), x.size, _ptr(out))
    return out


def dequantize_q3(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = blocks.size // 14 * 32
    out = np.empty(n, dtype=np.float32)
    lib().orc_dequantize_q3(_ptr(blocks), n, _ptr(out))
    return out


def tiled_gemm(dtype: int, x: np.ndarray, w: np.ndarray, bias: np.ndarray, in_dim: int, out_dim: int,
               n_threads: int = 1) -> np.ndarray:
    """matmul_tiled_{fp32,q8,q4}_parallel: [L, in] x W[out, in]^T + b -> [L, out]."""
    x = _f32(x)
    seq_len = x.size // in_dim
    out = np.empty((seq_len, out_dim), dtype=np.float32)
    w = np.ascontiguousarray(w)
    lib().orc_tiled_gemm(dtype, _ptr(out), _ptr(x), _ptr(w), _ptr(_f32(bias)), in_dim, out_dim, seq_len, n_threads)
    return out


def layer_norm(x, w, b) -> np.ndarray:
    x, w, b = _f32(x), _f32(w), _f32(b)
    out = np.empty_like(x)
    lib().orc_layer_norm(_ptr(out), _ptr(x), _ptr(w), _ptr(b), x.size)
    return out


def gelu(x: float) -> float:
    return float(lib().orc_gelu(float(x)))


def softmax(x) -> np.ndarray:
    x = _f32(x).copy()
    lib().orc_softmax(_ptr(x), x.size)
    return x


def log_softmax_canonical(logits) -> np.ndarray:
    x = _f32(logits)
    out = np.empty(33, dtype=np.float32)
    lib().orc_log_softmax_canonical(_ptr(x), _ptr(out))
    return out


# CANONICAL_AAS token ids in column order (src/benchmark.rs:702-707).
CANONICAL_IDS = (5, 23, 13, 9, 18, 6, 21, 12, 15, 4, 20, 17, 14, 16, 10, 8, 11, 7, 22, 19)


def dms_scores(logits_row, wt_tok: int) -> tuple[np.ndarray, float]:
    """One masked-marginal row of run_pipeline_dms_with_mode (src/pipeline.rs:150-171): the
    canonical log-softmax of the masked position's logits, the Shannon entropy over ids 4..=23
    (f32 sum, terms with p <= 1e-12 skipped), and the 20 deltas log P(aa) - log P(wt) in
    CANONICAL_AAS order (0 for the wild-type column)."""
    lp = log_softmax_canonical(logits_row)
    ent = np.float32(0.0)
    for i in range(4, 24):
        p = np.float32(np.exp(lp[i]))
        if p > 1e-12:
            ent = np.float32(ent - p * lp[i])
    deltas = np.array([0.0 if aa == wt_tok else lp[aa] - lp[wt_tok] for aa in CANONICAL_IDS], dtype=np.float32)
    return deltas, float(ent)


def rope_tables(max_len: int, head_dim: int):
    cos = np.empty((max_len, head_dim // 2), dtype=np.float32)
    sin = np.empty_like(cos)
    lib().orc_rope_tables(max_len, head_dim, _ptr(cos), _ptr(sin))
    return cos, sin


def accumulate_head_apc(head_att, contact_logits: np.ndarray, seq_len: int, n_res: int, w: float) -> None:
    head_att = _f32(head_att)
    assert contact_logits.dtype == np.float32 and contact_logits.flags.c_contiguous
    lib().orc_accumulate_head_apc(_ptr(head_att), _ptr(contact_logits), seq_len, n_res, float(w))


def forward(cfg, dtype: int, tensors: dict, tokens, n_threads: int | None = None,
            contact_w=None, contact_b: float = 0.0, want_hidden: bool = False, on_layer=None):
    """One sequence through the reference forward (FP32 / Q8_0 / Q4_0 / Q3_LUT by ``dtype``).

    ``cfg`` has dim, hidden_dim, n_layers, n_heads, vocab_size; ``tensors`` maps TENSOR_NAMES to
    numpy arrays (float32, or uint8 block bytes for quantized matrices). Returns a dict with
    ``logits`` [L, V], and ``hidden`` [L, d] / ``contacts`` [n, n] when requested.
    """
    toks = np.ascontiguousarray(tokens, dtype=np.int32)
    L = toks.size
    c5 = np.array([cfg.dim, cfg.hidden_dim, cfg.n_layers, cfg.n_heads, cfg.vocab_size], dtype=np.int32)
    arrs = [np.ascontiguousarray(tensors[n]) for n in TENSOR_NAMES]
    ptrs = (ctypes.c_void_p * 20)(*[a.ctypes.data for a in arrs])
    logits = np.empty((L, cfg.vocab_size), dtype=np.float32)
    hidden = np.empty((L, cfg.dim), dtype=np.float32) if want_hidden else None
    n = max(L - 2, 0)
    contacts = None
    cw = None
    if contact_w is not None:
        cw = _f32(contact_w)
        assert cw.size == cfg.n_layers * cfg.n_heads
        contacts = np.empty((n, n), dtype=np.float32)
    if on_layer is not None:
        def _cb(layer, xptr, _user):
            on_layer(layer, np.ctypeslib.as_array(xptr, shape=(L, cfg.dim)).copy())
        cb = _LAYER_CB(_cb)
    else:
        cb = _LAYER_CB()
    nthr = n_threads if n_threads is not None else (os.cpu_count() or 1)
    rc = lib().orc_forward(
        _ptr(c5), dtype, ptrs, arrs[19].size, _ptr(toks), L, nthr, _ptr(cw), float(contact_b),
        _ptr(logits), _ptr(hidden), _ptr(contacts) if contacts is not None and n > 0 else None, cb, None,
    )
    if rc != 0:
        raise ValueError(f"orc_forward rejected its arguments (rc={rc})")
    out = {"logits": logits}
    if want_hidden:
        out["hidden"] = hidden
    if contacts is not None:
        out["contacts"] = contacts
    return out
