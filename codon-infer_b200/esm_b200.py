"""Python front end of libesm_b200.so (ctypes over the C ABI in include/esm_b200.h).

Mirrors codon-infer's model API for the encoder forward: EsmConfig presets, weight loading
(host tensors in EsmWeights order, or CODQ / grouped_canonical_v1 files), the Q8_0/Q4_0
quantizers, the tokenizer, and forward_bidirectional over a batch. The library is required: there
is no CPU fallback, and loading fails loudly when it is missing.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from synth import random_sequences, synth_fp32_tensors  # noqa: F401 (re-exported)

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libesm_b200.so"

ESM_OK, ESM_EINVAL, ESM_EFORMAT, ESM_ECAPACITY, ESM_ECUDA, ESM_ENCCL, ESM_ETIMEOUT, ESM_ENOMEM, ESM_EIO = range(9)
DTYPE_FP32, DTYPE_Q8_0, DTYPE_Q4_0, DTYPE_Q3_LUT = 0, 1, 2, 3
ARCH_8M, ARCH_35M, ARCH_150M, ARCH_650M, ARCH_3B = range(5)
Q8_BLOCK_BYTES, Q4_BLOCK_BYTES = 36, 20
MASK_ID = 32

# EsmWeights field order (also the grouped_canonical_v1 / CODQ file order).
TENSOR_NAMES = (
    "tok_emb", "ln1_w", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
    "ln2_w", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b", "lnf_w", "lnf_b", "classifier",
)
MATRICES = ("wq", "wk", "wv", "wo", "fc1_w", "fc2_w")
PROFILE_KINDS = ("dequant", "norm", "gemm", "attention", "contact", "head")
# CANONICAL_AAS order of the mutational-scan columns (src/benchmark.rs:702-707).
CANONICAL_AAS = "ACDEFGHIKLMNPQRSTVWY"
CANONICAL_IDS = (5, 23, 13, 9, 18, 6, 21, 12, 15, 4, 20, 17, 14, 16, 10, 8, 11, 7, 22, 19)


class EsmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[esm error {code}] {msg}")
        self.code = code


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("dim", "hidden_dim", "n_layers", "n_heads", "vocab_size", "max_seq_len", "arch")]


@dataclass(frozen=True)
class EsmConfig:
    """EsmConfig (src/lib.rs:76-84)."""
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    vocab_size: int = 33
    max_seq_len: int = 1024
    arch: int = 0

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @staticmethod
    def preset(arch: int) -> "EsmConfig":
        c = _Config()
        _check(lib().esm_config_preset(arch, ctypes.byref(c)), "esm_config_preset")
        return EsmConfig(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.vocab_size, c.max_seq_len, c.arch)

    def c_struct(self) -> _Config:
        return _Config(self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.vocab_size, self.max_seq_len,
                       self.arch)

    def lm_head_floats(self) -> int:
        d, V = self.dim, self.vocab_size
        return 3 * d + d * d + V * d + V


def esm2_8m() -> EsmConfig: return EsmConfig.preset(ARCH_8M)
def esm2_35m() -> EsmConfig: return EsmConfig.preset(ARCH_35M)
def esm2_150m() -> EsmConfig: return EsmConfig.preset(ARCH_150M)
def esm2_650m() -> EsmConfig: return EsmConfig.preset(ARCH_650M)
def esm2_3b() -> EsmConfig: return EsmConfig.preset(ARCH_3B)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with codon-infer_b200/build.py "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        sig = {
            "esm_config_preset": [i32, vp],
            "esm_config_detect_file": [ctypes.c_char_p, vp, vp],
            "esm_get_config": [vp, vp, vp],
            "esm_quantize_q8": [vp, i64, vp],
            "esm_quantize_q4": [vp, i64, vp],
            "esm_quantize_q3": [vp, i64, vp],
            "esm_tokenize": [ctypes.c_char_p, vp, i32, vp],
            "esm_ctx_create": [i32, vp],
            "esm_ctx_destroy": [vp],
            "esm_load_file": [vp, ctypes.c_char_p, vp],
            "esm_load_host": [vp, vp, i32, vp, vp],
            "esm_load_host_quantized": [vp, vp, i32, vp, vp],
            "esm_load_file_quantized": [vp, ctypes.c_char_p, vp, i32],
            "esm_quantize_device": [i32, vp, i64, vp, vp],
            "esm_contact_top_pairs": [vp, vp, i32, ctypes.c_char_p, i32, i32, f32, vp, vp, vp, vp, vp],
            "esm_contacts_pipeline": [vp, ctypes.c_char_p, i32, i32, f32, vp, vp, vp, vp, vp, vp, vp],
            "esm_set_contact_head": [vp, vp, i32, f32],
            "esm_reserve": [vp, i32, i32, i32, i32],
            "esm_forward": [vp, vp, vp, i32, i32, vp, vp, vp],
            "esm_forward_ext": [vp, vp, vp, i32, i32, vp, vp, vp, vp],
            "esm_forward_device": [vp, vp, vp, i32, vp, vp, vp, vp, vp, i32],
            "esm_matmul_tiled": [vp, i32, vp, vp, vp, i32, i32, i32, vp],
            "esm_dms_masked_marginal": [vp, vp, i32, i32, vp, vp],
            "esm_dms_wildtype_marginal": [vp, vp, i32, i32, i32, vp, vp],
            "esm_dms_masked_marginal_range": [vp, vp, i32, i32, i32, i32, vp, vp],
            "esm_partition": [vp, i32, i32, i32, i32, vp],
            "esm_group_create": [vp, i32, vp],
            "esm_group_destroy": [vp],
            "esm_group_size": [vp, vp],
            "esm_group_ctx": [vp, i32, vp],
            "esm_group_load_host": [vp, vp, i32, vp, vp],
            "esm_group_load_file": [vp, ctypes.c_char_p, vp],
            "esm_group_set_contact_head": [vp, vp, i32, f32],
            "esm_group_reserve": [vp, i32, i32, i32, i32],
            "esm_group_forward": [vp, vp, vp, i32, i32, vp, vp, vp],
            "esm_group_dms_masked_marginal": [vp, vp, i32, i32, vp, vp],
            "esm_check_device": [vp],
            "esm_probe_wait_timeout": [vp, i32],
            "esm_profile_enable": [vp, i32],
            "esm_profile_read": [vp, i32, vp, vp, vp, vp],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.esm_last_error.argtypes = [vp]
        L.esm_last_error.restype = ctypes.c_char_p
        L.esm_group_last_error.argtypes = [vp]
        L.esm_group_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _check(rc: int, what: str, ctx=None) -> None:
    if rc != ESM_OK:
        msg = lib().esm_last_error(ctx).decode() if ctx else what
        raise EsmError(rc, f"{what}: {msg}")


def _p(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


# ---- quantizers / tokenizer ------------------------------------------------------------------

def quantize_q8(x) -> np.ndarray:
    """BlockQ8_0 blocks (36 bytes each) of a float32 array whose size is a multiple of 32."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * Q8_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().esm_quantize_q8(_p(x), x.size, _p(out)), "esm_quantize_q8")
    return out


def quantize_q4(x) -> np.ndarray:
    """BlockQ4_0 blocks (20 bytes each) of a float32 array whose size is a multiple of 32."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * Q4_BLOCK_BYTES, dtype=np.uint8)
    _check(lib().esm_quantize_q4(_p(x), x.size, _p(out)), "esm_quantize_q4")
    return out


def quantize_q3(x) -> np.ndarray:
    """BlockQ3_LUT blocks (14 bytes each) of a float32 array whose size is a multiple of 32."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.empty(x.size // 32 * 14, dtype=np.uint8)
    _check(lib().esm_quantize_q3(_p(x), x.size, _p(out)), "esm_quantize_q3")
    return out


def quantize_device(dtype: int, d_src: int, n: int, d_dst: int, stream: int = 0) -> None:
    """esm_quantize_device on raw device pointers (e.g. torch tensors' data_ptr())."""
    rc = lib().esm_quantize_device(dtype, d_src, n, d_dst, stream or None)
    if rc != ESM_OK:
        raise EsmError(rc, "esm_quantize_device")


def tokenize(seq: str) -> np.ndarray:
    """Tokenizer::encode: <cls> + residue ids + <eos> (int32)."""
    cap = len(seq.encode()) + 2
    out = np.empty(cap, dtype=np.int32)
    n = ctypes.c_int32(0)
    _check(lib().esm_tokenize(seq.encode(), _p(out), cap, ctypes.byref(n)), "esm_tokenize")
    return out[: n.value].copy()


def detect_file(path: str) -> tuple[EsmConfig, int]:
    c = _Config()
    dt = ctypes.c_int32(0)
    _check(lib().esm_config_detect_file(str(path).encode(), ctypes.byref(c), ctypes.byref(dt)), "detect_file")
    return EsmConfig(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.vocab_size, c.max_seq_len, c.arch), dt.value


# ---- synthetic weights ---------------------------------------------------------------------------

def quantize_tensors(t: dict, dtype: int) -> dict:
    """Applies EsmWeights::quantize_q8 / quantize_q4 (src/lib.rs:558-607): the six matrices become
    blocks; for Q8_0 the token embedding is quantized too, for Q4_0 it stays FP32."""
    if dtype == DTYPE_FP32:
        return dict(t)
    out = dict(t)
    if dtype == DTYPE_Q3_LUT:
        # EsmWeights::quantize_q3 (src/lib.rs:609-633): Q4_0 attention matrices, Q3_LUT fc1 / fc2.
        for m in MATRICES:
            out[m] = quantize_q3(t[m]) if m in ("fc1_w", "fc2_w") else quantize_q4(t[m])
        return out
    q = quantize_q8 if dtype == DTYPE_Q8_0 else quantize_q4
    for m in MATRICES:
        out[m] = q(t[m])
    if dtype == DTYPE_Q8_0:
        out["tok_emb"] = quantize_q8(t["tok_emb"])
    return out


def write_codq(path: str, cfg: EsmConfig, dtype: int, tensors: dict) -> None:
    """Writes a CODQ v1 file (64-byte header + tensors in EsmWeights order), as
    EsmWeightsQ8::save_to_file_with_header / EsmWeightsQ4::save_to_file do."""
    hdr = np.zeros(64, dtype=np.uint8)
    hdr[0:4] = np.frombuffer(b"CODQ", dtype=np.uint8)
    hdr[4:32] = np.array([1, dtype, cfg.arch, cfg.n_layers, cfg.dim, cfg.hidden_dim, cfg.vocab_size],
                         dtype="<u4").view(np.uint8)
    with open(path, "wb") as f:
        f.write(hdr.tobytes())
        for n in TENSOR_NAMES:
            f.write(np.ascontiguousarray(tensors[n]).tobytes())


# ---- model ----------------------------------------------------------------------------------

class Model:
    """One context on one GPU: weights, contact head and workspace."""

    def __init__(self, device: int = 0):
        self._ctx = ctypes.c_void_p()
        rc = lib().esm_ctx_create(device, ctypes.byref(self._ctx))
        if rc != ESM_OK:
            raise EsmError(rc, f"esm_ctx_create(device={device}) failed")
        self.device = device
        self.cfg: EsmConfig | None = None

    def close(self) -> None:
        if self._ctx:
            lib().esm_ctx_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, rc: int, what: str) -> None:
        if rc != ESM_OK:
            raise EsmError(rc, f"{what}: {lib().esm_last_error(self._ctx).decode()}")

    def load_tensors(self, cfg: EsmConfig, dtype: int, tensors: dict) -> None:
        arrs = [np.ascontiguousarray(tensors[n]) for n in TENSOR_NAMES]
        ptrs = (ctypes.c_void_p * 20)(*[a.ctypes.data if a.size else None for a in arrs])
        sizes = (ctypes.c_size_t * 20)(*[a.nbytes for a in arrs])
        c = cfg.c_struct()
        self._chk(lib().esm_load_host(self._ctx, ctypes.byref(c), dtype, ptrs, sizes), "esm_load_host")
        self.cfg = cfg

    def load_tensors_quantized(self, cfg: EsmConfig, dtype: int, fp32_tensors: dict) -> None:
        """FP32 tensors (synth_fp32_tensors layout) quantized to `dtype` on the device while loading
        (EsmWeights::quantize_q8 / quantize_q4)."""
        arrs = [np.ascontiguousarray(fp32_tensors[n], dtype=np.float32) for n in TENSOR_NAMES]
        ptrs = (ctypes.c_void_p * 20)(*[a.ctypes.data if a.size else None for a in arrs])
        sizes = (ctypes.c_size_t * 20)(*[a.nbytes for a in arrs])
        c = cfg.c_struct()
        self._chk(lib().esm_load_host_quantized(self._ctx, ctypes.byref(c), dtype, ptrs, sizes),
                  "esm_load_host_quantized")
        self.cfg = cfg

    def load_file_quantized(self, path: str, dtype: int, cfg: EsmConfig | None = None) -> None:
        c = cfg.c_struct() if cfg else None
        self._chk(lib().esm_load_file_quantized(self._ctx, str(path).encode(), ctypes.byref(c) if c else None, dtype),
                  "esm_load_file_quantized")
        self.cfg = self.loaded_config()[0]

    def contact_top_pairs(self, d_map: int, n: int, seq: str, min_separation: int = 6,
                          max_k: int | None = None, top_l_factor: float = 1.0) -> dict:
        """Ranked contact pairs of one sequence's n x n map in device memory (a device pointer), as
        compute_pipeline_contacts_parallel ranks them; see esm_contact_top_pairs."""
        cap = 4096
        pos1 = np.zeros(cap, dtype=np.int32)
        pos2 = np.zeros(cap, dtype=np.int32)
        score = np.zeros(cap, dtype=np.float32)
        n_out = ctypes.c_int32(0)
        enr = ctypes.c_float(0.0)
        self._chk(lib().esm_contact_top_pairs(self._ctx, d_map, n, seq.encode(), min_separation,
                                              -1 if max_k is None else max_k, top_l_factor, _p(pos1), _p(pos2),
                                              _p(score), ctypes.byref(n_out), ctypes.byref(enr)),
                  "esm_contact_top_pairs")
        k = n_out.value
        return {"pos1": pos1[:k], "pos2": pos2[:k], "score": score[:k], "cys_enrichment": enr.value}

    def contacts_pipeline(self, seq: str, min_separation: int = 6, max_k: int | None = None,
                          top_l_factor: float = 1.0, want_map: bool = False, want_logits: bool = False) -> dict:
        """compute_pipeline_contacts_parallel for one residue string in one call (esm_contacts_pipeline):
        the forward with contacts and the pair ranking run on the GPU; the n x n map and the logits
        come back only when asked for."""
        n = len(seq.encode())
        cap = 4096
        pos1 = np.zeros(cap, dtype=np.int32)
        pos2 = np.zeros(cap, dtype=np.int32)
        score = np.zeros(cap, dtype=np.float32)
        cmap = np.empty((n, n), dtype=np.float32) if want_map else None
        logits = np.empty((n + 2, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        n_out = ctypes.c_int32(0)
        enr = ctypes.c_float(0.0)
        self._chk(lib().esm_contacts_pipeline(self._ctx, seq.encode(), min_separation, -1 if max_k is None else max_k,
                                              top_l_factor, _p(logits), _p(cmap), _p(pos1), _p(pos2), _p(score),
                                              ctypes.byref(n_out), ctypes.byref(enr)), "esm_contacts_pipeline")
        k = n_out.value
        res = {"pos1": pos1[:k], "pos2": pos2[:k], "score": score[:k], "cys_enrichment": enr.value}
        if want_map:
            res["contact_probs"] = cmap
        if want_logits:
            res["logits"] = logits
        return res

    def load_file(self, path: str, cfg: EsmConfig | None = None) -> None:
        c = cfg.c_struct() if cfg else None
        self._chk(lib().esm_load_file(self._ctx, str(path).encode(), ctypes.byref(c) if c else None), "esm_load_file")
        self.cfg = self.loaded_config()[0]

    def loaded_config(self) -> tuple[EsmConfig, int]:
        """The configuration and storage type of the loaded weights (a CODQ header's, when the
        file has one)."""
        c = _Config()
        dt = ctypes.c_int32(0)
        self._chk(lib().esm_get_config(self._ctx, ctypes.byref(c), ctypes.byref(dt)), "esm_get_config")
        return EsmConfig(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.vocab_size, c.max_seq_len, c.arch), dt.value

    def set_contact_head(self, w, b: float) -> None:
        w = np.ascontiguousarray(w, dtype=np.float32)
        self._chk(lib().esm_set_contact_head(self._ctx, _p(w), w.size, float(b)), "esm_set_contact_head")

    def reserve(self, max_tokens: int, max_seqs: int, max_len: int, contacts: bool = False) -> None:
        self._chk(lib().esm_reserve(self._ctx, max_tokens, max_seqs, max_len, int(contacts)), "esm_reserve")

    def forward(self, seqs, lengths=None, want_hidden: bool = False, want_contacts: bool = False,
                logits_out: np.ndarray | None = None, hidden_out: np.ndarray | None = None,
                contacts_out: np.ndarray | None = None, want_layers: bool = False) -> dict:
        """Batched forward_bidirectional from host memory.

        `seqs` is a list of int token arrays, or a right-padded int32 [B, Lmax] array together with
        `lengths`. `logits_out`, `hidden_out` and `contacts_out` may be preallocated (e.g. pinned)
        float32 arrays of shape [B, Lmax, vocab], [B, Lmax, dim] and [B, Lmax - 2, Lmax - 2]; a
        contact map of a long batch is large (536 MB for 8 x 4096), and copying it into fresh
        pageable memory on every call costs more than the forward. `want_layers` adds "layers", the
        residual stream after every layer [n_layers, B, Lmax, dim] (the on_layer hook of the
        reference's _ext forwards). Returns padded outputs; padding positions are zero."""
        if isinstance(seqs, np.ndarray) and seqs.ndim == 2:
            tokens = np.ascontiguousarray(seqs, dtype=np.int32)
            lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        else:
            lengths = np.array([len(s) for s in seqs], dtype=np.int32)
            tokens = np.zeros((len(seqs), int(lengths.max())), dtype=np.int32)
            for i, s in enumerate(seqs):
                tokens[i, : len(s)] = s
        B, Lmax = tokens.shape
        cfg = self.cfg
        if logits_out is None:
            logits_out = np.empty((B, Lmax, cfg.vocab_size), dtype=np.float32)
        assert logits_out.shape == (B, Lmax, cfg.vocab_size) and logits_out.dtype == np.float32
        assert logits_out.flags.c_contiguous
        hidden = None
        if want_hidden:
            hidden = hidden_out if hidden_out is not None else np.empty((B, Lmax, cfg.dim), dtype=np.float32)
            assert hidden.shape == (B, Lmax, cfg.dim) and hidden.dtype == np.float32 and hidden.flags.c_contiguous
        contacts = None
        if want_contacts:
            np_ = max(Lmax - 2, 0)
            contacts = contacts_out if contacts_out is not None else np.empty((B, np_, np_), dtype=np.float32)
            assert contacts.shape == (B, np_, np_) and contacts.dtype == np.float32 and contacts.flags.c_contiguous
        if want_layers:
            layers = np.empty((cfg.n_layers, B, Lmax, cfg.dim), dtype=np.float32)
            self._chk(lib().esm_forward_ext(self._ctx, _p(tokens), _p(lengths), B, Lmax, _p(logits_out), _p(hidden),
                                            _p(contacts), _p(layers)), "esm_forward_ext")
        else:
            self._chk(lib().esm_forward(self._ctx, _p(tokens), _p(lengths), B, Lmax, _p(logits_out), _p(hidden),
                                        _p(contacts)), "esm_forward")
        res = {"logits": logits_out, "lengths": lengths}
        if want_layers:
            res["layers"] = layers
        if want_hidden:
            res["hidden"] = hidden
        if want_contacts:
            res["contacts"] = contacts
        return res

    def forward_device(self, d_tokens, cu_seqlens, d_logits, d_hidden=None, d_contacts=None, d_layer_hidden=None,
                       stream=None, sync: bool = False) -> None:
        """Packed forward on device buffers (torch CUDA tensors or raw pointers)."""
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)

        def ptr(t):
            if t is None:
                return None
            return ctypes.c_void_p(t if isinstance(t, int) else t.data_ptr())
        s = None if stream is None else ctypes.c_void_p(stream if isinstance(stream, int) else stream.cuda_stream)
        self._chk(lib().esm_forward_device(self._ctx, ptr(d_tokens), _p(cu), cu.size - 1, ptr(d_logits),
                                           ptr(d_hidden), ptr(d_contacts), ptr(d_layer_hidden), s, int(sync)),
                  "esm_forward_device")

    def dms_wildtype_marginal(self, residues, window_size: int = 0, stride: int = 0):
        """Wild-type-marginal scan (no masking, sliding windows); same outputs as dms_masked_marginal."""
        r = np.ascontiguousarray(residues, dtype=np.int32)
        deltas = np.empty((r.size, 20), dtype=np.float32)
        ent = np.empty(r.size, dtype=np.float32)
        self._chk(lib().esm_dms_wildtype_marginal(self._ctx, _p(r), r.size, window_size, stride, _p(deltas),
                                                  _p(ent)), "esm_dms_wildtype_marginal")
        return deltas, ent

    def dms_masked_marginal(self, residues, window_size: int = 0):
        """Masked-marginal deep mutational scan of one sequence (residue token ids, no <cls>/<eos>).
        Returns (deltas [n, 20] in CANONICAL_AAS order, entropy [n])."""
        r = np.ascontiguousarray(residues, dtype=np.int32)
        deltas = np.empty((r.size, 20), dtype=np.float32)
        ent = np.empty(r.size, dtype=np.float32)
        self._chk(lib().esm_dms_masked_marginal(self._ctx, _p(r), r.size, window_size, _p(deltas), _p(ent)),
                  "esm_dms_masked_marginal")
        return deltas, ent

    def dms_masked_marginal_range(self, residues, pos_begin: int, pos_end: int, window_size: int = 0):
        """Rows [pos_begin, pos_end) of dms_masked_marginal on the same sequence (the block of a
        scan one GPU runs when the scan is split across GPUs)."""
        r = np.ascontiguousarray(residues, dtype=np.int32)
        m = pos_end - pos_begin
        deltas = np.empty((max(m, 0), 20), dtype=np.float32)
        ent = np.empty(max(m, 0), dtype=np.float32)
        self._chk(lib().esm_dms_masked_marginal_range(self._ctx, _p(r), r.size, window_size, pos_begin, pos_end,
                                                      _p(deltas), _p(ent)), "esm_dms_masked_marginal_range")
        return deltas, ent

    def matmul_tiled(self, dtype: int, x, w, bias, in_dim: int, out_dim: int) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        seq_len = x.size // in_dim
        w = np.ascontiguousarray(w)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        out = np.empty((seq_len, out_dim), dtype=np.float32)
        self._chk(lib().esm_matmul_tiled(self._ctx, dtype, _p(x), _p(w), _p(b), in_dim, out_dim, seq_len, _p(out)),
                  "esm_matmul_tiled")
        return out

    def profile_enable(self, on: bool = True) -> None:
        self._chk(lib().esm_profile_enable(self._ctx, int(on)), "esm_profile_enable")

    def profile_read(self) -> dict:
        """Per kernel class: total ms, launches, algorithmic FLOPs and bytes since profile_enable."""
        out = {}
        for k, name in enumerate(PROFILE_KINDS):
            ms, n, fl, by = ctypes.c_double(), ctypes.c_int64(), ctypes.c_double(), ctypes.c_double()
            self._chk(lib().esm_profile_read(self._ctx, k, ctypes.byref(ms), ctypes.byref(n), ctypes.byref(fl),
                                             ctypes.byref(by)), "esm_profile_read")
            out[name] = {"ms": ms.value, "launches": n.value, "flops": fl.value, "bytes": by.value}
        return out

    def probe_wait_timeout(self, limit_ms: int = 50) -> int:
        """Runs the bounded-wait self-test; returns the status (ESM_ETIMEOUT when it works)."""
        return lib().esm_probe_wait_timeout(self._ctx, limit_ms)

    def check_device(self) -> None:
        self._chk(lib().esm_check_device(self._ctx), "esm_check_device")


# ---- several GPUs from one process -------------------------------------------------------------

def partition(lengths, parts: int, dim: int, hidden_dim: int) -> list[range]:
    """esm_partition: contiguous cost-balanced blocks of sequence indices, one per device."""
    ln = np.ascontiguousarray(lengths, dtype=np.int32)
    bounds = np.zeros(parts + 1, dtype=np.int32)
    _check(lib().esm_partition(_p(ln), ln.size, dim, hidden_dim, parts, _p(bounds)), "esm_partition")
    return [range(int(bounds[r]), int(bounds[r + 1])) for r in range(parts)]


class Group:
    """esm_group: one context per device of one host process, with the batch split across them."""

    def __init__(self, devices):
        devs = np.ascontiguousarray(devices, dtype=np.int32)
        self._g = ctypes.c_void_p()
        rc = lib().esm_group_create(_p(devs), devs.size, ctypes.byref(self._g))
        if rc != ESM_OK:
            raise EsmError(rc, f"esm_group_create(devices={list(devices)}) failed")
        self.devices = [int(d) for d in devs]
        self.cfg: EsmConfig | None = None

    def close(self) -> None:
        if self._g:
            lib().esm_group_destroy(self._g)
            self._g = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _chk(self, rc: int, what: str) -> None:
        if rc != ESM_OK:
            raise EsmError(rc, f"{what}: {lib().esm_group_last_error(self._g).decode()}")

    def load_tensors(self, cfg: EsmConfig, dtype: int, tensors: dict) -> None:
        arrs = [np.ascontiguousarray(tensors[n]) for n in TENSOR_NAMES]
        ptrs = (ctypes.c_void_p * 20)(*[a.ctypes.data if a.size else None for a in arrs])
        sizes = (ctypes.c_size_t * 20)(*[a.nbytes for a in arrs])
        c = cfg.c_struct()
        self._chk(lib().esm_group_load_host(self._g, ctypes.byref(c), dtype, ptrs, sizes), "esm_group_load_host")
        self.cfg = cfg

    def set_contact_head(self, w, b: float) -> None:
        w = np.ascontiguousarray(w, dtype=np.float32)
        self._chk(lib().esm_group_set_contact_head(self._g, _p(w), w.size, float(b)), "esm_group_set_contact_head")

    def reserve(self, max_tokens: int, max_seqs: int, max_len: int, contacts: bool = False) -> None:
        self._chk(lib().esm_group_reserve(self._g, max_tokens, max_seqs, max_len, int(contacts)), "esm_group_reserve")

    def forward(self, seqs, want_hidden: bool = False, want_contacts: bool = False) -> dict:
        lengths = np.array([len(s) for s in seqs], dtype=np.int32)
        B, Lmax = len(seqs), int(lengths.max())
        tokens = np.zeros((B, Lmax), dtype=np.int32)
        for i, s in enumerate(seqs):
            tokens[i, : len(s)] = s
        cfg = self.cfg
        logits = np.empty((B, Lmax, cfg.vocab_size), dtype=np.float32)
        hidden = np.empty((B, Lmax, cfg.dim), dtype=np.float32) if want_hidden else None
        np_ = max(Lmax - 2, 0)
        contacts = np.empty((B, np_, np_), dtype=np.float32) if want_contacts else None
        self._chk(lib().esm_group_forward(self._g, _p(tokens), _p(lengths), B, Lmax, _p(logits), _p(hidden),
                                          _p(contacts)), "esm_group_forward")
        res = {"logits": logits, "lengths": lengths}
        if want_hidden:
            res["hidden"] = hidden
        if want_contacts:
            res["contacts"] = contacts
        return res

    def dms_masked_marginal(self, residues, window_size: int = 0):
        r = np.ascontiguousarray(residues, dtype=np.int32)
        deltas = np.empty((r.size, 20), dtype=np.float32)
        ent = np.empty(r.size, dtype=np.float32)
        self._chk(lib().esm_group_dms_masked_marginal(self._g, _p(r), r.size, window_size, _p(deltas), _p(ent)),
                  "esm_group_dms_masked_marginal")
        return deltas, ent
