"""Seeded synthetic workloads: ESM-2 architecture presets, random-init weights and residue sequences.

Pure numpy: importing this module loads no native library, so the CPU baseline of the benchmark
and the fixture generators build the very same inputs as the GPU path without touching the
product library.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

MASK_ID = 32
# (dim, hidden_dim, n_layers, n_heads) of EsmConfig::esm2_8m() .. esm2_3b(), src/lib.rs:87-150.
PRESET_DIMS = {
    0: (320, 1280, 6, 20),
    1: (480, 1920, 12, 20),
    2: (640, 2560, 30, 20),
    3: (1280, 5120, 33, 20),
    4: (2560, 10240, 36, 40),
}


@dataclass(frozen=True)
class Arch:
    """The architecture fields a forward needs (the same attribute names as EsmConfig)."""
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


def preset(arch: int) -> Arch:
    d, F, nl, H = PRESET_DIMS[arch]
    return Arch(d, F, nl, H, 33, 1024, arch)


def synth_fp32_tensors(cfg, seed: int = 0, std: float = 0.02, bias_std: float = 0.0,
                       ln_jitter: float = 0.0, tie_decoder: bool = True, with_classifier: bool = True) -> dict:
    """Seeded random-init ESM-2 weights in EsmWeights order (float32 numpy arrays).

    Matrices and the embedding ~ N(0, std); biases ~ N(0, bias_std) (0 by default); LayerNorm
    gamma = 1 + N(0, ln_jitter), beta = N(0, ln_jitter). The classifier is
    [lm_ln_w | lm_ln_b | dense_w | dense_b | dec_w | dec_b] with dec_w a copy of the embedding
    when tie_decoder (the ESM-2 LM head is tied to the token embedding).
    """
    rng = np.random.default_rng(seed)
    d, F, nl, V = cfg.dim, cfg.hidden_dim, cfg.n_layers, cfg.vocab_size

    def normal(n, s):
        if s == 0.0:
            return np.zeros(n, dtype=np.float32)
        a = rng.standard_normal(n, dtype=np.float32)
        a *= np.float32(s)
        return a

    def gamma(n):
        return (np.ones(n, dtype=np.float32) + normal(n, ln_jitter)).astype(np.float32)

    t = {}
    t["tok_emb"] = normal(V * d, std)
    t["ln1_w"] = gamma(nl * d)
    t["ln1_b"] = normal(nl * d, ln_jitter)
    for w, b in (("wq", "bq"), ("wk", "bk"), ("wv", "bv"), ("wo", "bo")):
        t[w] = normal(nl * d * d, std)
        t[b] = normal(nl * d, bias_std)
    t["ln2_w"] = gamma(nl * d)
    t["ln2_b"] = normal(nl * d, ln_jitter)
    t["fc1_w"] = normal(nl * F * d, std)
    t["fc1_b"] = normal(nl * F, bias_std)
    t["fc2_w"] = normal(nl * d * F, std)
    t["fc2_b"] = normal(nl * d, bias_std)
    t["lnf_w"] = gamma(d)
    t["lnf_b"] = normal(d, ln_jitter)
    if with_classifier:
        dec_w = t["tok_emb"].copy() if tie_decoder else normal(V * d, std)
        t["classifier"] = np.concatenate([
            gamma(d), normal(d, ln_jitter), normal(d * d, std), normal(d, bias_std), dec_w, normal(V, bias_std),
        ]).astype(np.float32)
    else:
        t["classifier"] = np.zeros(0, dtype=np.float32)
    return t


def random_sequences(n: int, lengths, seed: int = 0) -> list[np.ndarray]:
    """Token sequences <cls> + residues uniform over the 20 canonical ids 4..23 + <eos>."""
    rng = np.random.default_rng(seed)
    lens = [lengths] * n if np.isscalar(lengths) else list(lengths)
    out = []
    for L in lens:
        s = np.empty(L, dtype=np.int32)
        s[0], s[-1] = 0, 2
        s[1:-1] = rng.integers(4, 24, size=L - 2, dtype=np.int32)
        out.append(s)
    return out


# ---- the benchmark configurations ----------------------------------------------------------------
# Tokens include <cls>/<eos>. c4 is the headline. `batch` is the whole workload of one GPU at N = 1.
CONFIGS = {
    "c1": dict(arch=0, dtype=0, batch=1, lengths="fixed", seq_len=128, contacts=True, dms=False,
               desc="ESM-2 8M FP32 forward, 1 x L=128, contact head on"),
    "c2": dict(arch=1, dtype=1, batch=32, lengths="uniform", seq_len=512, min_len=64, contacts=False, dms=False,
               desc="ESM-2 35M Q8_0 forward, 32 sequences with L in U[64, 512], right-padded"),
    "c3": dict(arch=2, dtype=0, batch=300, lengths="fixed", seq_len=302, contacts=False, dms=True,
               desc="ESM-2 150M FP32 masked-marginal scan: 300 single-<mask> variants of a 300-residue wild type"),
    "c4": dict(arch=3, dtype=2, batch=64, lengths="fixed", seq_len=1024, contacts=False, dms=False,
               desc="ESM-2 650M Q4_0 forward, 64 x L=1024, logits out"),
    "c5": dict(arch=4, dtype=1, batch=8, lengths="fixed", seq_len=4096, contacts=True, dms=False,
               desc="ESM-2 3B Q8_0 forward, 8 x L=4096, contact maps on"),
}
WEIGHT_SEED = 0          # synth_fp32_tensors seed of every benchmark model
CONTACT_HEAD_SEED = 7    # contact-regression weights N(0, 0.1), bias 0
DMS_WILDTYPE_SEED = 2000


def contact_head(cfg) -> np.ndarray:
    """The benchmark's random-init logistic-regression contact head, N(0, 0.1) per (layer, head)."""
    rng = np.random.default_rng(CONTACT_HEAD_SEED)
    return (rng.standard_normal(cfg.n_layers * cfg.n_heads) * 0.1).astype(np.float32)


def dms_wildtype(seq_len: int) -> np.ndarray:
    """Residue ids (no <cls>/<eos>) of the mutational-scan wild type of seq_len - 2 residues."""
    return random_sequences(1, seq_len, seed=DMS_WILDTYPE_SEED)[0][1:-1].copy()


def dms_variant(wildtype: np.ndarray, p: int) -> np.ndarray:
    """Tokens of the variant with residue p (0-based) replaced by <mask>."""
    s = np.concatenate([[0], wildtype, [2]]).astype(np.int32)
    s[1 + p] = MASK_ID
    return s


def workload_sequences(c: dict, batch: int, seed_offset: int = 0, first: int = 0) -> list[np.ndarray]:
    """Token sequences of a benchmark batch. Fixed- and uniform-length batches draw from seed
    1000 + seed_offset (lengths from 3000 + seed_offset); a scan's batch is the single-<mask>
    variants first .. first + batch - 1 of the wild type."""
    if c["dms"]:
        wt = dms_wildtype(c["seq_len"])
        n = len(wt)
        return [dms_variant(wt, p % n) for p in range(first, first + batch)]
    if c["lengths"] == "uniform":
        rng = np.random.default_rng(3000 + seed_offset)
        lens = rng.integers(c["min_len"], c["seq_len"] + 1, size=batch)
        return random_sequences(batch, lens, seed=1000 + seed_offset)
    return random_sequences(batch, c["seq_len"], seed=1000 + seed_offset)
