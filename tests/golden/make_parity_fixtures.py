"""Generate oracle fixtures at the benchmark's own shapes, for the GPU parity tests.

    python tests/golden/make_parity_fixtures.py [c3] [c4] [c5]     (default: all three)

The CPU oracle (oracle/esm_oracle.cpp, the restatement of codon-infer's forward) runs the very
inputs the benchmark feeds the GPU: the seeded random-init weights of each model
(synth.synth_fp32_tensors, seed 0), quantized by the oracle's bit-exact quantizers, and the first
sequences of the benchmark batch (synth.workload_sequences). At these sizes the oracle takes
minutes (3B at L = 4096: about a quarter of an hour on 8 cores), so the GPU tests compare against
these committed outputs instead of running it:

  parity_c4.npz  ESM-2 650M Q4_0, 33 layers: sequences 0 and 1 of the 64 x 1024 batch, logits.
  parity_c5.npz  ESM-2 3B Q8_0, 36 layers, contact head on: sequence 0 of the 8 x 4096 batch,
                 logits [4096, 33]; contact probabilities [4094, 4094] as a seeded sample of
                 entries, the two corner blocks whole, and every row's sum.
  parity_c3.npz  ESM-2 150M FP32 masked-marginal scan of the 300-residue wild type: 16 positions
                 spread over the sequence, their [20] deltas and entropy (run_pipeline_dms_with_mode,
                 src/pipeline.rs:109-175), and the full logits of those 16 variants.

Nothing here needs the reference checkout or a GPU.
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (ROOT / "codon-infer_b200", ROOT / "oracle"):
    sys.path.insert(0, str(p))

import oracle  # noqa: E402
import synth  # noqa: E402

C5_SAMPLE = 200_000       # sampled (i, j) entries of the 4094 x 4094 contact map
C5_SAMPLE_SEED = 4242
C5_CORNER = 192           # leading and trailing corner blocks kept whole
C3_POSITIONS = (0, 1, 2, 37, 75, 112, 149, 150, 187, 224, 250, 262, 280, 297, 298, 299)


def c5_sample_indices(n: int) -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(C5_SAMPLE_SEED)
    return rng.integers(0, n, size=C5_SAMPLE), rng.integers(0, n, size=C5_SAMPLE)


def _weights(c: dict):
    cfg = synth.preset(c["arch"])
    t = oracle.quantize_tensors(synth.synth_fp32_tensors(cfg, seed=synth.WEIGHT_SEED), c["dtype"])
    return cfg, t


def make_c4() -> None:
    c = synth.CONFIGS["c4"]
    cfg, t = _weights(c)
    seqs = synth.workload_sequences(c, 2)
    logits = []
    for s in seqs:
        t0 = time.time()
        logits.append(oracle.forward(cfg, c["dtype"], t, s)["logits"])
        print(f"c4 sequence: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(HERE / "parity_c4.npz", tokens=np.stack(seqs), logits=np.stack(logits))


def make_c5() -> None:
    c = synth.CONFIGS["c5"]
    cfg, t = _weights(c)
    s = synth.workload_sequences(c, 1)[0]
    cw = synth.contact_head(cfg)
    t0 = time.time()
    out = oracle.forward(cfg, c["dtype"], t, s, contact_w=cw, contact_b=0.0)
    print(f"c5 sequence: {time.time() - t0:.1f} s", flush=True)
    cm = out["contacts"]
    n = cm.shape[0]
    ii, jj = c5_sample_indices(n)
    k = C5_CORNER
    np.savez_compressed(
        HERE / "parity_c5.npz", tokens=s, logits=out["logits"], contact_sample=cm[ii, jj],
        contact_head=cm[:k, :k], contact_tail=cm[n - k:, n - k:],
        contact_row_sums=cm.astype(np.float64).sum(1).astype(np.float32))


def make_c3() -> None:
    c = synth.CONFIGS["c3"]
    cfg, t = _weights(c)
    wt = synth.dms_wildtype(c["seq_len"])
    deltas = np.zeros((len(C3_POSITIONS), 20), np.float32)
    ent = np.zeros(len(C3_POSITIONS), np.float32)
    full = []
    for k, p in enumerate(C3_POSITIONS):
        toks = synth.dms_variant(wt, p)
        lg = oracle.forward(cfg, c["dtype"], t, toks)["logits"]
        deltas[k], ent[k] = oracle.dms_scores(lg[p + 1], int(wt[p]))
        full.append(lg)
    np.savez_compressed(HERE / "parity_c3.npz", wildtype=wt, positions=np.array(C3_POSITIONS, np.int32),
                        deltas=deltas, entropy=ent, variant_logits=np.stack(full))


if __name__ == "__main__":
    which = sys.argv[1:] or ["c3", "c4", "c5"]
    for w in which:
        {"c3": make_c3, "c4": make_c4, "c5": make_c5}[w]()
        print(f"{w} written", flush=True)
