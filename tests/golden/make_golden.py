"""Generate the golden fixtures that pin the CPU oracle to an independent ESM-2 implementation.

Run once, in a container that has the reference checkout and HF ``transformers``:

    python tests/golden/make_golden.py /path/to/codon-infer

What it does:
  * reads codon-infer's bundled real ESM-2 8M weights, ``esm2_8m_weights.bin`` (grouped_canonical_v1
    FP32, no header; layout in EsmWeights::from_file, src/lib.rs:369-395, written by
    scripts/export_weights.py:68-120);
  * reads the 8M contact-regression constants from ``src/contact_heads.rs:5-22`` (Meta's trained
    ``esm.contact_head.regression`` for esm2_t6_8M_UR50D);
  * builds HF ``EsmForMaskedLM`` offline from that config, loads the weights by state-dict mapping,
    and runs three sequences (the test_peptidase.fasta record, the masked "MCMP*TTD" of
    src/lib.rs:6966, and the 36-residue 1CHL peptide of src/lib.rs:8519);
  * writes ``esm2_8m_hf.npz``: per sequence its tokens, logits [L,33], final hidden state
    (emb_layer_norm_after output) [L,320] and contact probabilities [L-2, L-2], plus the contact
    head weights. The weights file itself (30 MB) is not committed; tests that need it skip when
    it is absent.

The codon-infer documentation reports cos >= 0.999999 between its FP32 forward and HF for the 8M
model (docs/benchmarks_v1.6.0.md:18), which is the bar these fixtures let the oracle be held to.
"""
from __future__ import annotations

import os
import re
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "esm2_8m_hf.npz"

D, F, NL, H, V = 320, 1280, 6, 20, 33
SEQUENCES = {
    "peptidase": "AQVGDSGGPMLCNGQLQGVTSWGYVCAQPEYPGVYTEVS",
    "masked": "MCMP*TTD",
    "chl": "MCMPCFTTDHQMARKCDDCCGGKGRGKCYGPQCLCR",
}
AA_IDS = {c: i for i, c in enumerate("LAGVSERTIDPKQNFYMHWC", start=4)}
AA_IDS.update({"X": 24, "B": 25, "U": 26, "Z": 27, "O": 28, ".": 29, "-": 30, "*": 32})


def encode(seq: str) -> list[int]:
    """Tokenizer::encode, src/lib.rs:6511-6521."""
    return [0] + [AA_IDS.get(c, 3) for c in seq] + [2]


def read_grouped(path: Path) -> dict[str, np.ndarray]:
    raw = np.fromfile(path, dtype="<f4")
    sizes = [
        ("tok_emb", V * D), ("ln1_w", NL * D), ("ln1_b", NL * D), ("wq", NL * D * D), ("bq", NL * D),
        ("wk", NL * D * D), ("bk", NL * D), ("wv", NL * D * D), ("bv", NL * D), ("wo", NL * D * D),
        ("bo", NL * D), ("ln2_w", NL * D), ("ln2_b", NL * D), ("fc1_w", NL * F * D), ("fc1_b", NL * F),
        ("fc2_w", NL * D * F), ("fc2_b", NL * D), ("lnf_w", D), ("lnf_b", D),
        ("classifier", 3 * D + D * D + V * D + V),
    ]
    out, off = {}, 0
    for name, n in sizes:
        out[name] = raw[off:off + n].copy()
        off += n
    assert off == raw.size, (off, raw.size)
    return out


def read_contact_head_8m(path: Path) -> tuple[np.ndarray, float]:
    text = path.read_text()
    bias = float(re.search(r"CONTACT_HEAD_8M_BIAS: f32 = ([-+0-9.eE]+)_f32", text).group(1))
    body = re.search(r"CONTACT_HEAD_8M_WEIGHT: \[f32; 120\] = \[(.*?)\];", text, re.S).group(1)
    w = np.array([float(v) for v in re.findall(r"([-+0-9.eE]+)_f32", body)], dtype=np.float32)
    assert w.size == NL * H
    return w, bias


def main(ref_root: Path) -> None:
    import torch
    from transformers import EsmConfig, EsmForMaskedLM

    t = read_grouped(ref_root / "esm2_8m_weights.bin")
    cw, cb = read_contact_head_8m(ref_root / "src" / "contact_heads.rs")

    cfg = EsmConfig(vocab_size=V, hidden_size=D, num_hidden_layers=NL, num_attention_heads=H,
                    intermediate_size=F, position_embedding_type="rotary", token_dropout=True,
                    emb_layer_norm_before=False, mask_token_id=32, pad_token_id=1, layer_norm_eps=1e-5,
                    hidden_act="gelu", max_position_embeddings=1026)
    model = EsmForMaskedLM(cfg).eval().float()
    sd = model.state_dict()

    def put(key, arr, shape):
        sd[key] = torch.from_numpy(np.asarray(arr, dtype=np.float32).reshape(shape).copy())

    put("esm.embeddings.word_embeddings.weight", t["tok_emb"], (V, D))
    for l in range(NL):
        p = f"esm.encoder.layer.{l}."
        sl = slice(l * D * D, (l + 1) * D * D)
        sv = slice(l * D, (l + 1) * D)
        put(p + "attention.self.query.weight", t["wq"][sl], (D, D))
        put(p + "attention.self.query.bias", t["bq"][sv], (D,))
        put(p + "attention.self.key.weight", t["wk"][sl], (D, D))
        put(p + "attention.self.key.bias", t["bk"][sv], (D,))
        put(p + "attention.self.value.weight", t["wv"][sl], (D, D))
        put(p + "attention.self.value.bias", t["bv"][sv], (D,))
        put(p + "attention.output.dense.weight", t["wo"][sl], (D, D))
        put(p + "attention.output.dense.bias", t["bo"][sv], (D,))
        put(p + "attention.LayerNorm.weight", t["ln1_w"][sv], (D,))
        put(p + "attention.LayerNorm.bias", t["ln1_b"][sv], (D,))
        put(p + "intermediate.dense.weight", t["fc1_w"][l * F * D:(l + 1) * F * D], (F, D))
        put(p + "intermediate.dense.bias", t["fc1_b"][l * F:(l + 1) * F], (F,))
        put(p + "output.dense.weight", t["fc2_w"][l * D * F:(l + 1) * D * F], (D, F))
        put(p + "output.dense.bias", t["fc2_b"][sv], (D,))
        put(p + "LayerNorm.weight", t["ln2_w"][sv], (D,))
        put(p + "LayerNorm.bias", t["ln2_b"][sv], (D,))
    put("esm.encoder.emb_layer_norm_after.weight", t["lnf_w"], (D,))
    put("esm.encoder.emb_layer_norm_after.bias", t["lnf_b"], (D,))
    c = t["classifier"]  # [lm_ln_w d | lm_ln_b d | dense_w d*d | dense_b d | dec_w 33*d | dec_b 33]
    put("lm_head.layer_norm.weight", c[0:D], (D,))
    put("lm_head.layer_norm.bias", c[D:2 * D], (D,))
    put("lm_head.dense.weight", c[2 * D:2 * D + D * D], (D, D))
    put("lm_head.dense.bias", c[2 * D + D * D:3 * D + D * D], (D,))
    put("lm_head.decoder.weight", c[3 * D + D * D:3 * D + D * D + V * D], (V, D))
    put("lm_head.bias", c[3 * D + D * D + V * D:], (V,))
    put("esm.contact_head.regression.weight", cw, (1, NL * H))
    put("esm.contact_head.regression.bias", [cb], (1,))
    model.load_state_dict(sd)
    model.set_attn_implementation("eager")

    fixtures = {"contact_w": cw, "contact_b": np.float32(cb)}
    with torch.no_grad():
        for name, seq in SEQUENCES.items():
            toks = torch.tensor([encode(seq)], dtype=torch.long)
            out = model(input_ids=toks, output_hidden_states=True)
            contacts = model.esm.predict_contacts(toks, torch.ones_like(toks))
            fixtures[f"{name}_tokens"] = toks[0].numpy().astype(np.int32)
            fixtures[f"{name}_logits"] = out.logits[0].numpy().astype(np.float32)
            fixtures[f"{name}_hidden"] = out.hidden_states[-1][0].numpy().astype(np.float32)
            fixtures[f"{name}_contacts"] = contacts[0].numpy().astype(np.float32)
    np.savez_compressed(OUT, **fixtures)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    # The codon-infer checkout: the argument, else CODON_INFER_REF, else a sibling of this repository.
    default = os.environ.get("CODON_INFER_REF", str(Path(__file__).resolve().parents[3] / "reference"))
    main(Path(sys.argv[1] if len(sys.argv) > 1 else default))
