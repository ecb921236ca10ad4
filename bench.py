"""Throughput benchmark of the B200 ESM-2 encoder forward (codon-infer's hot path).

Workload (default): ESM-2 650M with Q4_0 weights (random-init N(0, 0.02), quantized by the
bit-exact BlockQ4_0 quantizer), 64 sequences x L = 1024 tokens of uniform-random residues per GPU,
logits [64, 1024, 33] out. Metric: residues/s over the whole job (tokens incl. <cls>/<eos>).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU, NCCL)

Scaling is weak: every rank runs its own 64-sequence batch (sequences are independent), and the
only collective is the gather of the logits to all ranks after each forward. `value` times
device-resident inputs with CUDA events; `e2e` times the host API (esm_forward: pinned host
tokens in, host logits out) with the copies inside the timed region. --impl reference times the
CPU restatement of the reference forward (the reference crate is Rust and cannot be built in this
image) on the host cores, one 1024-token sequence per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "codon-infer_b200"))

UNIT = "residues/s"
# The benchmark configurations (tokens include <cls>/<eos>). c4 is the headline and the default.
CONFIGS = {
    "c1": dict(arch=0, dtype=0, batch=1, lengths="fixed", seq_len=128, contacts=True, dms=False,
               desc="ESM-2 8M FP32 forward, 1 x L=128, contact head on"),
    "c2": dict(arch=1, dtype=1, batch=32, lengths="uniform", seq_len=512, min_len=64, contacts=False, dms=False,
               desc="ESM-2 35M Q8_0 forward, 32 sequences with L in U[64, 512], right-padded"),
    "c3": dict(arch=2, dtype=0, batch=300, lengths="fixed", seq_len=302, contacts=False, dms=True,
               desc="ESM-2 150M FP32 masked-marginal scan: 300 single-<mask> variants of a 300-residue wild type"),
    "c4": dict(arch=3, dtype=2, batch=64, lengths="fixed", seq_len=1024, contacts=False, dms=False,
               desc="ESM-2 650M Q4_0 forward, 64 x L=1024 per GPU, logits out"),
    "c5": dict(arch=4, dtype=1, batch=8, lengths="fixed", seq_len=4096, contacts=True, dms=False,
               desc="ESM-2 3B Q8_0 forward, 8 x L=4096 per GPU, contact maps on"),
}


def metric_name(cfg_name, c, batch):
    return {
        "c4": "residues/sec, ESM-2 650M Q4_0 forward (64 x L=1024 per GPU)",
    }.get(cfg_name, f"residues/sec, {c['desc']}")


def workload_sequences(esm, c, batch, rank):
    """Token sequences of one rank's batch (seeded per rank)."""
    if c["dms"]:
        wt = esm.random_sequences(1, c["seq_len"], seed=2000)[0]
        out = []
        for p in range(batch):
            v = wt.copy()
            v[1 + (p % (c["seq_len"] - 2))] = esm.MASK_ID
            out.append(v)
        return out
    if c["lengths"] == "uniform":
        rng = np.random.default_rng(3000 + rank)
        lens = rng.integers(c["min_len"], c["seq_len"] + 1, size=batch)
        return esm.random_sequences(batch, lens, seed=1000 + rank)
    return esm.random_sequences(batch, c["seq_len"], seed=1000 + rank)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), d.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = gpu_indices
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.gpus is not None:
            cmd += ["-i", ",".join(str(g) for g in self.gpus)]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if not vis:
        return local_rank
    ids = [v.strip() for v in vis.split(",")]
    if local_rank < len(ids) and ids[local_rank].isdigit():
        return int(ids[local_rank])
    return None


def cpu_forward_rate(cfg, dtype, tensors, seq_len, seed, threads):
    """Oracle forward of one sequence: residues/s on `threads` host threads."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    import esm_b200 as esm
    s = esm.random_sequences(1, seq_len, seed=seed)[0]
    t0 = time.perf_counter()
    oracle.forward(cfg, dtype, tensors, s, n_threads=threads)
    return seq_len / (time.perf_counter() - t0)


def run_reference(args):
    """CPU arm: the restated reference forward on the host cores, one sequence per step."""
    import esm_b200 as esm
    rank = int(os.environ.get("RANK", "0"))
    c = CONFIGS[args.config]
    batch = args.batch or c["batch"]
    if rank != 0:
        return
    cfg = esm.EsmConfig.preset(c["arch"])
    t = esm.quantize_tensors(esm.synth_fp32_tensors(cfg, seed=0), c["dtype"])
    threads = os.cpu_count() or 1
    seq_len = c["seq_len"]
    for w in range(args.warmup):
        cpu_forward_rate(cfg, c["dtype"], t, seq_len, 1000 + w, threads)
    t0 = time.perf_counter()
    for k in range(args.steps):
        cpu_forward_rate(cfg, c["dtype"], t, seq_len, 2000 + k, threads)
    dt = time.perf_counter() - t0
    value = args.steps * seq_len / dt
    sample = f"1 sequence x L={seq_len} per step (of the {batch}-sequence per-GPU batch), all layers"
    line = {
        "impl": "reference", "metric": metric_name(args.config, c, batch), "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded uniform residues, random-init N(0,0.02) weights)",
        "config": {"workload": c["desc"] + f" (CPU: {seq_len}-token sequences)", "seq_len": seq_len},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist
    import esm_b200 as esm

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    c = CONFIGS[args.config]
    arch, dtype, seq_len = c["arch"], c["dtype"], c["seq_len"]
    batch = args.batch or c["batch"]  # a smaller per-GPU batch is for profiler captures only
    cfg = esm.EsmConfig.preset(arch)
    t32 = esm.synth_fp32_tensors(cfg, seed=0)
    tensors = esm.quantize_tensors(t32, dtype)
    del t32
    model = esm.Model(local)
    model.load_tensors(cfg, dtype, tensors)
    if c["contacts"]:
        cw = (np.random.default_rng(7).standard_normal(cfg.n_layers * cfg.n_heads) * 0.1).astype(np.float32)
        model.set_contact_head(cw, 0.0)
    seqs = workload_sequences(esm, c, batch, rank)
    lengths = np.array([len(q) for q in seqs], dtype=np.int32)
    T = int(lengths.sum())
    Lmax = int(lengths.max())
    model.reserve(T, batch, Lmax, contacts=c["contacts"])
    host_tokens = np.zeros((batch, Lmax), dtype=np.int32)
    for i, q in enumerate(seqs):
        host_tokens[i, : len(q)] = q
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    d_tokens = torch.from_numpy(np.concatenate(seqs).astype(np.int32)).to(dev)
    d_logits = torch.empty(T, cfg.vocab_size, device=dev)
    n_map = int(sum(max(int(L) - 2, 0) ** 2 for L in lengths))
    d_contacts = torch.empty(max(n_map, 1), device=dev) if c["contacts"] else None
    gathered = torch.empty(world * T, cfg.vocab_size, device=dev) if world > 1 else None
    # A dedicated stream: the forward is enqueued on it and the CUDA events are recorded on it.
    # (torch's default stream has handle 0, which the C ABI reads as "the context's own stream".)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    def step():
        model.forward_device(d_tokens, cu, d_logits, d_contacts=d_contacts, stream=stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered, d_logits)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    model.check_device()

    sampler = ClockSampler([physical_gpu(local)] if physical_gpu(local) is not None else None)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    model.check_device()
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T * args.steps / (ms / 1000.0)
    if ms <= 0.0:
        raise SystemExit("timed region is empty: the forward did not run on the timed stream")

    # End to end through the host API: pinned host tokens in, results back to host every step.
    host_tok = torch.from_numpy(host_tokens).pin_memory()
    host_logits = torch.empty(batch, Lmax, cfg.vocab_size, dtype=torch.float32).pin_memory()
    tok_np, log_np = host_tok.numpy(), host_logits.numpy()
    host_con, con_np = None, None
    if c["contacts"]:
        np_ = max(Lmax - 2, 0)
        host_con = torch.empty(batch, np_, np_, dtype=torch.float32).pin_memory()
        con_np = host_con.numpy()
    d2h = batch * Lmax * cfg.vocab_size * 4 + (batch * max(Lmax - 2, 0) ** 2 * 4 if c["contacts"] else 0)

    def e2e_step():
        model.forward(tok_np, lengths=lengths, logits_out=log_np, want_contacts=c["contacts"], contacts_out=con_np)

    e2e_steps = max(1, min(args.steps, 5))
    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e_value = world * T * e2e_steps / e2e_s
    dms_rate = None
    if c["dms"]:
        # The public mutational-scan call on the same wild type: masked variants built, run and
        # scored inside the library, scores [n, 20] back to host.
        residues = esm.random_sequences(1, c["seq_len"], seed=2000)[0][1:-1]  # the wild type
        model.dms_masked_marginal(residues)
        t0 = time.perf_counter()
        model.dms_masked_marginal(residues)
        dms_rate = len(residues) / (time.perf_counter() - t0)

    # Per-kernel-class device time of one step (CUDA events around each launch, its own stream).
    model.profile_enable(True)
    model.forward_device(d_tokens, cu, d_logits, d_contacts=d_contacts, stream=stream)
    torch.cuda.synchronize(dev)
    prof = model.profile_read()
    model.profile_enable(False)
    launches_per_step = sum(v["launches"] for v in prof.values()) + 1  # + sequence setup

    burst, sustained, hbm, peak_kind = measured_peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0
    traffic = None
    tp = ROOT / "profiles" / "gemm_tc_650m_q4_traffic.txt"
    if tp.exists():
        for ln in tp.read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch:"):
                traffic = float(ln.split(":", 1)[1])
    roofline = {
        "kernel": "gemm_tc_kernel (tcgen05 projections: QKV, O, fc1, fc2, LM dense)",
        "bound": "tensor", "achieved": gemm_tflops, "peak": sustained, "unit": "TFLOP/s",
        "frac": gemm_tflops / sustained if sustained else None, "traffic": traffic,
        "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside the step)",
        "step_share": g["ms"] / sum(v["ms"] for v in prof.values()),
    }
    breakdown = {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                     "tflops": round(v["flops"] / (v["ms"] / 1000) / 1e12, 1) if v["ms"] > 0 and v["flops"] else None,
                     "gbs": round(v["bytes"] / (v["ms"] / 1000) / 1e9, 1) if v["ms"] > 0 and v["bytes"] else None}
                 for k, v in prof.items()}
    total_flops = sum(v["flops"] for v in prof.values())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate = cpu_forward_rate(cfg, dtype, tensors, seq_len, 4242, threads)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"1 sequence x L={seq_len}, full {cfg.n_layers}-layer forward "
                         "(CPU restatement of the reference)"}

    if rank == 0:
        line = {
            "metric": metric_name(args.config, c, batch), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded uniform residues, random-init N(0,0.02) weights)",
            "config": {"workload": c["desc"], "batch_per_gpu": batch, "seq_len": Lmax, "tokens_per_gpu": T,
                       "arithmetic": "f16 tensor-core operands, f32 accumulate; "
                                     + ["FP32", "Q8_0", "Q4_0"][dtype] + " weights dequantised per layer",
                       "parallelism": f"sequence-sharded x{world}, logits all-gather",
                       "l2": "no flush: the per-step working set (activations, weights) exceeds the 126 MB L2"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(host_tokens.nbytes + 4 * batch),
                    "d2h_bytes_per_step": int(d2h), "steps": e2e_steps},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roofline,
            "achieved_model_tflops": total_flops / (ms / args.steps / 1000.0) / 1e12,
            "kernel_breakdown_ms_per_step": breakdown,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if dms_rate is not None:
            line["dms_variants_per_s"] = dms_rate
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c4",
                    help="c4 (headline, default): 650M Q4_0 64 x 1024; c1/c2/c3/c5: the other benchmark configs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
