"""Throughput benchmark of the B200 ESM-2 encoder forward (codon-infer's hot path).

Workload (default, c4): ESM-2 650M with Q4_0 weights (random-init N(0, 0.02), quantized by the
bit-exact BlockQ4_0 quantizer), 64 sequences x L = 1024 tokens of uniform-random residues per GPU,
logits [64, 1024, 33] out. Metric: residues/s over the whole job (tokens incl. <cls>/<eos>).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|vendor] [--config c1..c5]
  torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU, NCCL)

Scaling. Forward configurations (c1, c2, c4, c5) are weak-scaled in `value`: every rank runs its
own batch (sequences are independent) and the only collective is the gather of the logits after
each forward. With N > 1 the line also carries `strong_scaling`: the one 64 x 1024 batch of c4 (the
configuration's own "sequences are sharded across 1/2/4/8 GPUs") split into N cost-balanced
contiguous blocks (esm_partition), each rank running its block, then the logits gathered. The
mutational scan (c3) is strong-scaled: the 300 masked variants of the one wild type are split
into N contiguous blocks and only the per-variant rows cross between GPUs.

`value` times device-resident inputs with CUDA events; `e2e` times the host API (esm_forward, or
esm_dms_masked_marginal_range for the scan: host buffers in and out) with the copies inside the
timed region. --impl reference times the CPU restatement of the reference forward (the reference
crate is Rust and cannot be built in this image) on the host cores, one sequence per step; that
arm loads only the oracle library. --impl vendor times the same projections and attention with
cuBLAS and cuDNN (a yardstick for the kernels, not a forward; see run_vendor).
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

import synth  # noqa: E402  (numpy only: no native library is loaded by this import)

UNIT = "residues/s"
CONFIGS = synth.CONFIGS
_json_out = sys.stdout


def emit(line: dict) -> None:
    _json_out.write(json.dumps(line) + "\n")
    _json_out.flush()


def metric_name(cfg_name, c):
    return {
        "c4": "residues/sec, ESM-2 650M Q4_0 forward (64 x L=1024 per GPU)",
    }.get(cfg_name, f"residues/sec, {c['desc']}")


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


def oracle_module():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    return oracle


def cpu_sample(c, k):
    """The k-th CPU sample sequence of a workload: a masked variant of the scan (c3), a sequence of
    the ragged batch (c2), else one full-length sequence, capped at 1024 tokens (c5's 4096-token
    sequences would take minutes each on the host)."""
    if c["dms"]:
        return synth.workload_sequences(c, 1, first=37 * k)[0]
    if c["lengths"] == "uniform":
        seqs = synth.workload_sequences(c, c["batch"])
        return seqs[k % len(seqs)]
    return synth.random_sequences(1, min(c["seq_len"], 1024), seed=5000 + k)[0]


def cpu_rate(oracle, cfg, c, tensors, k0, n, threads):
    """Oracle forwards of n sample sequences: (residues/s, residues)."""
    res = 0
    t0 = time.perf_counter()
    for k in range(k0, k0 + n):
        s = cpu_sample(c, k)
        cw = synth.contact_head(cfg) if c["contacts"] else None
        oracle.forward(cfg, c["dtype"], tensors, s, n_threads=threads, contact_w=cw, contact_b=0.0)
        res += len(s)
    return res / (time.perf_counter() - t0), res


def cpu_weights(oracle, c):
    cfg = synth.preset(c["arch"])
    t = oracle.quantize_tensors(synth.synth_fp32_tensors(cfg, seed=synth.WEIGHT_SEED), c["dtype"])
    return cfg, t


def cpu_sample_desc(c, cfg):
    L = min(c["seq_len"], 1024)
    what = {True: f"one masked variant of the {c['seq_len']}-token scan",
            False: f"one {L}-token sequence" if c["lengths"] == "fixed" else "one sequence of the ragged batch"}[c["dms"]]
    heads = ", contact head on" if c["contacts"] else ""
    return f"{what} per step, full {cfg.n_layers}-layer forward{heads} (CPU restatement of the reference)"


def run_reference(args):
    """CPU arm: the restated reference forward on the host cores, one sequence per step. Loads the
    oracle library only (weights quantized by the oracle's own quantizers)."""
    rank = int(os.environ.get("RANK", "0"))
    c = CONFIGS[args.config]
    if rank != 0:
        return
    oracle = oracle_module()
    cfg, t = cpu_weights(oracle, c)
    threads = os.cpu_count() or 1
    cpu_rate(oracle, cfg, c, t, 0, args.warmup, threads)
    t0 = time.perf_counter()
    _, res = cpu_rate(oracle, cfg, c, t, 100, args.steps, threads)
    dt = time.perf_counter() - t0
    value = res / dt
    line = {
        "impl": "reference", "metric": metric_name(args.config, c), "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong" if c["dms"] else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded uniform residues, random-init N(0,0.02) weights)",
        "config": {"workload": c["desc"], "cpu_sample": cpu_sample_desc(c, cfg)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": cpu_sample_desc(c, cfg)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def timed_loop(step, steps, stream, dev, world, dist):
    """Runs `steps` steps between a barrier + synchronize on both sides; CUDA events on the
    launching stream; max over ranks (ms)."""
    import torch
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def max_over_ranks(x, dev, world, dist):
    import torch
    if world == 1:
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class PackedBatch:
    """A batch on the device in the packed layout, with a gather buffer of `rows_max` rows per rank
    for the outputs that cross between GPUs."""

    def __init__(self, torch, dev, seqs, vocab, contacts, world, rows_max):
        self.seqs = seqs
        self.lengths = np.array([len(q) for q in seqs], dtype=np.int32)
        self.T = int(self.lengths.sum())
        self.cu = np.concatenate([[0], np.cumsum(self.lengths)]).astype(np.int32)
        self.tokens = torch.from_numpy(np.concatenate(seqs).astype(np.int32)).to(dev) if seqs else None
        self.logits = torch.zeros(max(self.T, rows_max, 1), vocab, device=dev)
        n_map = int(sum(max(int(L) - 2, 0) ** 2 for L in self.lengths))
        self.contacts = torch.empty(max(n_map, 1), device=dev) if contacts else None
        self.rows_max = rows_max
        self.gathered = torch.empty(world * rows_max, vocab, device=dev) if world > 1 else None


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
    arch, dtype = c["arch"], c["dtype"]
    batch = args.batch or c["batch"]  # a smaller batch is for profiler captures only
    cfg = esm.EsmConfig.preset(arch)
    t32 = esm.synth_fp32_tensors(cfg, seed=synth.WEIGHT_SEED)
    tensors = esm.quantize_tensors(t32, dtype)
    del t32
    model = esm.Model(local)
    model.load_tensors(cfg, dtype, tensors)
    if c["contacts"]:
        model.set_contact_head(synth.contact_head(cfg), 0.0)
    V = cfg.vocab_size

    if c["dms"]:
        # Strong scaling of the scan: this rank's contiguous block of the masked variants.
        lens_all = [c["seq_len"]] * batch
        blocks = esm.partition(lens_all, world, cfg.dim, cfg.hidden_dim)
        mine = blocks[rank]
        seqs = synth.workload_sequences(c, len(mine), first=mine.start) if len(mine) else []
        scaling = "strong"
        total_tokens = batch * c["seq_len"]
        rows_max = max(len(b) for b in blocks)  # one masked row per variant crosses between GPUs
    else:
        seqs = synth.workload_sequences(c, batch, seed_offset=rank)
        scaling = "weak"
        total_tokens = None
        rows_max = sum(len(q) for q in seqs)
    pb = PackedBatch(torch, dev, seqs, V, c["contacts"], world, rows_max)
    Lmax = int(pb.lengths.max()) if len(seqs) else c["seq_len"]
    model.reserve(max(pb.T, c["seq_len"]), max(len(seqs), 1), Lmax, contacts=c["contacts"])
    if c["dms"]:
        mask_rows = torch.from_numpy((pb.cu[:-1] + 1 + (np.arange(len(seqs)) + mine.start) % (c["seq_len"] - 2))
                                     .astype(np.int64)).to(dev)
        sel = torch.zeros(rows_max, V, device=dev)
    # A dedicated stream: the forward is enqueued on it and the CUDA events are recorded on it.
    # (torch's default stream has handle 0, which the C ABI reads as "the context's own stream".)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    def step():
        if pb.T:
            model.forward_device(pb.tokens, pb.cu, pb.logits, d_contacts=pb.contacts, stream=stream)
        if world > 1:
            if c["dms"]:
                if pb.T:
                    sel[: len(seqs)] = pb.logits.index_select(0, mask_rows)
                dist.all_gather_into_tensor(pb.gathered, sel)
            else:
                dist.all_gather_into_tensor(pb.gathered, pb.logits[: pb.rows_max])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    model.check_device()

    sampler = ClockSampler([physical_gpu(local)] if physical_gpu(local) is not None else None)
    sampler.start()
    time.sleep(0.3)
    ms = timed_loop(step, args.steps, stream, dev, world, dist)
    clocks = sampler.stop()
    model.check_device()
    if ms <= 0.0:
        raise SystemExit("timed region is empty: the forward did not run on the timed stream")
    if total_tokens is None:  # weak scaling: the tokens of every rank's own batch
        total_tokens = pb.T
        if world > 1:
            tt = torch.tensor([pb.T], device=dev, dtype=torch.int64)
            dist.all_reduce(tt)
            total_tokens = int(tt.item())
    value = total_tokens * args.steps / (ms / 1000.0)

    # Strong scaling of the headline batch (N > 1): the one batch split across the ranks.
    strong = None
    if world > 1 and not c["dms"]:
        all_seqs = synth.workload_sequences(c, batch, seed_offset=0)
        parts = esm.partition([len(q) for q in all_seqs], world, cfg.dim, cfg.hidden_dim)
        rows = [sum(len(all_seqs[i]) for i in p) for p in parts]
        sb = PackedBatch(torch, dev, [all_seqs[i] for i in parts[rank]], V, c["contacts"], world, max(rows))

        def sstep():
            if sb.T:
                model.forward_device(sb.tokens, sb.cu, sb.logits, d_contacts=sb.contacts, stream=stream)
            dist.all_gather_into_tensor(sb.gathered, sb.logits[: sb.rows_max])

        for _ in range(args.warmup):
            sstep()
        torch.cuda.synchronize(dev)
        sms = timed_loop(sstep, args.steps, stream, dev, world, dist)
        tot = sum(rows)
        strong = {"value": tot * args.steps / (sms / 1000.0), "unit": UNIT, "ms_per_step": sms / args.steps,
                  "sequences_total": len(all_seqs), "tokens_total": tot,
                  "sequences_per_gpu": [len(p) for p in parts], "scaling": "strong",
                  "collective": "NCCL all_gather of the logits after each forward"}
        del sb
        model.check_device()

    # End to end through the host API: host buffers in, results back to host every step.
    e2e_steps = max(1, min(args.steps, 5))
    if c["dms"]:
        wt = synth.dms_wildtype(c["seq_len"])
        scores = torch.zeros(rows_max, 21, device=dev)
        gathered_scores = torch.empty(world * rows_max, 21, device=dev) if world > 1 else None

        def e2e_step():
            if len(mine):
                d, e = model.dms_masked_marginal_range(wt, mine.start, mine.stop)
                scores[: len(mine), :20] = torch.from_numpy(d)
                scores[: len(mine), 20] = torch.from_numpy(e)
            if world > 1:
                dist.all_gather_into_tensor(gathered_scores, scores)
                gathered_scores.cpu()
        h2d = int(wt.nbytes)
        d2h = int(len(mine) * 21 * 4 * (world if world > 1 else 1))
    else:
        host_tokens = np.zeros((len(seqs), Lmax), dtype=np.int32)
        for i, q in enumerate(seqs):
            host_tokens[i, : len(q)] = q
        host_tok = torch.from_numpy(host_tokens).pin_memory()
        host_logits = torch.empty(len(seqs), Lmax, V, dtype=torch.float32).pin_memory()
        tok_np, log_np = host_tok.numpy(), host_logits.numpy()
        con_np = None
        if c["contacts"]:
            np_ = max(Lmax - 2, 0)
            con_np = torch.empty(len(seqs), np_, np_, dtype=torch.float32).pin_memory().numpy()

        def e2e_step():
            model.forward(tok_np, lengths=pb.lengths, logits_out=log_np, want_contacts=c["contacts"],
                          contacts_out=con_np)
        h2d = int(host_tokens.nbytes + 4 * len(seqs))
        d2h = len(seqs) * Lmax * V * 4 + (len(seqs) * max(Lmax - 2, 0) ** 2 * 4 if c["contacts"] else 0)
    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = max_over_ranks(time.perf_counter() - t0, dev, world, dist)
    e2e_value = total_tokens * e2e_steps / e2e_s

    # Per-kernel-class device time of one step (CUDA events around each launch, its own stream).
    model.profile_enable(True)
    if pb.T:
        model.forward_device(pb.tokens, pb.cu, pb.logits, d_contacts=pb.contacts, stream=stream)
    torch.cuda.synchronize(dev)
    prof = model.profile_read()
    model.profile_enable(False)
    launches_per_step = sum(v["launches"] for v in prof.values()) + 1  # + sequence setup

    burst, sustained, hbm, peak_kind = measured_peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0
    traffic = None
    tp = ROOT / "profiles" / "gemm_tc_650m_q4_traffic.txt"
    if tp.exists() and args.config == "c4":
        for ln in tp.read_text().splitlines():
            if ln.startswith("dram_bytes_per_launch:"):
                traffic = float(ln.split(":", 1)[1])
    tot_ms = sum(v["ms"] for v in prof.values())
    roofline = {
        "kernel": "gemm_tc_kernel (tcgen05 projections: QKV, O, fc1, fc2, LM dense)",
        "bound": "tensor", "achieved": gemm_tflops, "peak": sustained, "unit": "TFLOP/s",
        "frac": gemm_tflops / sustained if sustained else None, "traffic": traffic,
        "peak_source": f"{peak_kind} bf16_tflops_sustained (kernel timed inside the step)",
        "step_share": g["ms"] / tot_ms if tot_ms > 0 else None,
    }
    breakdown = {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                     "tflops": round(v["flops"] / (v["ms"] / 1000) / 1e12, 1) if v["ms"] > 0 and v["flops"] else None,
                     "gbs": round(v["bytes"] / (v["ms"] / 1000) / 1e9, 1) if v["ms"] > 0 and v["bytes"] else None}
                 for k, v in prof.items()}
    total_flops = sum(v["flops"] for v in prof.values())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        oracle = oracle_module()
        ccfg, ct = cpu_weights(oracle, c)
        threads = os.cpu_count() or 1
        rate, _ = cpu_rate(oracle, ccfg, c, ct, 100, 1, threads)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port", "sample": cpu_sample_desc(c, ccfg)}

    if rank == 0:
        cfg_desc = {"workload": c["desc"] + (" per GPU" if scaling == "weak" else ""),
                    "batch_per_gpu": len(seqs), "seq_len": Lmax, "tokens_per_gpu": pb.T,
                    "arithmetic": "f16 tensor-core operands, f32 accumulate; "
                                  + ["FP32", "Q8_0", "Q4_0"][dtype] + " weights dequantised per layer",
                    "parallelism": (f"variant-sharded x{world} (contiguous blocks), masked-row all-gather" if c["dms"]
                                    else f"sequence-sharded x{world}, logits all-gather"),
                    "scaling_of_value": scaling,
                    "l2": "no flush: the per-step working set (activations, weights) exceeds the 126 MB L2"}
        line = {
            "metric": metric_name(args.config, c), "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded uniform residues, random-init N(0,0.02) weights)",
            "config": cfg_desc,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": int(d2h),
                    "steps": e2e_steps},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roofline,
            "achieved_model_tflops": total_flops / (ms / args.steps / 1000.0) / 1e12 if pb.T else None,
            "kernel_breakdown_ms_per_step": breakdown,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if strong is not None:
            line["strong_scaling"] = strong
        if c["dms"]:
            line["dms_variants_per_s"] = batch * e2e_steps / e2e_s
        emit(line)
    model.close()
    if world > 1:
        dist.destroy_process_group()


def run_vendor(args):
    """Vendor-library yardstick for the same matmul and attention work: per layer, the four
    projections as cuBLAS fp16 GEMMs (torch.matmul, plain outputs) and the attention as cuDNN's
    fused kernel (torch SDPA, dense [B, H, L, dh]), in forward order so that every call runs at the
    clock a full forward gets. No embedding, LayerNorm, bias, RoPE, GELU, residual, LM head or
    contact head, so it is a lower bound on a vendor-library forward, not one. Fixed-length
    forward configs only (c1, c4, c5); one GPU."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    c = CONFIGS[args.config]
    if c["dms"] or c["lengths"] != "fixed" or args.gpus != 1:
        emit({"impl": "vendor", "unavailable": "fixed-length forward configs on one GPU only"})
        return
    cfg = synth.preset(c["arch"])
    d, F_, H, nl = cfg.dim, cfg.hidden_dim, cfg.n_heads, cfg.n_layers
    B, L = args.batch or c["batch"], c["seq_len"]
    M, dh = B * L, d // H
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(0)
    shapes = [(3 * d, d), (d, d), (F_, d), (d, F_)]
    A = [torch.randn(M, k, device=dev, dtype=torch.float16, generator=g) for _, k in shapes]
    W = [torch.randn(n, k, device=dev, dtype=torch.float16, generator=g) * 0.02 for n, k in shapes]
    q, k, v = (torch.randn(B, H, L, dh, device=dev, dtype=torch.float16, generator=g) for _ in range(3))

    def events():
        return [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(nl)]

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def step(ev):
        for l in range(nl):
            e = ev[l]
            e[0].record()
            torch.matmul(A[0], W[0].t())
            e[1].record()
            F.scaled_dot_product_attention(q, k, v)
            e[2].record()
            for i in (1, 2, 3):
                torch.matmul(A[i], W[i].t())
            e[3].record()

    with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
        warm = events()
        for _ in range(args.warmup):
            step(warm)
        timed = [events() for _ in range(args.steps)]
        torch.cuda.synchronize()
        t0.record()
        for ev in timed:
            step(ev)
        t1.record()
        torch.cuda.synchronize()
    gemm = sum(e[0].elapsed_time(e[1]) + e[2].elapsed_time(e[3]) for ev in timed for e in ev)
    attn = sum(e[1].elapsed_time(e[2]) for ev in timed for e in ev)
    ms = t0.elapsed_time(t1) / args.steps
    emit({"impl": "vendor", "metric": metric_name(args.config, c), "value": M / (ms / 1000.0), "unit": UNIT,
          "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "n_gpus": 1,
          "config": {"workload": c["desc"], "batch_per_gpu": B, "seq_len": L},
          "parts_ms_per_step": {"gemm_cublas": gemm / args.steps, "attention_cudnn": attn / args.steps},
          "note": "projections (cuBLAS) and attention (cuDNN) only, in forward order; no other work"})


def main():
    # The JSON line is the only thing on stdout: everything else written to file descriptor 1
    # (library banners such as NCCL's version line at communicator set-up) goes to stderr.
    global _json_out
    _json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "vendor"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c4",
                    help="c4 (headline, default): 650M Q4_0 64 x 1024; c1/c2/c3/c5: the other benchmark configs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="override the per-GPU batch (profiling captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "vendor":
        run_vendor(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
