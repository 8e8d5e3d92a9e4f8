#!/usr/bin/env python
"""Serving benchmark: bge-m3-shaped mixed-tenant embedding with 10,000 resident rank-16 adapters.

Workload (one step = one batch through the hot path): a bge-m3 / XLM-R-large
shaped encoder (24 layers, hidden 1024, 16 heads, FFN 4096, vocab 250002),
seeded random init, bf16; LoRA rank 16 on query / key / value / attention-output
dense; 10,000 synthetic adapters (A, B ~ N(0, 0.02)) resident in the slot cache;
64 sequences per GPU padded to 512 tokens with real lengths uniform in
[32, 512] (a stratified draw, so every batch size carries the same mean
length); tenant ids Zipf(1.1) over the 10,000; CLS pooling + L2 normalisation.
Synthetic seeded data of that shape stands in for real requests.

Metric: sequences/s of the whole job (``value``, inputs resident in HBM, device
timed), the same end to end through the public API from pinned host buffers
(``e2e``), the dominant kernel against its roofline (``roofline``: the q/k/v
projection GEMM with the LoRA delta in its accumulator, tensor-bound), the
LoRA shrink's HBM bandwidth (``lora_hbm``), the LoRA overhead against the base
forward (``lora_overhead``: the same step with ``apply_lora=False``), the
isolated LoRA op at 64 x 256 x 1024 (``op``), the reference's own GPU path
(``ref_gpu``: stock encoder + per-row ``torch.bmm`` hooks) and its CPU path
(``cpu_baseline``) on the same box.

    python bench.py [--gpus N --steps K --warmup W]          # this implementation
    python bench.py --impl reference [--steps K --warmup W]  # the reference's CPU path
    python bench.py --mode op|classify|register               # the other workloads

N > 1 runs under torchrun, one process per GPU, each GPU with its own replica of
the model and the 10,000-adapter cache.  One global batch of N x 64 rows is
split across the ranks balanced on the cost of the padding-free forward (real
tokens, with attention's length term), and the embeddings are all-gathered over
NCCL every step (weak scaling).  Prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "sequences/sec at bge-m3 shape, 10k adapters; LoRA-kernel HBM GB/s vs peak"
TARGETS = ["query", "key", "value", "dense"]
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes (read + write) of one q/k/v lf_linear_lora_shrink launch at 17,410 tokens x
# 3072 x 1024, rank 16, 39 segments, from one ncu capture (dram__bytes_read.sum 52.6 MB +
# dram__bytes_write.sum 63.2 MB) of `bench.py --layers 2 --adapters 500 --steps 1
# --warmup 1 --no-cpu-baseline --no-e2e --no-extras` (same tokens and segments as the
# full workload; the adapters read are the batch's tenants in both).
NCU_TRAFFIC_QKV_GEMM = 115.9e6
# DRAM bytes (read 70.05 MB + write 0.13 MB) and duration (21.66 us) of one lf_lora_apply
# launch (the one-launch kernel) on the isolated op at rank 16, from one ncu capture
NCU_TRAFFIC_LORA_OP_R16 = 70.18e6
NCU_DURATION_LORA_OP_R16 = 21.66


def bge_m3_config(layers: int = 24):
    from transformers import XLMRobertaConfig

    return XLMRobertaConfig(vocab_size=250002, hidden_size=1024, num_hidden_layers=layers, num_attention_heads=16,
                            intermediate_size=4096, max_position_embeddings=8194, pad_token_id=1, type_vocab_size=1,
                            layer_norm_eps=1e-5)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["serve", "op", "classify", "register", "xl", "mixed"], default="serve",
                    help="serve: the bge-m3 embedding workload; op: the isolated LoRA op "
                         "Y = X W + (X A_t) B_t at X (64, 256, 1024); classify: 128 x 128 rows, 2,000 tenants "
                         "with heads, rank 8 on query+value; register: adapter registration latency; xl: XLM-R-XL "
                         "shape, rank 32 on query+value, 512 x 256 rows (set --batch 512 --seq 256 --rank 32 "
                         "--layers 36 --adapters 4000); mixed: ranks 8/16/32 from native-rank buckets against "
                         "one padded store")
    ap.add_argument("--batch", type=int, default=64, help="rows per GPU")
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--adapters", type=int, default=10000)
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--min-len", type=int, default=32)
    ap.add_argument("--cpu-rows", type=int, default=2, help="sequences per CPU-baseline step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="serve: skip the ablation, isolated-op and reference-GPU legs")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ranks", default="8,16,64", help="--mode op: LoRA ranks to measure")
    ap.add_argument("--persistent", type=int, default=1, help="0: per-tile expand kernel only")
    ap.add_argument("--no-pack", action="store_true", help="serve: run the padded forward instead of the packed one")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------
def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def measured_hbm_peak() -> tuple[float, str]:
    pk = _peaks()
    if "hbm_gbs" in pk:
        return float(pk["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s for a kernel timed inside the step: the burst figure, the
    stricter denominator (the sustained figure comes from a GEMM loop whose clocks
    settled lower than this step's; both clocks are recorded)."""
    pk = _peaks()
    if "bf16_tflops" in pk:
        return float(pk["bf16_tflops"]), "measured burst (MEASURED_PEAKS.json bf16_tflops)"
    return FALLBACK_BF16_TFLOPS, "fallback (burst)"


def measured_tensor_peak_sustained() -> float | None:
    """The sustained dense bf16 TFLOP/s (a seconds-long GEMM loop under the power cap), if measured."""
    v = _peaks().get("bf16_tflops_sustained")
    try:
        return float(v) if v else None
    except (TypeError, ValueError):
        return None


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.spans: list[tuple[float, float]] = []
        self.path = Path(tempfile.gettempdir()) / f"latefuse_b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
        if not self.gpus:
            return self
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", ",".join(map(str, self.gpus))], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()
            self.proc_done = True

    def span(self, t0: float, t1: float) -> None:
        """Wall-clock bounds of a timed region: only samples inside one count."""
        self.spans.append((t0, t1))

    def summary(self) -> dict:
        if not getattr(self, "proc_done", False) or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        import datetime

        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                continue
            if self.spans and not any(a <= ts <= b for a, b in self.spans):
                continue
            parts = parts[1:]
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_info() -> dict:
    model = "unknown"
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    quota = None
    try:
        q, per = Path("/sys/fs/cgroup/cpu.max").read_text().split()
        quota = None if q == "max" else float(q) / float(per)
    except Exception:
        pass
    return {"cpu": model, "usable_cores": len(os.sched_getaffinity(0)), "cgroup_quota": quota}


def events(n: int) -> list:
    return [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]


def median_ms(pairs) -> float:
    return statistics.median(a.elapsed_time(b) for a, b in pairs) if pairs else 0.0


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_inputs(args, rows: int, seed: int | None = None):
    """``rows`` right-padded rows (stratified lengths U[min_len, seq]) and their Zipf(1.1) tenants."""
    from latefuse_b200.synthetic import ragged_batch, zipf_tenants

    seed = args.seed if seed is None else seed
    ids, mask = ragged_batch(rows, args.seq, min_len=min(args.min_len, args.seq), max_len=args.seq, vocab=250002,
                             pad_id=1, cls_id=0, low_id=5, seed=seed, stratified=True)
    tenants = zipf_tenants(args.adapters, rows, alpha=1.1, seed=seed)
    return ids, mask, [f"adapter_{int(t)}" for t in tenants]


def build_ours(args, dev, rank=None, targets=None, adapters=None):
    import latefuse_b200 as lf

    hf = bge_m3_config(args.layers)
    cfg = lf.LoraServingConfig(model_name="bge-m3-shape (synthetic)", lora_rank=rank or args.rank,
                               batch_size=args.batch, max_seq_len=args.seq, target_modules=targets or TARGETS,
                               device=dev, dtype=torch.bfloat16, hf_config=hf)
    model = lf.EncoderWithLora.random_init(hf, cfg, seed=args.seed)
    n = adapters or args.adapters
    store = lf.AdapterStore(cfg, capacity=n)
    store.fill_random_(n, std=0.02, generator=torch.Generator(device=dev).manual_seed(args.seed + 1))
    return cfg, model, store


def run_serve(args):
    import torch.distributed as dist

    import latefuse_b200 as lf
    from latefuse_b200 import _native as nat
    from latefuse_b200.dp import DataParallelEmbedder, partition_rows, partition_tokens

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    cfg, model, store = build_ours(args, dev)
    emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False,
                                 pack_tokens=not args.no_pack)
    H = cfg.hidden_size
    n_glob = world * args.batch
    ids, mask, tenants = make_inputs(args, n_glob)
    lengths = mask.sum(1).tolist()
    pack = not args.no_pack
    parts = partition_tokens(lengths, world) if pack else partition_rows(lengths, world)
    mine = parts[rank]
    counts = [len(p) for p in parts]
    my_ids, my_mask = ids[mine], mask[mine]
    my_lengths = [lengths[i] for i in mine]
    my_tenants = [tenants[i] for i in mine]
    packed = model.pack(my_ids, my_lengths, store.slots(my_tenants)) if pack else None
    batch = None if pack else emb._get_assembler().batch_lora(my_tenants, args.seq, my_lengths)
    ids_d, mask_d = my_ids.to(dev), my_mask.to(dev)
    send = torch.zeros(max(counts), H, dtype=torch.bfloat16, device=dev)
    recv = torch.empty(world * max(counts), H, dtype=torch.bfloat16, device=dev)

    def step(apply_lora=True, gather_ev=None):
        with torch.no_grad():
            if packed is not None:
                pooled = model.encode_pooled_packed(packed, store, pooling="cls", apply_lora=apply_lora)
            else:
                pooled = model.encode_pooled(ids_d, mask_d, batch, pooling="cls", apply_lora=apply_lora)
            out = lf.head.l2_normalize(pooled)
            if world > 1:
                send[: out.shape[0]].copy_(out)
                if gather_ev is not None:
                    gather_ev[0].record()
                dist.all_gather_into_tensor(recv, send)
                if gather_ev is not None:
                    gather_ev[1].record()
        return out

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, n):
        """Device time per step of ``n`` calls, max over ranks, and the wall-clock span."""
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        t0 = time.time()
        start.record()
        for i in range(n):
            fn(i)
        end.record()
        barrier()
        t1 = time.time()
        ms = start.elapsed_time(end) / n
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms, (t0, t1)

    # clocks are sampled from the warm-up on (nvidia-smi takes a moment to start);
    # only the samples inside the timed regions are reported
    clocks = ClockSampler(list(range(torch.cuda.device_count())) if rank == 0 else [])
    clocks.__enter__()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    emb.check_device_status()

    # ---- device-timed region: inputs resident in HBM, no instrumentation ----
    n0 = nat.launch_count()
    ms, span = timed(lambda i: step(True), args.steps)
    clocks.span(*span)
    launches = nat.launch_count() - n0
    emb.check_device_status()
    # ---- the same steps again with CUDA events around the LoRA launches and the
    # all-gather, for the per-kernel figures (events add a little time of their own) ----
    model.lora_events = []
    gathers = events(args.steps)
    ms_instrumented, span = timed(lambda i: step(True, gathers[i]), args.steps)
    clocks.span(*span)
    lora_events = model.lora_events
    model.lora_events = None
    emb.check_device_status()
    by_kind: dict[str, list[float]] = {}
    for kind, s_ev, e_ev in lora_events:
        by_kind.setdefault(kind, []).append(s_ev.elapsed_time(e_ev))
    gather_ms = median_ms(gathers) if world > 1 else 0.0
    lora_ms_step = sum(sum(v) for v in by_kind.values()) / args.steps
    shrink_ms_step = sum(sum(by_kind.get(k, [])) for k in ("qkv_shrink", "dense_shrink")) / args.steps
    fused = "qkv_gemm" in by_kind
    gemm_ms = statistics.median(by_kind["qkv_gemm"]) if fused else 0.0

    # ---- LoRA overhead: the same step without the adapters (reference method:
    # benchmarks/profiling/forward_breakdown.py:208-255) ----
    ablation = None
    if not args.no_extras:
        for _ in range(args.warmup):
            step(False)
        ms_base, span = timed(lambda i: step(False), args.steps)
        clocks.span(*span)
        ablation = {"ms_lora": ms, "ms_base": ms_base, "overhead_vs_base": (ms - ms_base) / ms_base,
                    "share_of_lora_step": (ms - ms_base) / ms, "target_overhead_vs_base": 0.10,
                    "note": "base = the same packed forward with apply_lora=False (projections on cuBLAS, no "
                            "shrink); lora = q/k/v and attention-output projections on this library's GEMM, "
                            "each computing its shrink and adding the delta in its accumulator"}

    segs = packed.segments if packed is not None else batch.segments
    n_unique = len(set(my_tenants))
    R = args.rank
    T_tok = segs.n_tokens
    if fused:
        gemm_flops = 2.0 * T_tok * 3 * H * (H + R)
        tpeak, tpeak_src = measured_tensor_peak()
        tach = gemm_flops / (gemm_ms * 1e-3) / 1e12
        roofline = {
            "bound": "tensor", "achieved": tach, "peak": tpeak, "unit": "TFLOP/s", "frac": tach / tpeak,
            "traffic": NCU_TRAFFIC_QKV_GEMM if (pack and R == 16 and args.batch == 64 and args.seq == 512) else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one lf_linear_lora_shrink q/k/v "
                              "launch (2-layer, 500-adapter capture of the same 17,410-token batch)"
                              if NCU_TRAFFIC_QKV_GEMM is not None else "not captured for this kernel build",
            "kernel": "lf_linear_lora: q/k/v projection (T x 3072 x 1024) with the per-row LoRA delta in the "
                      "tcgen05 accumulator (one launch per layer)",
            "algorithmic_flops_per_launch": gemm_flops, "launch_ms": gemm_ms, "tokens_per_launch": T_tok,
            "peak_source": tpeak_src,
        }
        tsus = measured_tensor_peak_sustained()
        roofline["frac_of_sustained"] = tach / tsus if tsus else None
        roofline["peak_sustained"] = tsus
    else:
        roofline = {"bound": "tensor", "achieved": None, "peak": None, "unit": "TFLOP/s", "frac": None,
                    "traffic": None, "kernel": "cuBLAS projections (this configuration does not use lf_linear_lora)"}
    hpeak, hpeak_src = measured_hbm_peak()
    lora_hbm = None
    if shrink_ms_step > 0:
        n_blk = (T_tok + 127) // 128 + segs.n_segs
        shrink_bytes_step = args.layers * sum(
            T_tok * H * 2 + n_unique * m * H * R * 2 + m * n_blk * 128 * R * 2 for m in (3, 1))
        shrink_gbs = shrink_bytes_step / (shrink_ms_step * 1e-3) / 1e9
        lora_hbm = {
            "kernel": "lf_lora_shrink_blocked (per layer: q/k/v and attention-output shrinks)",
            "achieved": shrink_gbs, "peak": hpeak, "unit": "GB/s", "frac": shrink_gbs / hpeak,
            "algorithmic_bytes_per_step": shrink_bytes_step, "ms_per_step": shrink_ms_step, "peak_source": hpeak_src,
            "launches_per_step": 2 * args.layers,
            "note": "the expand runs inside the projection GEMM (u and B reads, K = rank MMAs)",
        }

    # ---- end to end through the public API from pinned host buffers ----
    e2e = None
    if not args.no_e2e:
        ids_h, mask_h = ids.pin_memory(), mask.pin_memory()
        my_ids_h, my_mask_h = my_ids.pin_memory(), my_mask.pin_memory()
        out_h = torch.empty(n_glob, H, dtype=torch.bfloat16).pin_memory()
        runner = DataParallelEmbedder(emb) if world > 1 else None
        # copied to the device each step: this rank's packed token tables and segment table
        h2d = packed.host_bytes if packed is not None else (my_ids.numel() * 8 + my_mask.numel() * 8
                                                            + segs.host.numel() * 4)
        d2h = out_h.numel() * 2

        def e2e_run(n):
            # every step: its host batch packed and copied in, its embeddings copied out to
            # pinned host memory and waited for; the next batch is prepared and launched
            # while the previous one computes (two in flight)
            if runner is not None:
                outs = runner.embed_tokens_stream(((ids_h, mask_h, tenants) for _ in range(n)), depth=2)
            else:
                outs = emb.embed_tokens_stream(((my_ids_h, my_mask_h, my_tenants) for _ in range(n)), depth=2)
            for host in outs:
                out_h[:host.shape[0]].copy_(host)

        e2e_run(args.warmup)
        barrier()
        t0 = time.perf_counter()
        e2e_run(args.steps)
        barrier()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = t.item()
        e2e = {"value": n_glob / (e2e_ms * 1e-3), "unit": "sequences/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": ("DataParallelEmbedder.embed_tokens_stream" if world > 1
                        else "MultiTenantEmbedder.embed_tokens_stream")
                       + "(pinned host ids/mask, tenant ids; two batches in flight) -> pinned host embeddings, "
                         "each waited for"}
    clocks.__exit__(None, None, None)

    op = ref_gpu = cpu = None
    if rank == 0 and world == 1 and not args.no_extras:
        ref_gpu = reference_gpu(args, dev, my_ids, my_mask, my_tenants, store, model)
        op = op_results(args, dev, steps=max(args.steps, 10), warmup=args.warmup)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, steps=3, warmup=1, rows=args.cpu_rows)

    if lora_hbm is None and op is not None and "r16" in op.get("results", {}):
        # the shrink runs inside the projection GEMM's launch here, so the LoRA kernels'
        # bandwidth is read off the same kernels as an isolated op
        r16 = op["results"]["r16"]
        lora_hbm = {
            "kernel": "lf_lora_apply as the isolated op, one launch (shrink and expand in one kernel, u kept on "
                      "chip): X (64, 256, 1024) bf16, rank 16, 10,000 resident adapters, L2 flushed clean before each call",
            "achieved": r16["apply_flushed_gbs"], "peak": op.get("peak_gbs"), "unit": "GB/s",
            "frac": r16["apply_flushed_frac_of_hbm"], "algorithmic_bytes": r16["algorithmic_bytes"],
            "us": r16["apply_flushed_us"], "two_launch_us": r16["two_launch_flushed_us"],
            "traffic": NCU_TRAFFIC_LORA_OP_R16,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch (y's writes stay in L2)",
            "ncu_duration_us": NCU_DURATION_LORA_OP_R16,
            "ncu_frac": r16["algorithmic_bytes"] / (NCU_DURATION_LORA_OP_R16 * 1e-6) / 1e9 / op.get("peak_gbs"),
            # the same call timed inside the op, right after the base GEMM (Y = X W + delta)
            "in_op_us": r16["delta_us"], "in_op_frac": r16["delta_frac_of_hbm"],
            "note": "in the serving step the shrink and the expand run inside the q/k/v and attention-output "
                    "projection GEMMs (lf_linear_lora_shrink): no separate launch exists to time, and their "
                    "in-step cost is lora_overhead",
        }
    if fused:
        # the q/k/v launch also computes the shrink: 2 T H (3 R) FLOPs more
        shrink_flops = 2.0 * T_tok * H * 3 * R if model.fuse_shrink else 0.0
        roofline["algorithmic_flops_per_launch"] += shrink_flops
        roofline["achieved"] = roofline["algorithmic_flops_per_launch"] / (gemm_ms * 1e-3) / 1e12
        roofline["frac"] = roofline["achieved"] / roofline["peak"]
        if shrink_flops:
            roofline["kernel"] = ("lf_linear_lora_shrink: q/k/v projection (T x 3072 x 1024) computing its LoRA "
                                  "shrink and adding the per-row delta in the tcgen05 accumulator (one launch per "
                                  "layer)")

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    real_tokens = sum(lengths)
    line = {
        "metric": METRIC,
        "value": n_glob / (ms * 1e-3),
        "unit": "sequences/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init bge-m3-shaped encoder, 10,000 random rank-16 adapters, "
                "Zipf(1.1) tenants, lengths U[32,512] stratified)",
        "tokens_per_s": real_tokens / (ms * 1e-3),
        "config": {
            "workload": f"bge-m3 shape ({args.layers}L, H1024, 16 heads, FFN 4096, vocab 250002) bf16 embedding "
                        f"forward, LoRA r={args.rank} on query/key/value/attention-output dense, {args.adapters} "
                        f"resident adapters, {args.batch} rows per GPU x {args.seq} right-padded (lengths "
                        f"U[{args.min_len},{args.seq}]), Zipf(1.1) tenants, CLS pooling + L2 norm",
            "global_batch": n_glob,
            "seq_len": args.seq,
            "real_tokens_global": real_tokens,
            "real_tokens_rank0": T_tok if packed is not None else segs.real_tokens,
            "rows_per_rank": counts,
            "padded_tokens_per_gpu_step": args.batch * args.seq,
            "tokens_computed": "real tokens only (packed, attention per sequence)" if packed is not None
                               else "all padded positions (LoRA on real tokens only)",
            "partition": "balanced on packed cost (tokens + attention length term)" if pack else "equal rows",
            "parallelism": f"dp{world}",
            "adapters": args.adapters,
            "rank": args.rank,
            "unique_tenants_rank0": n_unique,
            "l2": "inputs larger than L2: every step streams 1.1 GB of weights and >0.5 GB of activations",
        },
        "roofline": roofline,
        "lora_share_of_step": lora_ms_step / ms,
        "lora_share_note": ("shrink + fused projection GEMM launches (the GEMM includes the base projection)"
                            if fused else "shrink + expand launches"),
        "allgather_ms": gather_ms,
        "ms_per_step_instrumented": ms_instrumented,
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "clocks": clocks.summary(),
    }
    for key, val in (("lora_overhead", ablation), ("lora_hbm", lora_hbm), ("e2e", e2e), ("op", op),
                     ("ref_gpu", ref_gpu), ("cpu_baseline", cpu)):
        if val is not None:
            line[key] = val
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the reference's GPU path on the same device: stock encoder + per-row bmm hooks
# ---------------------------------------------------------------------------
def _hf_bge_m3(args, dev):
    """A bge-m3-shaped HuggingFace ``XLMRobertaModel`` in bf16 on ``dev`` (N(0, .02) weights)."""
    from transformers import XLMRobertaModel

    with torch.device("meta"):
        model = XLMRobertaModel(bge_m3_config(args.layers))
    model = model.to_empty(device=dev).eval()
    g = torch.Generator(device=dev).manual_seed(args.seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "LayerNorm.weight" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, 0.02, generator=g)
        for name, b in model.named_buffers():
            if name.endswith("position_ids"):
                b.copy_(torch.arange(b.shape[-1], device=dev).expand_as(b))
            else:
                b.zero_()
    return model.to(torch.bfloat16)


def reference_gpu(args, dev, ids, mask, tenants, store, model_ours) -> dict:
    """The reference's serving forward on this GPU (``src/latefuse/model/hf_wrapper.py:
    169-219``): the stock HF encoder on the padded batch, each targeted projection
    followed in a forward hook by ``cat`` of the rows' factors, two ``torch.bmm`` and
    the add.  The rows' factors are views of this library's slot cache, so the
    reference's per-batch assembly (``weights/batch.py:44-102``) is not timed."""
    suffix = {"query": "attention.self.query", "key": "attention.self.key", "value": "attention.self.value",
              "dense": "attention.output.dense"}
    hf = _hf_bge_m3(args, dev)
    L = args.layers
    rows = [store.get(t) for t in tenants]
    handles = []
    mods = dict(hf.named_modules())
    for m in TARGETS:
        for layer in range(L):
            def hook(_mod, inputs, output, m=m, layer=layer):
                a = torch.cat([w.wa[m][layer].unsqueeze(0) for w in rows], 0)
                b = torch.cat([w.wb[m][layer].unsqueeze(0) for w in rows], 0)
                return output + torch.bmm(torch.bmm(inputs[0], a), b)

            handles.append(mods[f"encoder.layer.{layer}.{suffix[m]}"].register_forward_hook(hook))
    ids_d, mask_d = ids.to(dev), mask.to(dev)

    def fwd():
        with torch.no_grad():
            out = hf(input_ids=ids_d, attention_mask=mask_d).last_hidden_state[:, 0]
            return torch.nn.functional.normalize(out, p=2, dim=-1)

    for _ in range(2):
        fwd()
    steps = 5
    ev = events(1)[0]
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(steps):
        fwd()
    ev[1].record()
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / steps
    for h in handles:
        h.remove()
    del hf
    torch.cuda.empty_cache()
    return {"value": ids.shape[0] / (ms * 1e-3), "unit": "sequences/s", "ms_per_step": ms,
            "sample": f"the same {ids.shape[0]} rows padded to {ids.shape[1]} as the reference computes them, "
                      f"{steps} timed steps, bf16, stock XLMRobertaModel (sdpa attention) + per-row bmm hooks on "
                      "query/key/value/dense; assembly not timed",
            "kind": "port of the reference's hf engine on the same GPU"}


# ---------------------------------------------------------------------------
# isolated LoRA op (64, 256, 1024) bf16
# ---------------------------------------------------------------------------
def op_results(args, dev, steps: int, warmup: int) -> dict:
    """``Y = X W + (X A_t) B_t`` at X (64, 256, 1024) bf16 with 10,000 resident adapters and
    Zipf(1.1) tenants per row, for each rank of ``args.ranks``.  The delta's algorithmic
    bytes are 3*T*H*2 + U*4*H*r (x read, y read and written, each unique tenant's A and B)."""
    from latefuse_b200 import _native as nat
    from latefuse_b200.lora import FactorCache, SegmentTable, lora_apply, lora_expand, lora_shrink, workspace_bytes
    from latefuse_b200.synthetic import zipf_tenants

    nat.set_option(nat.LF_OPT_PERSISTENT, args.persistent)
    B, S, H = 64, 256, 1024
    T = B * S
    g = torch.Generator(device=dev).manual_seed(args.seed)
    peak, _ = measured_hbm_peak()
    out = {}
    for R in [int(r) for r in str(args.ranks).split(",")]:
        x = torch.randn(T, H, device=dev, dtype=torch.bfloat16, generator=g)
        w = (torch.randn(H, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        cache = torch.empty(args.adapters, 1, 2, H * R, device=dev, dtype=torch.bfloat16).normal_(0, 0.02, generator=g)
        fc = FactorCache(a=cache, b=cache, a_offset=0, b_offset=H * R, a_slot_stride=cache.stride(0),
                         b_slot_stride=cache.stride(0), a_module_stride=cache.stride(1),
                         b_module_stride=cache.stride(1), n_slots=args.adapters, hidden=H, rank=R)
        slots = [int(t) for t in zipf_tenants(args.adapters, B, 1.1, seed=args.seed)]
        segs = SegmentTable.for_padded(slots, S, dev)
        ws = torch.empty(workspace_bytes(torch.bfloat16, T, R, 1), dtype=torch.uint8, device=dev)
        y = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        # L2 flush between steps: 256 MB written, then another 256 MB read, so that L2 holds no
        # dirty lines whose write-back the timed kernel would otherwise pay for
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
        flush_r = torch.ones(256 * 1024 * 1024 // 8, dtype=torch.int64, device=dev)

        def flush_l2():
            flush.zero_()
            flush_r.max()

        def op(times=None):
            torch.matmul(x, w, out=y)
            if times is not None:
                times[0].record()
            lora_apply(x, y, fc, segs, [0], [0], ws)
            if times is not None:
                times[1].record()

        for _ in range(warmup):
            op()
        torch.cuda.synchronize()
        ev, ops = events(steps), events(steps)
        n0 = nat.launch_count()
        for i in range(steps):
            flush_l2()
            ops[i][0].record()
            op(ev[i])
            ops[i][1].record()
        torch.cuda.synchronize()
        delta_ms, op_ms = median_ms(ev), median_ms(ops)
        launches = (nat.launch_count() - n0) / steps
        # the delta on its own with L2 flushed before each call: lf_lora_apply as one launch
        # (the default), as the shrink + expand launches, and each of those launches alone
        u = ws[: T * R * 2].view(torch.bfloat16).view(1, T, R)
        ap, two, sh, ex = [], [], [], []

        def two_launch():
            nat.set_option(nat.LF_OPT_FUSED_APPLY, 0)
            lora_apply(x, y, fc, segs, [0], [0], ws)
            nat.set_option(nat.LF_OPT_FUSED_APPLY, 1)

        for _ in range(steps):
            for fn, acc in ((lambda: lora_apply(x, y, fc, segs, [0], [0], ws), ap), (two_launch, two),
                            (lambda: lora_shrink(x, u, fc, segs, [0]), sh),
                            (lambda: lora_expand(u, y, fc, segs, [0], [0], True), ex)):
                flush_l2()
                a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a_.record()
                fn()
                b_.record()
                acc.append((a_, b_))
        torch.cuda.synchronize()
        apply_ms, two_ms, shrink_ms, expand_ms = median_ms(ap), median_ms(two), median_ms(sh), median_ms(ex)
        U = len(set(slots))
        algo = 3 * T * H * 2 + U * 4 * H * R
        flops = 2 * T * H * H + 4 * T * H * R
        out[f"r{R}"] = {"delta_us": delta_ms * 1e3, "delta_gbs": algo / (delta_ms * 1e-3) / 1e9,
                        "delta_frac_of_hbm": algo / (delta_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": algo,
                        "apply_flushed_us": apply_ms * 1e3, "apply_flushed_gbs": algo / (apply_ms * 1e-3) / 1e9,
                        "apply_flushed_frac_of_hbm": algo / (apply_ms * 1e-3) / 1e9 / peak,
                        "two_launch_flushed_us": two_ms * 1e3,
                        "unique_tenants": U, "op_us": op_ms * 1e3, "op_tflops": flops / (op_ms * 1e-3) / 1e12,
                        "shrink_us": shrink_ms * 1e3,
                        "shrink_gbs": (T * H * 2 + U * 2 * H * R) / (shrink_ms * 1e-3) / 1e9,
                        "expand_us": expand_ms * 1e3,
                        "expand_gbs": (2 * T * H * 2 + U * 2 * H * R) / (expand_ms * 1e-3) / 1e9,
                        "launches_per_op": launches}
        del cache, x, y, w, ws, flush, flush_r
        torch.cuda.empty_cache()
    return {"workload": "Y = X W + (X A_t) B_t, X (64,256,1024) bf16, 10,000 adapters, Zipf(1.1) tenants, "
                        "L2 flushed between steps (256 MB written, then 256 MB of another buffer read)", "peak_gbs": peak,
            "results": out}


def run_op(args):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res = op_results(args, dev, args.steps, args.warmup)
    print(json.dumps({"mode": "op", **res}), flush=True)


# ---------------------------------------------------------------------------
# classification: 2,000 tenants with heads
# ---------------------------------------------------------------------------
def run_classify(args):
    """Classification at 128 x 128 rows on the bge-m3-shaped encoder, rank 8 on
    query+value, 2,000 tenants each with an adapter and a head of U[2, 20] labels
    (coef ~ N(0, .05), intercept ~ N(0, .1)), Zipf(1.1) tenants: one step = the
    packed forward with the pooler, the heads and the masked softmax on the device."""
    import latefuse_b200 as lf
    from latefuse_b200 import _native as nat
    from latefuse_b200.synthetic import ragged_batch, zipf_tenants

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_t, B, S = 2000, 128, 128
    cfg, model, store = build_ours(args, dev, rank=8, targets=["query", "value"], adapters=n_t)
    clf = lf.MultiTenantClassifier(cfg, engine="bert", model=model, store=store, tokenizer=False)
    g = torch.Generator().manual_seed(args.seed + 5)
    for i in range(n_t):
        n = int(torch.randint(2, 21, (1,), generator=g))
        clf.heads.load(f"adapter_{i}", torch.randn(n, 1024, generator=g) * 0.05, torch.randn(n, generator=g) * 0.1)
    ids, mask = ragged_batch(B, S, min_len=S, max_len=S, vocab=250002, pad_id=1, cls_id=0, low_id=5,
                             seed=args.seed)
    tenants = [f"adapter_{int(t)}" for t in zipf_tenants(n_t, B, alpha=1.1, seed=args.seed)]
    pb = model.pack(ids, [S] * B, store.slots(tenants))
    table, num_labels, n_max = clf.heads.head_table(tenants)
    coef, bias = clf.heads.packed
    logits = torch.empty(B, n_max, dtype=torch.bfloat16, device=dev)
    probs = torch.empty(B, n_max, dtype=torch.float32, device=dev)
    head_ev = events(args.steps)

    def step(i=None):
        with torch.no_grad():
            pooled = model.encode_pooled_packed(pb, store, "auto")
            if i is not None:
                head_ev[i][0].record()
            lf.head.head_forward(pooled, pooling="none", coef=coef, bias=bias, head_table=table, n_max=n_max,
                                 logits_out=logits, probs_out=probs)
            if i is not None:
                head_ev[i][1].record()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    start, end = events(1)[0]
    n0 = nat.launch_count()
    start.record()
    for i in range(args.steps):
        step(i)
    end.record()
    torch.cuda.synchronize()
    clf.check_device_status()
    ms = start.elapsed_time(end) / args.steps
    head_ms = median_ms(head_ev)
    uniq = {t: n for t, n in zip(tenants, num_labels)}
    head_bytes = B * 1024 * 2 + sum(n * 1024 * 2 + n * 2 for n in uniq.values()) + B * n_max * (2 + 4) + B * 8
    peak, src = measured_hbm_peak()
    e2e_ms = None
    if not args.no_e2e:
        ids_h, mask_h = ids.pin_memory(), mask.pin_memory()
        for _ in range(args.warmup):
            out = clf.classify_tokens(ids_h, mask_h, tenants)[1].cpu()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            out = clf.classify_tokens(ids_h, mask_h, tenants)[1].cpu()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        del out
    print(json.dumps({
        "mode": "classify", "metric": "sequences/sec, classification", "value": B / (ms * 1e-3),
        "unit": "sequences/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
        "config": {"workload": f"bge-m3 shape ({args.layers}L) bf16 classification, LoRA r=8 on query+value, "
                               f"{n_t} tenants with heads of U[2,20] labels, {B}x{S} rows, Zipf(1.1) tenants, pooler "
                               "(auto) + per-tenant head + masked softmax",
                   "unique_tenants": len(uniq), "n_max": n_max},
        "head": {"kernel": "lf_head_forward (gather-GEMV over the packed head cache + masked softmax/sigmoid)",
                 "us": head_ms * 1e3, "algorithmic_bytes": head_bytes,
                 "achieved_gbs": head_bytes / (head_ms * 1e-3) / 1e9,
                 "frac_of_hbm": head_bytes / (head_ms * 1e-3) / 1e9 / peak, "peak_source": src},
        "e2e": None if e2e_ms is None else {"value": B / (e2e_ms * 1e-3), "unit": "sequences/s",
                                            "ms_per_step": e2e_ms,
                                            "path": "MultiTenantClassifier.classify_tokens -> host probabilities"},
        "gpu_launches_per_step": (nat.launch_count() - n0) / args.steps,
    }), flush=True)


# ---------------------------------------------------------------------------
# mixed ranks: native-rank buckets against one padded store
# ---------------------------------------------------------------------------
def run_mixed(args):
    """A fleet of ``--adapters`` adapters with ranks drawn uniformly from 8, 16 and 32
    on the bge-m3 shape (q/k/v/dense), served at r_max 32 two ways (the reference's
    ``benchmarks/profiling/mixed_rank_bench.py`` arms): every adapter zero-padded into
    one rank-32 store, and each at its own rank in a rank bucket with the batch's
    adapters gathered into an r_max staging cache per batch (``RankBucketStore``).
    One step = ``embed_tokens`` of the 64 x 512 stratified batch from host tensors."""
    import latefuse_b200 as lf
    from latefuse_b200 import _native as nat
    from latefuse_b200.rank_buckets import RankBucketStore

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, mix = args.adapters, (8, 16, 32)
    cfg, model, padded = build_ours(args, dev, rank=32, adapters=n)
    g = torch.Generator().manual_seed(args.seed + 7)
    ranks = [mix[int(i)] for i in torch.randint(0, len(mix), (n,), generator=g)]
    fleet = RankBucketStore(cfg)
    fleet.fill_random_(ranks, std=0.02, generator=torch.Generator(device=dev).manual_seed(args.seed + 8))
    ids, mask, tenants = make_inputs(args, args.batch)
    ids_h, mask_h = ids.pin_memory(), mask.pin_memory()
    out = {}
    for name, store in (("padded", padded), ("native_buckets", fleet)):
        emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False)
        for _ in range(args.warmup):
            emb.embed_tokens(ids_h, mask_h, tenants)
        torch.cuda.synchronize()
        ev = events(1)[0]
        t0 = time.perf_counter()
        ev[0].record()
        for _ in range(args.steps):
            emb.embed_tokens(ids_h, mask_h, tenants)
        ev[1].record()
        torch.cuda.synchronize()
        emb.check_device_status()
        ms = ev[0].elapsed_time(ev[1]) / args.steps
        out[name] = {"value": args.batch / (ms * 1e-3), "ms_per_step": ms,
                     "wall_ms_per_step": (time.perf_counter() - t0) * 1e3 / args.steps,
                     "adapter_bytes": store.memory_bytes()}
    uniq = len(set(tenants))
    print(json.dumps({
        "mode": "mixed", "metric": "sequences/sec, bge-m3 shape, mixed-rank fleet (r in 8/16/32, r_max 32)",
        "value": out["native_buckets"]["value"], "unit": "sequences/s", "steps": args.steps, "warmup": args.warmup,
        "dtype": "bf16",
        "config": {"workload": f"bge-m3 shape ({args.layers}L) bf16 embedding forward, LoRA on q/k/v/dense, {n} "
                               f"adapters with ranks uniform over {list(mix)} served at r_max 32, {args.batch} rows x "
                               f"{args.seq} (lengths U[{args.min_len},{args.seq}]), Zipf(1.1) tenants, CLS + L2",
                   "unique_tenants": uniq, "rank_counts": {str(r): ranks.count(r) for r in mix}},
        "arms": out,
        "memory_native_over_padded": out["native_buckets"]["adapter_bytes"] / out["padded"]["adapter_bytes"],
        "gpu_launches": nat.launch_count(),
    }), flush=True)


# ---------------------------------------------------------------------------
# XLM-R-XL scale-out (rank 32 on query+value, 512 x 256 rows)
# ---------------------------------------------------------------------------
def xl_config(layers: int = 36):
    from transformers import XLMRobertaXLConfig

    return XLMRobertaXLConfig(vocab_size=250002, hidden_size=2560, num_hidden_layers=layers, num_attention_heads=32,
                              intermediate_size=10240, max_position_embeddings=514, pad_token_id=1, type_vocab_size=1,
                              layer_norm_eps=1e-5)


def _hf_random(model_cls, hf_config, dev, seed: int):
    """A HuggingFace model built on ``dev`` with N(0, .02) weights, zero biases and unit
    LayerNorms, in bf16 (no host copy of the weights)."""
    with torch.device("meta"):
        model = model_cls(hf_config)
    model = model.to_empty(device=dev).eval()
    g = torch.Generator(device=dev).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "LayerNorm.weight" in name or "layer_norm.weight" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, 0.02, generator=g)
        for name, b in model.named_buffers():
            if name.endswith("position_ids"):
                b.copy_(torch.arange(b.shape[-1], device=dev).expand_as(b))
            else:
                b.zero_()
    return model.to(torch.bfloat16)


def run_xl(args):
    """XLM-R-XL shape (36 layers, hidden 2560, 32 heads of 80, FFN 10240), bf16, rank 32 on
    query+value, 512 x 256 rows per step, Zipf(1.1) tenants over the resident adapters:
    the stock HF encoder (sdpa attention, cuBLAS projections) with this library's LoRA
    kernels in its hooks (``engine="hf"``), against the reference's own hook body
    (``torch.bmm`` per row, ``src/latefuse/model/hf_wrapper.py:212-217``) on the same
    model and rows.  The reference's 50,000 adapters per GPU (1.18 TB) do not fit a
    180 GB device; ``--adapters`` sets the resident count (23.6 MB each)."""
    import latefuse_b200 as lf
    from latefuse_b200 import _native as nat
    from latefuse_b200.synthetic import ragged_batch, zipf_tenants
    from transformers import XLMRobertaXLModel

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S, R, targets = args.batch, args.seq, args.rank, ["query", "value"]
    hf_cfg = xl_config(args.layers)
    base = _hf_random(XLMRobertaXLModel, hf_cfg, dev, args.seed)
    cfg = lf.LoraServingConfig(model_name="xlm-roberta-xl-shape (synthetic)", lora_rank=R, batch_size=B,
                               max_seq_len=S, target_modules=targets, device=dev, dtype=torch.bfloat16,
                               hf_config=hf_cfg)
    store = lf.AdapterStore(cfg, capacity=args.adapters)
    store.fill_random_(args.adapters, std=0.02, generator=torch.Generator(device=dev).manual_seed(args.seed + 1))
    model = lf.HFEncoderWithLora(base, cfg)
    emb = lf.MultiTenantEmbedder(cfg, engine="hf", model=model, store=store, tokenizer=False)
    ids, mask = ragged_batch(B, S, min_len=S, max_len=S, vocab=250002, pad_id=1, cls_id=0, low_id=5, seed=args.seed)
    tenants = [f"adapter_{int(t)}" for t in zipf_tenants(args.adapters, B, alpha=1.1, seed=args.seed)]
    ids_d, mask_d = ids.to(dev), mask.to(dev)

    def ours():
        with torch.no_grad():
            return emb.embed_tokens(ids_d, mask_d, tenants)

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ev = events(1)[0]
        ev[0].record()
        for _ in range(steps):
            out = fn()
        ev[1].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) / steps, out

    n0 = nat.launch_count()
    with ClockSampler([0]) as sampler:
        t0 = time.time()
        ms, out_ours = timed(ours, args.steps)
        sampler.span(t0, time.time())
    launches = (nat.launch_count() - n0) / (args.steps + args.warmup)
    emb.check_device_status()
    # the same forward without adapters (the hooks are inert outside the engine's calls)
    ms_base, _ = timed(lambda: _base_only(base, ids_d, mask_d), max(2, args.steps // 2))

    # the reference's hook body on the same model (this library's hooks stay inert
    # outside its own forward calls)
    rows = [store.get(t) for t in tenants]
    suffix = {"query": "attention.self.query", "value": "attention.self.value"}
    mods = dict(base.named_modules())
    handles = []
    for m in targets:
        for layer in range(args.layers):
            def hook(_mod, inputs, output, m=m, layer=layer):
                a = torch.cat([w.wa[m][layer].unsqueeze(0) for w in rows], 0)
                b = torch.cat([w.wb[m][layer].unsqueeze(0) for w in rows], 0)
                return output + torch.bmm(torch.bmm(inputs[0], a), b)

            handles.append(mods[f"encoder.layer.{layer}.{suffix[m]}"].register_forward_hook(hook))
    ms_ref, out_ref = timed(lambda: _base_only(base, ids_d, mask_d), max(2, args.steps // 2))
    for h in handles:
        h.remove()
    err = ((out_ours.float() - out_ref.float()).norm(dim=-1) / out_ref.float().norm(dim=-1)).max().item()

    e2e_ms = None
    if not args.no_e2e:
        ids_h, mask_h = ids.pin_memory(), mask.pin_memory()
        for _ in range(args.warmup):
            emb.embed_tokens(ids_h, mask_h, tenants).cpu()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            emb.embed_tokens(ids_h, mask_h, tenants).cpu()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    flop_tok = 2 * args.layers * (4 * 2560 ** 2 + 2 * 2560 * 10240) + 4 * args.layers * S * 2560
    print(json.dumps({
        "mode": "xl", "metric": "sequences/sec, XLM-R-XL shape, rank 32 on query+value", "value": B / (ms * 1e-3),
        "unit": "sequences/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
        "data": f"synthetic (seeded random-init XLM-R-XL-shaped encoder, {args.adapters} random rank-{R} adapters, "
                "Zipf(1.1) tenants, full-length rows)",
        "config": {"workload": f"XLM-R-XL shape ({args.layers}L, H2560, 32 heads of 80, FFN 10240) bf16 embedding "
                               f"forward, LoRA r={R} on query+value, {args.adapters} resident adapters "
                               f"({args.adapters * store.slot_bytes / 1e9:.0f} GB), {B} rows x {S}, "
                               "CLS pooling + L2 norm", "global_batch": B, "seq_len": S,
                   "unique_tenants": len(set(tenants))},
        "tflops": flop_tok * B * S / (ms * 1e-3) / 1e12,
        "lora_overhead": {"ms_base": ms_base, "overhead_vs_base": (ms - ms_base) / ms_base,
                          "target_overhead_vs_base": 0.10},
        "ref_gpu": {"value": B / (ms_ref * 1e-3), "unit": "sequences/s", "ms_per_step": ms_ref,
                    "kind": "the reference's per-row torch.bmm hook body on the same model and rows (assembly not "
                            "timed)"},
        "parity_vs_ref_gpu_max_row_rel": err,
        "e2e": None if e2e_ms is None else {"value": B / (e2e_ms * 1e-3), "unit": "sequences/s",
                                            "ms_per_step": e2e_ms, "h2d_bytes_per_step": ids.numel() * 8 * 2,
                                            "d2h_bytes_per_step": B * 2560 * 2,
                                            "path": "MultiTenantEmbedder.embed_tokens(pinned host ids/mask) -> host"},
        "clocks": sampler.summary(),
        "gpu_launches_per_step": launches,
    }), flush=True)


def _base_only(base, ids_d, mask_d):
    """CLS + L2 of the HF model's own forward (whatever hooks it carries)."""
    with torch.no_grad():
        out = base(input_ids=ids_d, attention_mask=mask_d).last_hidden_state[:, 0]
        return torch.nn.functional.normalize(out.float(), p=2, dim=-1)


# ---------------------------------------------------------------------------
# registration latency
# ---------------------------------------------------------------------------
def run_register(args):
    """Adapter registration into the slot cache at the bge-m3 shape (24 layers, r=16,
    query/key/value/dense: 6.29 MB per adapter in bf16): PEFT files (f32 safetensors,
    page cache warm) through pinned slot images, and synthetic registration
    (``load_synthetic``: device RNG, no file), the reference's 0.29 ms/adapter arm
    (``src/latefuse/benchmark/churn.py:6-10``)."""
    from safetensors.torch import save_file

    import latefuse_b200 as lf

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hf = bge_m3_config(args.layers)
    cfg = lf.LoraServingConfig(model_name="bge-m3-shape (synthetic)", lora_rank=args.rank, batch_size=args.batch,
                               max_seq_len=args.seq, target_modules=TARGETS, device=dev, dtype=torch.bfloat16,
                               hf_config=hf)
    n_files, n_reg = 8, 200
    store = lf.AdapterStore(cfg, capacity=2 * n_reg + 16)
    key_fn = lf.peft_key_fn("xlm-roberta")
    g = torch.Generator().manual_seed(args.seed)
    with tempfile.TemporaryDirectory() as d:
        dirs = []
        for f in range(n_files):
            sd = {}
            for layer in range(args.layers):
                for m in TARGETS:
                    ka, kb = key_fn(layer, m)
                    sd[ka] = torch.randn(args.rank, 1024, generator=g) * 0.02
                    sd[kb] = torch.randn(1024, args.rank, generator=g) * 0.02
            p = Path(d) / f"a{f}"
            p.mkdir()
            save_file(sd, str(p / "adapter_model.safetensors"))
            (p / "adapter_config.json").write_text(json.dumps({"r": args.rank, "lora_alpha": 2 * args.rank,
                                                               "target_modules": TARGETS}))
            dirs.append(str(p))
        for i in range(n_files):  # warm the page cache and the registrar's pinned images
            lf.load_peft_adapter(store, f"warm{i}", dirs[i])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(n_reg):
            lf.load_peft_adapter(store, f"file{i}", dirs[i % n_files])
        torch.cuda.synchronize()
        file_ms = (time.perf_counter() - t0) * 1e3 / n_reg
    t0 = time.perf_counter()
    for i in range(n_reg):
        store.load_synthetic(f"syn{i}", seed=i)
    torch.cuda.synchronize()
    syn_ms = (time.perf_counter() - t0) * 1e3 / n_reg
    print(json.dumps({
        "mode": "register", "metric": "ms per adapter registration", "higher_is_better": False,
        "adapter_bytes": store.slot_bytes,
        "file_pinned_ms_per_adapter": file_ms,
        "file_pinned_gbs": store.slot_bytes / (file_ms * 1e-3) / 1e9,
        "synthetic_ms_per_adapter": syn_ms,
        "reference_synthetic_ms_per_adapter_a100": 0.29,
        "config": {"workload": f"bge-m3 shape ({args.layers}L, H1024), r={args.rank} on query/key/value/dense, "
                               f"{n_reg} registrations from {n_files} PEFT safetensors files (f32, page cache warm)"},
    }), flush=True)


# ---------------------------------------------------------------------------
# the reference's CPU path (oracle port): the hf engine's per-row bmm hooks
# ---------------------------------------------------------------------------
def build_cpu_reference(args, tenants):
    """A bge-m3-shaped HF model on the CPU (f32, the reference's CPU dtype) with the
    reference's per-row LoRA hooks, restated by the oracle."""
    from transformers import XLMRobertaModel

    from oracle.encoder import HookedEncoder

    hf = bge_m3_config(args.layers)
    with torch.device("meta"):
        model = XLMRobertaModel(hf)
    model = model.to_empty(device="cpu").eval()
    g = torch.Generator().manual_seed(args.seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "LayerNorm.weight" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, 0.02, generator=g)
        for name, b in model.named_buffers():
            if name.endswith("position_ids"):
                b.copy_(torch.arange(b.shape[-1]).expand_as(b))
            else:
                b.zero_()
    H, R, L = 1024, args.rank, args.layers
    adapters = {}
    for t in set(tenants):
        adapters[t] = {"wa": {m: torch.randn(L, H, R, generator=g) * 0.02 for m in TARGETS},
                       "wb": {m: torch.randn(L, R, H, generator=g) * 0.02 for m in TARGETS}}
    return HookedEncoder(model, adapters, TARGETS)


def cpu_baseline(args, steps: int, warmup: int, rows: int) -> dict:
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    ids, mask, tenants = make_inputs(args, args.batch)
    ids, mask, tenants = ids[:rows], mask[:rows], tenants[:rows]
    enc = build_cpu_reference(args, tenants)
    for _ in range(warmup):
        enc.encode_pooled(ids, mask, tenants, "cls")
    t0 = time.perf_counter()
    for _ in range(steps):
        torch.nn.functional.normalize(enc.encode_pooled(ids, mask, tenants, "cls"), dim=-1)
    dt = (time.perf_counter() - t0) / steps
    info = cpu_info()
    return {"value": rows / dt, "unit": "sequences/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of the {args.batch} sequences (padded to {args.seq} as the reference computes), "
                      f"{steps} timed steps after {warmup} warm-up, f32, oracle restatement of the reference hf "
                      f"engine (stock XLM-R forward + per-row bmm LoRA hooks)",
            **info}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    rows = args.cpu_rows
    cpu = cpu_baseline(args, steps=args.steps, warmup=args.warmup, rows=rows)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": cpu["value"],
        "unit": "sequences/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * rows / cpu["value"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (same seeded workload)",
        "config": {"workload": f"bge-m3 shape ({args.layers}L, H1024) embedding forward, LoRA r={args.rank} on "
                               f"query/key/value/dense, reference CPU path on a bounded sample of {rows} sequences "
                               "per step", "global_batch": rows, "seq_len": args.seq, "parallelism": "cpu"},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "sequences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    os.environ.setdefault("HF_HUB_OFFLINE", "1")
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "op":
        run_op(args)
    elif args.mode == "classify":
        run_classify(args)
    elif args.mode == "register":
        run_register(args)
    elif args.mode == "xl":
        run_xl(args)
    elif args.mode == "mixed":
        run_mixed(args)
    else:
        run_serve(args)


if __name__ == "__main__":
    main()
