#!/usr/bin/env python
"""Serving benchmark: bge-m3-shaped mixed-tenant embedding with 10,000 resident rank-16 adapters.

Workload (one step = one batch through the hot path): a bge-m3 / XLM-R-large
shaped encoder (24 layers, hidden 1024, 16 heads, FFN 4096, vocab 250002),
seeded random init, bf16; LoRA rank 16 on query / key / value / attention-output
dense; 10,000 synthetic adapters (A, B ~ N(0, 0.02)) resident in the slot cache;
a batch of 64 sequences padded to 512 tokens with real lengths uniform in
[32, 512]; tenant ids Zipf(1.1) over the 10,000; CLS pooling + L2 normalisation.
Synthetic seeded data of that shape stands in for real requests.

Metric: sequences/s of the whole job (``value``, inputs resident in HBM, device
timed) and the fused LoRA kernels' achieved HBM bandwidth against the measured
peak (``roofline``), with the same metric end to end through the public API
from pinned host buffers (``e2e``) and the reference's CPU path timed on the
host cores (``cpu_baseline``).

    python bench.py [--gpus N --steps K --warmup W]          # this implementation
    python bench.py --impl reference [--steps K --warmup W]  # the reference's CPU path

N > 1 runs under torchrun, one process per GPU, each GPU with its own replica of
the model and the 10,000-adapter cache and its own 64-row batch (weak scaling);
the embeddings are all-gathered over NCCL every step.  Prints one JSON line.
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
# DRAM bytes (read + write) of one LoRA op, averaged over the q/k/v op (182.85 MB) and the
# dense op (70.34 MB) of the bge-m3 step at r=16, from one ncu capture of the same launch
# shapes (the serve-traffic summary under profiles/ holds the command and the table).
NCU_TRAFFIC_PER_OP_R16 = (182.85e6 + 70.34e6) / 2
# DRAM bytes of one fused q/k/v projection launch (lf_linear_lora) of the same step, from one
# ncu capture (profiles/ holds the command and the table).
NCU_TRAFFIC_QKV_GEMM_R16 = 45.25e6 + 51.91e6
TARGETS = ["query", "key", "value", "dense"]
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0


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
    ap.add_argument("--mode", choices=["serve", "op"], default="serve",
                    help="serve: the bge-m3 embedding workload; op: the isolated LoRA op "
                         "Y = X W + (X A_t) B_t at X (64, 256, 1024), one JSON line per rank value")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--adapters", type=int, default=10000)
    ap.add_argument("--rank", type=int, default=16)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--min-len", type=int, default=32)
    ap.add_argument("--cpu-rows", type=int, default=2, help="sequences per CPU-baseline step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--ranks", default="8,16,64", help="--mode op: LoRA ranks to measure")
    ap.add_argument("--persistent", type=int, default=1, help="0: per-tile expand kernel only")
    ap.add_argument("--no-pack", action="store_true", help="serve: run the padded forward instead of the packed one")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------
def measured_hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s for a kernel timed inside a long step: the sustained figure."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return (float(json.loads(p.read_text())["bf16_tflops_sustained"]),
                    "measured (MEASURED_PEAKS.json bf16_tflops_sustained)")
        except Exception:
            pass
    return FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback (sustained)"


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"latefuse_b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
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

    def mark(self, begin: bool) -> None:
        """Wall-clock bounds of the timed region: only samples inside it count."""
        if begin:
            self.t_begin = time.time()
        else:
            self.t_end = time.time()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        import datetime

        t0, t1 = getattr(self, "t_begin", None), getattr(self, "t_end", None)
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
            if t0 is not None and t1 is not None and not (t0 <= ts <= t1):
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


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_inputs(args, rank: int):
    from latefuse_b200.synthetic import ragged_batch, zipf_tenants

    ids, mask = ragged_batch(args.batch, args.seq, min_len=min(args.min_len, args.seq), max_len=args.seq,
                             vocab=250002, pad_id=1, cls_id=0, low_id=5, seed=args.seed + rank)
    tenants = zipf_tenants(args.adapters, args.batch, alpha=1.1, seed=args.seed + rank)
    return ids, mask, [f"adapter_{int(t)}" for t in tenants]


def build_ours(args, dev):
    import latefuse_b200 as lf

    hf = bge_m3_config(args.layers)
    cfg = lf.LoraServingConfig(model_name="bge-m3-shape (synthetic)", lora_rank=args.rank, batch_size=args.batch,
                               max_seq_len=args.seq, target_modules=TARGETS, device=dev, dtype=torch.bfloat16,
                               hf_config=hf)
    model = lf.EncoderWithLora.random_init(hf, cfg, seed=args.seed)
    store = lf.AdapterStore(cfg, capacity=args.adapters)
    store.fill_random_(args.adapters, std=0.02, generator=torch.Generator(device=dev).manual_seed(args.seed + 1))
    emb = lf.MultiTenantEmbedder(cfg, engine="bert", model=model, store=store, tokenizer=False)
    return emb


def lora_bytes_per_step(segs, n_unique: int, layers: int, H: int, R: int) -> tuple[int, int]:
    """Algorithmic HBM bytes of the LoRA ops of one step (bf16): per layer the
    q/k/v op reads x once and reads+writes 3 output slices, the dense op reads x
    and reads+writes 1 slice, over the real (segment) tokens; plus each unique
    tenant's A and B factors once per module."""
    T = segs.real_tokens
    e = 2
    qkv = T * H * e + 3 * 2 * T * H * e + n_unique * 3 * 2 * H * R * e
    dense = T * H * e + 2 * T * H * e + n_unique * 2 * H * R * e
    return layers * (qkv + dense), 2 * layers


def run_ours(args):
    import torch.distributed as dist

    import latefuse_b200 as lf
    from latefuse_b200 import _native as nat

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    emb = build_ours(args, dev)
    model, store = emb.model, emb.store
    ids, mask, tenants = make_inputs(args, rank)
    lengths = mask.sum(1).tolist()
    ids_d, mask_d = ids.to(dev), mask.to(dev)
    batch = emb._get_assembler().batch_lora(tenants, args.seq, lengths)
    packed = None if args.no_pack else model.pack(ids, lengths, store.slots(tenants))
    emb.pack_tokens = packed is not None
    H = emb.config.hidden_size
    gathered = torch.empty(world * args.batch, H, dtype=torch.bfloat16, device=dev) if world > 1 else None

    def step():
        with torch.no_grad():
            if packed is not None:
                pooled = model.encode_pooled_packed(packed, store, pooling="cls")
            else:
                pooled = model.encode_pooled(ids_d, mask_d, batch, pooling="cls")
            out = lf.head.l2_normalize(pooled)
            if world > 1:
                dist.all_gather_into_tensor(gathered, out)
        return out

    # clocks are sampled from the warm-up on (nvidia-smi takes a moment to start);
    # only the samples inside the timed region are reported
    clocks = ClockSampler(list(range(torch.cuda.device_count())) if rank == 0 else [])
    clocks.__enter__()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    emb.check_device_status()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- device-timed region: inputs resident in HBM ----
    model.lora_events = []
    n0 = nat.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clocks.mark(True)
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    barrier()
    clocks.mark(False)
    clocks.__exit__(None, None, None)
    launches = nat.launch_count() - n0
    ms = start.elapsed_time(end) / args.steps
    events = model.lora_events
    model.lora_events = None
    by_kind: dict[str, list[float]] = {}
    for kind, s_ev, e_ev in events:
        by_kind.setdefault(kind, []).append(s_ev.elapsed_time(e_ev))
    lora_ms_step = sum(sum(v) for v in by_kind.values()) / args.steps
    fused = "qkv_gemm" in by_kind
    gemm_ms = statistics.median(by_kind["qkv_gemm"]) if fused else 0.0
    shrink_ms_step = sum(sum(by_kind.get(k, [])) for k in ("qkv_shrink", "dense_shrink")) / args.steps
    if world > 1:
        t = torch.tensor([ms, lora_ms_step, gemm_ms, shrink_ms_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, lora_ms_step, gemm_ms, shrink_ms_step = t.tolist()
    emb.check_device_status()

    segs = packed.segments if packed is not None else batch.segments
    n_unique = len(set(tenants))
    bytes_step, ops_step = lora_bytes_per_step(segs, n_unique, args.layers, H, args.rank)
    achieved = bytes_step / (lora_ms_step * 1e-3) / 1e9
    peak, peak_src = measured_hbm_peak()
    if fused:
        # the dominant kernel of this library: the q/k/v projection GEMM with the LoRA
        # delta in its accumulator (tensor-bound); and the shrink launches (HBM-bound)
        T_tok = segs.n_tokens
        R = args.rank
        gemm_flops = 2.0 * T_tok * 3 * H * (H + R)
        tpeak, tpeak_src = measured_tensor_peak()
        tach = gemm_flops / (gemm_ms * 1e-3) / 1e12
        n_blk = (T_tok + 127) // 128 + segs.n_segs
        shrink_bytes_step = args.layers * sum(
            T_tok * H * 2 + n_unique * m * H * R * 2 + m * n_blk * 128 * R * 2 for m in (3, 1))
        shrink_gbs = shrink_bytes_step / (shrink_ms_step * 1e-3) / 1e9
        roofline = {
            "bound": "tensor", "achieved": tach, "peak": tpeak, "unit": "TFLOP/s", "frac": tach / tpeak,
            "traffic": (NCU_TRAFFIC_QKV_GEMM_R16 if packed is not None and args.rank == 16 and args.batch == 64
                        and args.seq == 512 else None),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one lf_linear_lora q/k/v "
                              "launch of this workload (output writes still in L2 at kernel end not counted)",
            "kernel": "lf_linear_lora: q/k/v projection (T x 3072 x 1024) with the per-row LoRA delta in the "
                      "tcgen05 accumulator (one launch per layer)",
            "algorithmic_flops_per_launch": gemm_flops, "launch_ms": gemm_ms, "peak_source": tpeak_src,
        }
        lora_hbm = {
            "kernel": "lf_lora_shrink_blocked (per layer: q/k/v and attention-output shrinks)",
            "achieved": shrink_gbs, "peak": peak, "unit": "GB/s", "frac": shrink_gbs / peak,
            "algorithmic_bytes_per_step": shrink_bytes_step, "ms_per_step": shrink_ms_step, "peak_source": peak_src,
            "note": "the expand no longer exists as a kernel: the delta (u and B reads, K = rank MMAs) runs inside "
                    "the projection GEMM",
        }
    else:
        roofline = {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": (NCU_TRAFFIC_PER_OP_R16 if packed is not None and args.rank == 16 and args.batch == 64
                        and args.seq == 512 else None),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per LoRA op (shrink + expand) "
                              "of this workload; y writes still in L2 at kernel end are not counted",
            "kernel": "LoRA delta op = tcgen05 shrink + expand launches (per layer: q/k/v op, dense op)",
            "algorithmic_bytes_per_op": bytes_step / ops_step,
            "op_ms": lora_ms_step / ops_step,
            "peak_source": peak_src,
        }
        lora_hbm = None

    # ---- end to end through the public API from pinned host buffers ----
    e2e = None
    if not args.no_e2e:
        ids_h, mask_h = ids.pin_memory(), mask.pin_memory()
        out_h = torch.empty(args.batch, H, dtype=torch.bfloat16).pin_memory()
        # what embed_tokens copies to the device each step: the packed token
        # tables and segment table, or the padded ids/mask and segment table
        h2d = (packed.host_bytes if packed is not None
               else ids_h.numel() * 8 + mask_h.numel() * 8 + segs.host.numel() * 4)
        d2h = out_h.numel() * 2

        def e2e_step():
            vec = emb.embed_tokens(ids_h, mask_h, tenants)
            if world > 1:
                dist.all_gather_into_tensor(gathered, vec)
            out_h.copy_(vec, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        for _ in range(args.warmup):
            e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        barrier()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = t.item()
        e2e = {"value": world * args.batch / (e2e_ms * 1e-3), "unit": "sequences/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "MultiTenantEmbedder.embed_tokens(pinned host ids/mask, tenant ids) -> pinned host embeddings"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args, steps=3, warmup=1, rows=args.cpu_rows)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": world * args.batch / (ms * 1e-3),
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
                "Zipf(1.1) tenants, lengths U[32,512])",
        "config": {
            "workload": f"bge-m3 shape ({args.layers}L, H1024, 16 heads, FFN 4096, vocab 250002) bf16 embedding "
                        f"forward, LoRA r={args.rank} on query/key/value/attention-output dense, {args.adapters} "
                        f"resident adapters, batch {args.batch}x{args.seq} right-padded (lengths "
                        f"U[{args.min_len},{args.seq}]), Zipf(1.1) tenants, CLS pooling + L2 norm",
            "global_batch": world * args.batch,
            "seq_len": args.seq,
            "real_tokens_per_gpu_step": segs.real_tokens,
            "padded_tokens_per_gpu_step": args.batch * args.seq,
            "tokens_computed": "real tokens only (packed, attention per sequence)" if packed is not None
                               else "all padded positions (LoRA on real tokens only)",
            "parallelism": f"dp{world}",
            "adapters": args.adapters,
            "rank": args.rank,
            "unique_tenants_per_batch": n_unique,
            "l2": "inputs larger than L2: every step streams 1.1 GB of weights and >0.5 GB of activations",
        },
        "roofline": roofline,
        "lora_share_of_step": lora_ms_step / ms,
        "lora_share_note": ("shrink + fused projection GEMM launches (the GEMM includes the base projection)"
                            if fused else "shrink + expand launches"),
        "gpu_launches": launches,
        "gpu_launches_per_step": launches / args.steps,
        "clocks": clocks.summary(),
    }
    if lora_hbm is not None:
        line["lora_hbm"] = lora_hbm
    if e2e is not None:
        line["e2e"] = e2e
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


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
    ids, mask, tenants = make_inputs(args, 0)
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
            "sample": f"{rows} of the 64 sequences (padded to {args.seq} as the reference computes), {steps} timed "
                      f"steps after {warmup} warm-up, f32, oracle restatement of the reference hf engine "
                      f"(stock XLM-R forward + per-row bmm LoRA hooks)",
            **info}


def run_op(args):
    """The isolated op at (64, 256, 1024) bf16: base GEMM plus the late-fusion delta
    with 10,000 resident adapters and Zipf(1.1) tenants.  Reports the delta's
    achieved HBM bandwidth (algorithmic bytes 3*T*H*2 + U*4*H*r) and the whole op."""
    from latefuse_b200 import _native as nat
    from latefuse_b200.lora import FactorCache, SegmentTable, lora_apply, lora_expand, lora_shrink, workspace_bytes
    from latefuse_b200.synthetic import zipf_tenants

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    nat.set_option(nat.LF_OPT_PERSISTENT, args.persistent)
    B, S, H = 64, 256, 1024
    T = B * S
    g = torch.Generator(device=dev).manual_seed(args.seed)
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
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > L2, written between steps

        def op(times=None):
            torch.matmul(x, w, out=y)
            if times is not None:
                times[0].record()
            lora_apply(x, y, fc, segs, [0], [0], ws)
            if times is not None:
                times[1].record()

        for _ in range(args.warmup):
            op()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        ops = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        n0 = nat.launch_count()
        for i in range(args.steps):
            flush.zero_()
            ops[i][0].record()
            op(ev[i])
            ops[i][1].record()
        torch.cuda.synchronize()
        delta_ms = statistics.median(a.elapsed_time(b) for a, b in ev)
        op_ms = statistics.median(a.elapsed_time(b) for a, b in ops)
        launches = (nat.launch_count() - n0) / args.steps
        # each launch of the delta on its own (same inputs, L2 flushed before each)
        u = ws[: T * R * 2].view(torch.bfloat16).view(1, T, R)
        sh, ex = [], []
        for _ in range(args.steps):
            for fn, acc in ((lambda: lora_shrink(x, u, fc, segs, [0]), sh),
                            (lambda: lora_expand(u, y, fc, segs, [0], [0], True), ex)):
                flush.zero_()
                a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a_.record()
                fn()
                b_.record()
                acc.append((a_, b_))
        torch.cuda.synchronize()
        shrink_ms = statistics.median(a.elapsed_time(b) for a, b in sh)
        expand_ms = statistics.median(a.elapsed_time(b) for a, b in ex)
        U = len(set(slots))
        algo = 3 * T * H * 2 + U * 4 * H * R
        flops = 2 * T * H * H + 4 * T * H * R
        peak, src = measured_hbm_peak()
        out[f"r{R}"] = {"delta_us": delta_ms * 1e3, "delta_gbs": algo / (delta_ms * 1e-3) / 1e9,
                        "delta_frac_of_hbm": algo / (delta_ms * 1e-3) / 1e9 / peak, "algorithmic_bytes": algo,
                        "unique_tenants": U, "op_us": op_ms * 1e3, "op_tflops": flops / (op_ms * 1e-3) / 1e12,
                        "shrink_us": shrink_ms * 1e3, "shrink_gbs": (T * H * 2 + U * 2 * H * R) / (shrink_ms * 1e-3) / 1e9,
                        "expand_us": expand_ms * 1e3,
                        "expand_gbs": (2 * T * H * 2 + U * 2 * H * R) / (expand_ms * 1e-3) / 1e9,
                        "launches_per_op": launches}
        del cache, x, y, w, ws, flush
        torch.cuda.empty_cache()
    print(json.dumps({"mode": "op", "workload": "Y = X W + (X A_t) B_t, X (64,256,1024) bf16, "
                      f"{args.adapters} adapters, Zipf(1.1) tenants, L2 flushed between steps",
                      "peak_gbs": measured_hbm_peak()[0], "results": out}), flush=True)


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
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
