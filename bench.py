"""Throughput benchmark: MiniLM-L6 sentence embeddings (sentences/s) on 1..8 B200s.

Default workload (configs[3] of the task's baseline): sentences with lengths uniform in
[8, 128] tokens, length-sorted into batches of 1024, packed with cu_seqlens (no padding),
131,072 sentences per GPU per step (so 8 GPUs together process the 1,048,576-sentence
corpus each step); one weight replica per GPU, no inter-GPU traffic in the forward, and
the fp16 [n, 384] embeddings all-gathered over NCCL at the end of each step when N > 1.

A step = one pass of bert_embed over the rank's whole shard. Timing: W untimed warm-up
steps, then K steps between a barrier + cuda synchronize, CUDA events on the launch
stream, max over ranks. One JSON line from rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg3|cfg2|cfg1|cfg0|cfg4]
    python bench.py --impl reference ...   # CPU reference arm (torch fp32 forward, host cores)

Synthetic data: seeded random-init weights of the MiniLM architecture and seeded token ids
stand in for the pretrained checkpoint and the STS corpus (no network here).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "bert-by-hand_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (description, layers, packed, lengths spec, sentences per GPU, batch)
    "cfg3": ("MiniLM-L6 varlen, lengths U[8,128], length-bucketed batches of 1024, packed", 6, True,
             ("uniform", 8, 128), 131072, 1024),
    "cfg2": ("MiniLM-L6 varlen, lengths lognormal(ln 12, 0.555) clipped [5,64] (mean ~14), batches of 1024, packed",
             6, True, ("lognormal",), 131072, 1024),
    "cfg1": ("MiniLM-L6, batch 64 x 9 real tokens padded to seq 128", 6, False, ("fixed", 9, 128), 16384, 64),
    "cfg0": ("MiniLM-L6, batch 64 x 9 real tokens padded to seq 16", 6, False, ("fixed", 9, 16), 16384, 64),
    "cfg4": ("MiniLM-L12, batch 32 x 512 real tokens", 12, False, ("fixed", 512, 512), 1024, 32),
}

# GEMM shapes per token and layer, by kernel kind: (N, K)
GEMM_NK = {"qkv_gemm": (1152, 384), "o_gemm_ln": (384, 384), "ffn1_gemm_gelu": (1536, 384),
           "ffn2_gemm_ln": (384, 1536), "ffn_fused": (1536, 2 * 384)}  # fused: both FFN GEMMs
# algorithmic HBM bytes per token for the memory-bound kernels
MEM_BYTES = {"embed_ln": 8 + 768 + 768, "pool_l2": 768, "attention": 4 * 768}


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def make_lengths(spec, n, seed):
    import synthetic as sy

    if spec[0] == "uniform":
        return sy.lengths_uniform(n, spec[1], spec[2], seed)
    if spec[0] == "lognormal":
        return sy.lengths_lognormal(n, seed)
    return np.full(n, spec[1], np.int32)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic():
    """Per-token DRAM bytes of each kernel kind from a committed ncu capture, if any."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            q = "index,clocks.sm,clocks.max.sm,power.draw," + ",".join(self.FIELDS)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 4 + len(self.FIELDS):
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, v in zip(self.FIELDS, parts[4:]):
                if v.lower() == "active":
                    reasons.add(name.split(".")[-1])
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


_ORACLES = {}


def cpu_forward_rate(workload: str, budget_s: float, seed: int = 99, warm: bool = True):
    """Oracle (torch fp32, CPU) throughput on a bounded sample of the workload.

    Sentences come from the same length distribution; they are length-sorted into batches
    of 64 padded to the batch maximum (the reference's dynamic batching,
    bench/corpus.cu:80-118). Returns (sentences/s, cores, sample description)."""
    import torch

    from oracle import model as om

    desc, layers, packed, spec, _, _ = WORKLOADS[workload]
    torch.set_num_threads(os.cpu_count() or 1)
    if layers not in _ORACLES:
        _ORACLES[layers] = om.Oracle(om.make_weights(0, layers=layers), layers=layers)
    oracle = _ORACLES[layers]
    rng = np.random.default_rng(seed)
    B = 64 if spec[0] != "fixed" or spec[2] <= 128 else 8

    def one_batch():
        lens = np.sort(make_lengths(spec, B, int(rng.integers(1 << 30))))
        S = int(spec[2]) if spec[0] == "fixed" else int(lens.max())
        ids = np.zeros((B, S), np.int32)
        mask = np.zeros((B, S), np.int32)
        for b, L in enumerate(lens):
            ids[b, :L] = om.sentence_ids(rng, int(L))
            mask[b, :L] = 1
        return ids, np.zeros_like(ids), mask

    if warm:
        oracle.embed(*one_batch())
    done, t0 = 0, time.perf_counter()
    while True:
        oracle.embed(*one_batch())
        done += B
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, torch.get_num_threads(), f"{done} sentences in batches of {B} ({dt:.1f} s, torch fp32 CPU oracle)"


def run_reference(args):
    """--impl reference: the reference path's CPU implementation (oracle port) timed on the
    host cores, rank 0 only; K steps, each a bounded sample of the workload."""
    rank = env_int("RANK", 0)
    if rank != 0:
        return
    desc, layers, packed, spec, per_gpu, batch = WORKLOADS[args.workload]
    step_budget = float(os.environ.get("BBH_REF_STEP_SECONDS", "4"))
    rates = []
    cores, sample = 1, ""
    for i in range(args.warmup + args.steps):
        r, cores, sample = cpu_forward_rate(args.workload, step_budget, seed=1000 + i, warm=(i == 0))
        if i >= args.warmup:
            rates.append(r)
    value = statistics.mean(rates)
    line = {
        "impl": "reference", "metric": "sentences/s", "value": round(value, 2), "unit": "sentences/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 * step_budget, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {desc}", "layers": layers, "device": "cpu"},
        "cpu_baseline": {"value": round(value, 2), "unit": "sentences/s", "cores": cores, "kind": "port",
                         "sample": f"per step: {sample}"},
        "e2e": {"value": round(value, 2), "unit": "sentences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="bbh", choices=["bbh", "reference"])
    ap.add_argument("--workload", default="cfg3", choices=sorted(WORKLOADS))
    ap.add_argument("--sentences", type=int, default=0, help="sentences per GPU per step (default: workload's)")
    ap.add_argument("--no-gather", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--lanes", type=int, default=2, choices=[1, 2],
                    help="compute lanes: alternate batches over this many workspaces / streams")
    ap.add_argument("--gemm-pairs", type=int, default=1, choices=[0, 1, 2],
                    help="GEMM tiles: 0 = one SM per 128-row tile, 1 = SM pairs 256x192 (default), "
                         "2 = SM pairs 256x256 where N allows")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import bbh
    import synthetic as sy

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    desc, layers, packed, spec, per_gpu, batch = WORKLOADS[args.workload]
    n = args.sentences or per_gpu
    weights = sy.random_weights(0, layers)
    bbh.set_gemm_pairs(args.gemm_pairs)
    gw = bbh.ModelWeights.from_numpy(weights, layers, local)

    lengths = make_lengths(spec, n, seed=3 + 7919 * rank)
    corpus = sy.bucketed_corpus(lengths, batch, seed=3 + 104729 * rank)
    max_tokens = max(b.tokens for b in corpus.batches)
    max_len = int(lengths.max())
    if not packed:
        S = spec[2]
        max_tokens = batch * S
        max_len = S
    ws = bbh.Workspace(gw, max_tokens, batch, max_len)
    lanes = [ws] + [bbh.Workspace(gw, max_tokens, batch, max_len) for _ in range(args.lanes - 1)]
    ws.set_corpus_lanes(args.lanes)

    i32 = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.int32, device=dev)
    emb = torch.empty((n, 384), dtype=torch.float16, device=dev)
    if packed:
        d_ids, d_types = i32(corpus.ids), i32(corpus.types)
        d_cu = [i32(b.cu) for b in corpus.batches]
    else:
        S = spec[2]
        L = spec[1]
        pid = np.zeros((n, S), np.int32)
        pid[:, :L] = sy.sentence_tokens(np.full(n, L, np.int32), 3 + rank).reshape(n, L)
        pmask = np.zeros((n, S), np.int32)
        pmask[:, :L] = 1
        d_ids, d_types, d_mask = i32(pid), i32(np.zeros_like(pid)), i32(pmask)
    stream = torch.cuda.current_stream(dev)
    lane_streams = [stream] + [torch.cuda.Stream(dev) for _ in range(args.lanes - 1)]

    def forward_all(nlanes=None):
        # batch bi runs on lane bi % nlanes (its own workspace and stream); the current
        # stream orders the lanes' work before and after
        nl = nlanes or len(lanes)
        for ls in lane_streams[1:nl]:
            ls.wait_stream(stream)
        for bi, b in enumerate(corpus.batches):
            out = emb[b.first:b.first + b.count]
            lw, lst = lanes[bi % nl], lane_streams[bi % nl]
            if packed:
                lw.embed_varlen(d_ids[b.tok_start:b.tok_start + b.tokens], d_types[b.tok_start:b.tok_start + b.tokens],
                                d_cu[bi], b.max_len, out=out, stream=lst)
            else:
                lw.embed(d_ids[b.first:b.first + b.count], d_types[b.first:b.first + b.count],
                         d_mask[b.first:b.first + b.count], out=out, stream=lst)
        for ls in lane_streams[1:nl]:
            stream.wait_stream(ls)

    gather = world > 1 and not args.no_gather
    gathered = torch.empty((world * n, 384), dtype=torch.float16, device=dev) if gather else None

    def step():
        forward_all()
        if gather:
            dist.all_gather_into_tensor(gathered, emb)

    def sync_all():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-resident timed region ----------------
    for _ in range(args.warmup):
        step()
    if ws.device_error() != 0:
        raise RuntimeError("device flagged an input error")
    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                          if os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    sync_all()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    sync_all()
    clock_info = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    total_sentences = n * world * args.steps
    value = total_sentences / (ms / 1000.0)
    launches = args.steps * len(corpus.batches) * ws.launches_per_forward

    # ---------------- end to end through the public API, host buffers ----------------
    # Packed workloads: bbh_embed_corpus over the host corpus (pinned double-buffered
    # staging, H2D of ids/types/cu_seqlens, one graph replay per batch, D2H of the
    # embeddings to corpus order), timed on the host around the call, which returns when
    # every embedding is in host memory. Padded workloads: bbh_embed_padded (the same
    # staging around one bert_embed per batch of consecutive sentences).
    h2d = d2h = 0
    if packed:
        # the synthetic corpus stores its sentences length-sorted: sentence i has length
        # lengths[corpus.order[i]]
        offsets = np.zeros(n + 1, np.int64)
        offsets[1:] = np.cumsum(lengths[corpus.order])
        plan = bbh.plan_batches(np.diff(offsets).astype(np.int32), batch, max_tokens, 1)
        h_emb_np = np.zeros((n, 384), np.float16)
        host_ids, host_types = np.ascontiguousarray(corpus.ids), np.ascontiguousarray(corpus.types)

        def e2e_step():
            ws.embed_corpus(host_ids, host_types, offsets, plan, out=h_emb_np)

        sent_len = np.diff(offsets)
        for _, idx in plan.batches():
            h2d += 8 * int(sent_len[idx].sum()) + 4 * (len(idx) + 1)
        d2h = 768 * n
    else:
        host_ids = np.ascontiguousarray(pid, dtype=np.int32)
        host_types = np.zeros_like(host_ids)
        host_mask = np.ascontiguousarray(pmask, dtype=np.int32)
        h_emb_np = np.zeros((n, 384), np.float16)

        def e2e_step():
            # bert_embed per batch of the padded host corpus as one library call: pinned staging, copy
            # streams and compute lanes inside bbh_embed_padded
            ws.embed_padded(host_ids, host_types, host_mask, batch, out=h_emb_np)

        h2d = 12 * n * spec[2]
        d2h = 768 * n

    e2e_step()
    sync_all()
    e2e_steps = max(1, min(args.steps, 5))
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step()
    sync_all()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0) / e2e_steps
    e2e_value = n * world / (e2e_ms / 1000.0)

    # ---------------- per-kernel timing pass (same workload, eager, CUDA events) ----------------
    ws.set_kernel_timing(True)
    tok_per_step = int(sum(b.tokens for b in corpus.batches)) if packed else n * spec[2]
    kt_steps = 1
    for _ in range(kt_steps):
        forward_all(nlanes=1)
    kt = ws.kernel_times()
    ws.set_kernel_timing(False)
    hbm, tf_burst, tf_sust, peak_src = measured_peaks()
    per_kernel = {}
    for k, (kms, cnt) in kt.items():
        if cnt == 0:
            continue
        entry = {"ms_total": round(kms, 3), "launches": int(cnt), "us_per_launch": round(1000 * kms / cnt, 2)}
        toks = tok_per_step * kt_steps
        if k in GEMM_NK:
            N, K = GEMM_NK[k]
            entry["tflops"] = round(2.0 * toks * layers * N * K / (kms / 1000.0) / 1e12, 1)
        elif k in MEM_BYTES:
            entry["gbs"] = round(MEM_BYTES[k] * toks * (layers if k == "attention" else 1) / (kms / 1000.0) / 1e9, 1)
        per_kernel[k] = entry
    total_k = sum(v["ms_total"] for v in per_kernel.values())
    for v in per_kernel.values():
        v["share"] = round(v["ms_total"] / total_k, 3)
    dom = max(per_kernel, key=lambda k: per_kernel[k]["ms_total"])
    dk = per_kernel[dom]
    traffic = profiled_traffic()
    if dom in GEMM_NK:
        N, K = GEMM_NK[dom]
        achieved = dk["tflops"]
        peak = tf_sust
        unit, bound = "TFLOP/s", "tensor"
        tr = traffic.get(dom)
        traffic_b = round(tr["bytes_per_token"] * tok_per_step * kt_steps / dk["launches"]) if tr else None
    else:
        achieved = dk["gbs"]
        peak = hbm
        unit, bound = "GB/s", "hbm"
        tr = traffic.get(dom)
        traffic_b = round(tr["bytes_per_token"] * tok_per_step * kt_steps / dk["launches"]) if tr else None
    roofline = {"bound": bound, "kernel": dom, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": round(achieved / peak, 3), "traffic": traffic_b,
                "peak_source": f"{peak_src} ({'bf16 sustained' if bound == 'tensor' else 'hbm copy'})"}

    # ---------------- CPU baseline (rank 0, N = 1) ----------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, sample = cpu_forward_rate(args.workload, args.cpu_seconds)
        cpu = {"value": round(r, 2), "unit": "sentences/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        mean_len = float(lengths.mean()) if packed else float(spec[1])
        line = {
            "metric": "sentences/s", "value": round(value, 1), "unit": "sentences/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (seeded random-init MiniLM weights; token ids U[1000,30521] with [CLS]/[SEP])",
            "config": {
                "workload": f"{args.workload}: {desc}", "layers": layers, "sentences_per_gpu": n,
                "global_sentences_per_step": n * world, "batch": batch, "mean_len": round(mean_len, 2),
                "tokens_per_gpu_step": tok_per_step, "packed": packed, "parallelism": f"dp{world} (batch-sharded replicas)",
                "gather": "NCCL all_gather of fp16 embeddings each step" if gather else "none",
                "l2": "inputs larger than L2 (each step streams ~1 GB of activations per GPU)",
                "graph": "one CUDA graph per workspace, re-pointed per batch",
                "lanes": f"{args.lanes} (batches alternate over {args.lanes} workspaces / streams)",
                "gemm_tiles": ["one SM per 128-row tile", "SM pairs, 256x192", "SM pairs, 256x256 where N allows"][args.gemm_pairs],
            },
            "roofline": roofline,
            "kernels": per_kernel,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 1), "unit": "sentences/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "steps": e2e_steps,
                    "note": ("bbh_embed_corpus: host corpus -> pinned double-buffered staging -> H2D -> forward -> "
                             "D2H to corpus order, host-timed around the call" if packed else
                             "bbh_embed_padded: host ids/types/mask -> pinned double-buffered staging -> H2D -> bert_embed per batch -> D2H, host-timed around the call")},
            "gpu_launches": int(launches),
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
