#!/usr/bin/env python3
"""Benchmark: TriangleMix paged sparse prefill attention on B200.

Workload (one "step" = one prefill attention layer, BASELINE configs 0/3):
  Qwen3-8B geometry (Hq=32, Hkv=8, D=128, page 128), bf16 N(0,1) inputs with
  torch.Generator seed 0, random-permutation block table over 2x pages.
  Default: 8192-token prompt processed as one 8192-token chunk ("prefill_8k").
  --seq-len 32768 --query-tokens 8192 gives the 32K point of config 3.

Multi-GPU (torchrun, one rank per GPU): KV-head partition.  Rank r owns kv
heads [r*8/N, (r+1)*8/N) (query heads x4) of every layer; the job is N
layers, so each rank runs 8 kv-head-layers per step (per-GPU work fixed,
"scaling": "weak").  No collective touches the data path.

Output: one JSON line on rank 0 (see keys in main()).
  value        effective TFLOP/s over all ranks (unmasked QK^T + PV pairs)
  e2e          same metric through the public API with pinned host buffers
               (N = 1: the torch operator; N > 1: each rank's head slices
               through the C ABI), H2D of inputs and D2H of outputs timed
  roofline     dominant kernel vs measured bf16 tensor peak
  cpu_baseline oracle (port of the reference's torch CPU oracle) on a
               bounded row sample, rank 0 only
--impl reference times that CPU oracle on this host instead (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

QUERY_HEADS, KV_HEADS, HEAD_DIM, PAGE = 32, 8, 128, 128
SCALE = HEAD_DIM ** -0.5
METRIC = "TriangleMix prefill attn ms/layer + effective TFLOP/s @8K/32K; TTFT, 1-8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20


def effective_pairs(query_start: int, tq: int, seq: int, prompt: int) -> int:
    """Sum over rows of |key set| (closed form of the reference key sets)."""
    sb, se = 521, max(0, prompt - 128)
    total = 0
    for q in range(query_start, query_start + tq):
        if sb <= q < se:
            total += 8 + 513
        else:
            total += min(q + 1, seq)
    return total


def make_inputs(tq: int, seq: int, seed: int, rank: int = 0, world: int = 1):
    """Seeded host inputs of one full 8-head layer, sliced to this rank's KV heads."""
    from __graft_entry__ import load_package

    gen = torch.Generator().manual_seed(seed)
    logical = math.ceil(seq / PAGE)
    physical = 2 * logical
    perm = torch.randperm(physical, generator=gen)[:logical]
    table = perm.to(torch.int32).view(1, -1).contiguous()
    q = torch.randn(tq, QUERY_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    k = torch.randn(physical, PAGE, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    v = torch.randn(physical, PAGE, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    if world == 1:
        return q, k, v, table
    q, k, v, _ = load_package().sharding.shard_layer(q, k, v, rank, world)
    return q, k, v, table


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons)}


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profiled_traffic(workload: str, heads: int) -> dict | None:
    """DRAM bytes per launch from the committed ncu summary of this workload.

    The summary holds one ``traffic_bytes_per_launch: N`` line measured on the
    full 8-head layer; a head slice moves proportionally fewer bytes.
    """
    path = ROOT / "profiles" / f"tpsa_paged_kernel_{workload}.md"
    if not path.exists():
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", path.read_text(), re.M)
    if m is None:
        return None
    return {"bytes": int(m.group(1)) * heads // KV_HEADS, "source": f"profiles/{path.name}"}


_CPU_INPUTS: dict = {}


def cpu_baseline(tq: int, seq: int, query_start: int, prompt: int, budget_s: float) -> dict:
    """Time the oracle (port of the reference's CPU oracle) on a row sample."""
    from oracle.triangle_oracle import oracle_attention_rowwise, prepare_logical_kv

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    key = (tq, seq)
    if key not in _CPU_INPUTS:  # generated once per workload; not part of the timing
        q, k, v, table = make_inputs(tq, seq, 0)
        t0 = time.perf_counter()
        lkv = prepare_logical_kv(k, v, table, seq)
        _CPU_INPUTS[key] = (q, k, v, table, lkv, time.perf_counter() - t0)
    q, k, v, table, lkv, t_gather = _CPU_INPUTS[key]
    # A seeded random permutation of the rows: any prefix is a uniform sample
    # of dense-prefix, sparse-middle and dense-tail rows.
    order = torch.randperm(tq, generator=torch.Generator().manual_seed(1)).tolist()
    rows, pairs, start, t_rows = [], 0, time.perf_counter(), 0.0
    for i in range(0, tq, 32):
        chunk = order[i:i + 32]
        t0 = time.perf_counter()
        oracle_attention_rowwise(q, k, v, table, query_start, seq, prompt, SCALE, rows=chunk,
                                 logical_kv=lkv)
        t_rows += time.perf_counter() - t0
        pairs += sum(effective_pairs(query_start + r, 1, seq, prompt) for r in chunk)
        rows.extend(chunk)
        if time.perf_counter() - start > budget_s:
            break
    # The one cache gather is charged pro rata to the sampled rows.
    t_compute = t_rows + t_gather * len(rows) / tq
    flops = 4.0 * HEAD_DIM * QUERY_HEADS * pairs
    return {"value": flops / t_compute / 1e12, "unit": "TFLOP/s (effective)", "cores": threads,
            "kind": "port", "seconds": round(t_compute, 3),
            "sample": f"{len(rows)} of {tq} query rows (seeded uniform sample), all 32 heads, "
                      f"torch fp32 per-row gather+softmax, {threads} threads"}


def validate_shards(tm, rank: int, world: int, dev, out_shard, q0: int, seq: int, tq: int):
    """All-gather layer 0's head slices and compare with one full-layer launch."""
    gathered = tm.sharding.gather_output(out_shard, world)
    if rank != 0:
        return None
    q, k, v, table = (t.to(dev) for t in make_inputs(tq, seq, 0))
    full = torch.empty_like(q)
    plan = tm._native.make_plan(tq, q0, seq, seq, KV_HEADS, 0, SCALE)
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=dev)
    tm._native.paged_attention(q, k, v, table, full, q0, seq, seq, SCALE, workspace=ws)
    torch.cuda.synchronize(dev)
    d = (gathered.float() - full.float()).abs()
    return {"max_abs_vs_full_layer": float(d.max()), "mean_abs_vs_full_layer": float(d.mean()),
            "gathered_over": "nccl all_gather"}


def run_reference_arm(args, rank: int) -> None:
    if rank != 0:
        return
    tq, seq = args.query_tokens, args.seq_len
    q0 = seq - tq
    # Each step is a bounded row sample; the whole run stays near 150 s.
    budget = min(args.cpu_budget, 150.0 / (args.warmup + args.steps))
    vals = []
    for _ in range(args.warmup + args.steps):
        vals.append(cpu_baseline(tq, seq, q0, seq, budget))
    timed = vals[args.warmup:]
    value = sum(v["value"] for v in timed) / len(timed)
    pairs = effective_pairs(q0, tq, seq, seq)
    ms = 4.0 * HEAD_DIM * QUERY_HEADS * pairs / (value * 1e12) * 1e3
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s (effective)",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": workload_config(args),
            "cpu_baseline": {**timed[-1], "value": value},
            "e2e": {"value": value, "unit": "TFLOP/s (effective)", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def make_batch_inputs(batch: int, seed: int = 0):
    """B one-chunk prompts, lengths U[2048, 16384] (seeded),
    per-request block tables drawn from one shared random page pool."""
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(2048, 16385, (batch,), generator=gen).tolist()
    logical = [math.ceil(n / PAGE) for n in lens]
    physical = sum(logical) + batch
    perm = torch.randperm(physical, generator=gen).to(torch.int32)
    tables = torch.zeros(batch, max(logical), dtype=torch.int32)
    used = 0
    for i, n in enumerate(logical):
        tables[i, :n] = perm[used:used + n]
        used += n
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    q = torch.randn(cu[-1], QUERY_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    k = torch.randn(physical, PAGE, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    v = torch.randn(physical, PAGE, KV_HEADS, HEAD_DIM, generator=gen).to(torch.bfloat16)
    return lens, cu, q, k, v, tables


def run_batch(args) -> None:
    """Config 4 on one GPU: the whole packed batch per step through
    tpsa_paged_attention_varlen, beside the same requests as batch-one calls."""
    from __graft_entry__ import load_package

    tm = load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lens, cu, q, k, v, tables = make_batch_inputs(args.batch)
    qd, kd, vd, td = q.to(dev), k.to(dev), v.to(dev), tables.to(dev)
    out = torch.empty_like(qd)
    ws = torch.empty(tm._native.varlen_workspace_size(cu, lens, lens), dtype=torch.uint8,
                     device=dev)
    one = [torch.empty(tm._native.make_plan(n, 0, n, n).workspace_bytes, dtype=torch.uint8,
                       device=dev) for n in lens]
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def varlen_step():
        tm._native.paged_attention_varlen(qd, kd, vd, td, out, cu, lens, lens, SCALE,
                                          workspace=ws, stream=stream.cuda_stream)

    def batch_one_step():
        for i, n in enumerate(lens):
            tm._native.paged_attention(qd[cu[i]:cu[i + 1]], kd, vd, td[i:i + 1],
                                       out[cu[i]:cu[i + 1]], 0, n, n, SCALE, workspace=one[i],
                                       stream=stream.cuda_stream)

    def timed(fn) -> float:
        for _ in range(args.warmup):
            flush.fill_(1.0)
            fn()
        torch.cuda.synchronize(dev)
        ms = []
        for i in range(args.steps):
            flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms.append(e0.elapsed_time(e1))
        return sum(ms) / len(ms)

    sampler = ClockSampler(0)
    sampler.start()
    ms_varlen = timed(varlen_step)
    clocks = sampler.stop()
    ms_seq = timed(batch_one_step)
    status = tm._native.device_status(0)
    if status:
        raise RuntimeError(f"device status {status:#x}")
    pairs = sum(effective_pairs(0, n, n, n) for n in lens)
    flops = 4.0 * HEAD_DIM * QUERY_HEADS * pairs
    peaks, peak_kind = load_peaks()
    value = flops / (ms_varlen * 1e-3) / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s (effective)", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_varlen,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16, lengths U[2048,16384])",
            "config": {"workload": f"varlen_batch{args.batch}", "batch": args.batch,
                       "lengths": lens, "tokens": cu[-1],
                       "geometry": "Qwen3-8B attention (Hq=32, Hkv=8, D=128, page 128)",
                       "l2": "flushed between timed steps (256 MiB write)"},
            "gpu_launches": args.steps * ((args.batch + 15) // 16), "clocks": clocks,
            "roofline": {"bound": "tensor", "achieved": value, "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": value / peaks["bf16_tflops"],
                         "traffic": None, "peak_source": f"{peak_kind} bf16_tflops (burst)",
                         "kernel": "tpsa_paged_kernel<false, true>"},
            "batch_one_calls": {"ms_per_step": ms_seq,
                                "value": flops / (ms_seq * 1e-3) / 1e12,
                                "launches_per_step": args.batch}}
    print(json.dumps(line), flush=True)


# (prompt length, scheduler chunk).
CROSSOVER_PROMPTS = ((2869, 512), (4096, 512), (6144, 512), (8192, 512), (8320, 2048))


def flashinfer_paged_prefill(tq: int, seq: int, table, dev):
    """FlashInfer's paged prefill over the same 128-token pages (NHD, the
    BSND cache as is, no gather): causal, bottom-right aligned, GQA 4:1.
    Planned once here; returns fn(q, k_cache, v_cache, out)."""
    import flashinfer

    npages = math.ceil(seq / PAGE)
    ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    wrapper = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD")
    i32 = dict(dtype=torch.int32, device=dev)
    wrapper.plan(torch.tensor([0, tq], **i32), torch.tensor([0, npages], **i32),
                 table[0, :npages].to(**i32).contiguous(),
                 torch.tensor([seq - (npages - 1) * PAGE], **i32),
                 QUERY_HEADS, KV_HEADS, HEAD_DIM, PAGE, causal=True, sm_scale=SCALE,
                 q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)

    def run(q, k_cache, v_cache, out):
        wrapper.run(q, (k_cache, v_cache), out=out)
        return out
    return run


def fa2_gathered(tq: int, seq: int, dev):
    """flash_attn 2 varlen over the context gathered from the pages
    (FlashAttention-2's own paged mode needs 256-token pages); the gather is
    part of the timed call.  Returns fn(q, k_cache, v_cache, table)."""
    from flash_attn import flash_attn_varlen_func

    npages = math.ceil(seq / PAGE)
    cu_q = torch.tensor([0, tq], dtype=torch.int32, device=dev)
    cu_k = torch.tensor([0, seq], dtype=torch.int32, device=dev)

    def run(q, k_cache, v_cache, table):
        pages = table[0, :npages].long()
        kc = k_cache.index_select(0, pages).reshape(-1, KV_HEADS, HEAD_DIM)[:seq]
        vc = v_cache.index_select(0, pages).reshape(-1, KV_HEADS, HEAD_DIM)[:seq]
        return flash_attn_varlen_func(q, kc, vc, cu_q, cu_k, tq, seq, softmax_scale=SCALE,
                                      causal=True)
    return run


def stock_dense(tq: int, seq: int, table, dev) -> tuple[str, object]:
    """The dense paged attention a non-selected layer takes: FlashInfer's
    paged prefill at page 128 when it builds on this box, else flash_attn 2
    over the gathered context.  Returns (name, fn(q, k_cache, v_cache, table))."""
    try:
        fi = flashinfer_paged_prefill(tq, seq, table, dev)
        return "flashinfer_p128", lambda q, k, v, t: fi(q, k, v, torch.empty_like(q))
    except Exception:  # the flash_attn path is the recorded fallback
        fa2 = fa2_gathered(tq, seq, dev)
        return "fa2_gathered", fa2


class CallTimer:
    """Device time of one call: replayed from a CUDA graph (host launch cost
    kept out) when the call can be captured, else launched eagerly; L2 is
    flushed (256 MiB write) before every timed call, outside its events."""

    def __init__(self, dev, errors: list):
        self.dev = dev
        self.stream = torch.cuda.current_stream(dev)
        self.flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        self.errors = errors

    def prepare(self, name: str, fn, warmup: int):
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        self.stream.wait_stream(side)
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                fn()
            torch.cuda.synchronize(self.dev)
            return ("graph", graph)
        except RuntimeError as exc:
            self.errors.append(f"{name}: not captured ({str(exc).splitlines()[0]}); timed eagerly")
            torch.cuda.synchronize(self.dev)
            return ("eager", fn)

    def sample(self, prepared, iterations: int) -> float:
        kind, obj = prepared
        call = obj.replay if kind == "graph" else obj
        events = []
        for i in range(iterations):
            self.flush.fill_(float(i))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            call()
            e1.record(self.stream)
            events.append((e0, e1))
        torch.cuda.synchronize(self.dev)
        ms = sorted(a.elapsed_time(b) for a, b in events)
        return ms[len(ms) // 2]


def run_crossover(args) -> None:
    """BASELINE config 1 on one GPU: every chunk of each chunked prefill timed
    through this library (C ABI, batch-one) against dense causal paged
    attention on the same inputs.  Comparators: FlashInfer's paged prefill at
    page 128 (the stock dense paged attention of a serving engine on B200),
    this kernel's all-dense control (tpsa_paged_attention_dense), and
    flash_attn 2 over a gathered context.  Arms are timed in alternating
    order (ABCD on even repeats, DCBA on odd ones, the reference crossover's
    AB/BA scheme, operator/tests/npu_v2_crossover.py:233-305); each cell
    reports medians, the robust bound min(dense) / max(sparse), and the
    planner's quantities (sparse rows, saved QK pairs per head, reference
    kernel.py:185-269) so the direct-route thresholds can be calibrated."""
    import statistics

    from __graft_entry__ import load_package

    tm = load_package()
    kernel = tm.kernel
    cfg = kernel.TriangleMixConfig(enabled=True, layer_indices=frozenset())
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    errors: list[str] = []
    timer = CallTimer(dev, errors)
    repeats = max(2, args.repeats)
    iterations = max(3, args.steps)
    rows = []
    sampler = ClockSampler(0)
    sampler.start()
    cell = 0
    for prompt, chunk in CROSSOVER_PROMPTS:
        q, k, v, table = make_inputs(prompt, prompt, seed=0)
        qd, kd, vd, td = q.to(dev), k.to(dev), v.to(dev), table.to(dev)
        out_s, out_d, out_f = (torch.empty_like(qd) for _ in range(3))
        per_prompt = {"prompt_len": prompt, "chunk": chunk, "chunks": []}
        for q0 in range(0, prompt, chunk):
            tq = min(chunk, prompt - q0)
            seq = q0 + tq
            span = kernel.triangle_sparse_span(query_len=tq, seq_len=seq, prompt_len=prompt,
                                               config=cfg)
            ws_s = torch.empty(max(256, tm._native.make_plan(tq, q0, seq, prompt).workspace_bytes),
                               dtype=torch.uint8, device=dev)
            ws_d = torch.empty(max(256, tm._native.dense_workspace_size(tq, q0, seq)),
                               dtype=torch.uint8, device=dev)
            qc = qd[q0:seq]
            os_, od, of = out_s[q0:seq], out_d[q0:seq], out_f[q0:seq]
            arms = {
                "sparse": lambda: tm._native.paged_attention(qc, kd, vd, td, os_, q0, seq, prompt,
                                                             SCALE, workspace=ws_s),
                "dense_own": lambda: tm._native.paged_attention_dense(qc, kd, vd, td, od, q0, seq,
                                                                      SCALE, workspace=ws_d),
            }
            try:
                fi = flashinfer_paged_prefill(tq, seq, td, dev)
                arms["flashinfer_p128"] = lambda: fi(qc, kd, vd, of)
            except Exception as exc:  # recorded; the other arms still run
                if not any(e.startswith("flashinfer") for e in errors):
                    errors.append(f"flashinfer: {type(exc).__name__}: {str(exc).splitlines()[0]}")
            try:
                fa2 = fa2_gathered(tq, seq, dev)
                arms["fa2_gathered"] = lambda: fa2(qc, kd, vd, td)
            except Exception as exc:
                if not any(e.startswith("flash_attn") for e in errors):
                    errors.append(f"flash_attn: {type(exc).__name__}: {str(exc).splitlines()[0]}")
            prepared = {n: timer.prepare(n, fn, args.warmup) for n, fn in arms.items()}
            samples: dict[str, list[float]] = {n: [] for n in arms}
            names = list(arms)
            for r in range(repeats):
                order = names if (cell + r) % 2 == 0 else names[::-1]
                for n in order:
                    samples[n].append(timer.sample(prepared[n], iterations))
            cell += 1
            med = {n: statistics.median(v) for n, v in samples.items()}
            rec = {"query_start": q0, "query_len": tq, "seq_len": seq,
                   "sparse_rows": span.sparse_rows, "saved_qk": span.saved_qk,
                   "split": span.is_split, "ms": med,
                   "timing": {n: prepared[n][0] for n in arms},
                   "eligible_reference_thresholds": kernel.triangle_direct_eligible(
                       query_len=tq, seq_len=seq, prompt_len=prompt, config=cfg)}
            for n in arms:
                if n != "sparse":
                    rec[f"speedup_vs_{n}"] = med[n] / med["sparse"]
                    rec[f"robust_vs_{n}"] = min(samples[n]) / max(samples["sparse"])
            if "flashinfer_p128" in arms:
                # Both dense arms compute the same causal attention.
                d = (out_d[q0:seq].float() - out_f[q0:seq].float()).abs()
                rec["dense_own_vs_flashinfer"] = {"max_abs": float(d.max()),
                                                  "mean_abs": float(d.mean())}
            per_prompt["chunks"].append(rec)
            del prepared
        for n in ("sparse", "dense_own", "flashinfer_p128", "fa2_gathered"):
            if all(n in x["ms"] for x in per_prompt["chunks"]):
                per_prompt[f"ms_{n}_all"] = sum(x["ms"][n] for x in per_prompt["chunks"])
        rows.append(per_prompt)
    clocks = sampler.stop()
    status = tm._native.device_status(0)
    if status:
        raise RuntimeError(f"device status {status:#x}")
    stock = "flashinfer_p128" if all("flashinfer_p128" in x["ms"] for r in rows
                                     for x in r["chunks"]) else "fa2_gathered"
    calibration = {}
    for ref_arm in (stock, "dense_own"):
        chunks = [x for r in rows for x in r["chunks"] if x["sparse_rows"] > 0 and ref_arm in x["ms"]]
        losses = [x for x in chunks if x["ms"]["sparse"] >= x["ms"][ref_arm]]
        calibration[ref_arm] = {
            "chunks_with_sparse_rows": len(chunks),
            "sparse_faster": len(chunks) - len(losses),
            "robust_sparse_faster": sum(1 for x in chunks if x[f"robust_vs_{ref_arm}"] > 1.0),
            # Smallest saved-QK threshold above which every measured chunk
            # is faster through this library.
            "min_saved_qk_all_faster": (max(x["saved_qk"] for x in losses) + 1) if losses else 0,
            "losing_chunks": [(x["query_start"], x["seq_len"], x["saved_qk"]) for x in losses]}
    line = {"metric": "TriangleMix chunked-prefill crossover (BASELINE config 1)",
            "unit": "ms per call (median)", "n_gpus": 1, "iterations": iterations,
            "repeats": repeats, "warmup": args.warmup, "data": "synthetic (seeded N(0,1) bf16)",
            "stock_dense": stock,
            "arms": {"sparse": "tpsa_paged_attention (TriangleMix key sets)",
                     "dense_own": "tpsa_paged_attention_dense (same kernel, every row dense)",
                     "flashinfer_p128": "flashinfer BatchPrefillWithPagedKVCacheWrapper, NHD, "
                                        "page 128, causal",
                     "fa2_gathered": "flash_attn 2 varlen over the context gathered from the "
                                     "pages, gather timed"},
            "timing": "per call: CUDA graph replay (else eager), L2 flushed before every call; "
                      "sample = median of iterations; arms in alternating order per repeat",
            "errors": errors, "clocks": clocks, "prompts": rows, "calibration": calibration}
    print(json.dumps(line), flush=True)


# Qwen3-8B geometry, one 8320-token prompt, chunk 2048,
# TriangleMix on layers 5, 7, 10, 15-35.
QWEN3_8B = {"layers": 36, "hidden": 4096, "intermediate": 12288, "vocab": 151936,
            "rope_theta": 1.0e6, "eps": 1e-6}
TTFT_PROMPT, TTFT_CHUNK, TTFT_LAYERS = 8320, 2048, "5,7,10,15-35"


class Qwen3Prefill:
    """Random-init Qwen3-8B (bf16) prefill over a paged KV cache (page 128,
    random block table).  Layers whose index is selected and whose chunk the
    planner's gate admits (reference kernel.py:240-269, this package's B200
    thresholds) run triangle_direct_paged_attention; every other layer runs
    the dense baseline of run_crossover.  Synthetic weights: N(0, 0.02)."""

    def __init__(self, tm, dev, seed: int = 0):
        c = QWEN3_8B
        self.tm, self.dev, self.c = tm, dev, c
        g = torch.Generator(device=dev).manual_seed(seed)
        h, inter, nl = c["hidden"], c["intermediate"], c["layers"]
        qkv = (QUERY_HEADS + 2 * KV_HEADS) * HEAD_DIM

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * 0.02).to(
                torch.bfloat16)

        self.embed = w(c["vocab"], h)
        self.lm_head = w(h, c["vocab"])
        self.layers = [dict(wqkv=w(h, qkv), wo=w(QUERY_HEADS * HEAD_DIM, h), wgu=w(h, 2 * inter),
                            wd=w(inter, h)) for _ in range(nl)]
        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
        self.norm_in = [ones(h) for _ in range(nl)]
        self.norm_post = [ones(h) for _ in range(nl)]
        self.q_norm = [ones(HEAD_DIM) for _ in range(nl)]
        self.k_norm = [ones(HEAD_DIM) for _ in range(nl)]
        self.norm_final = ones(h)
        pages = math.ceil(TTFT_PROMPT / PAGE)
        perm = torch.randperm(2 * pages, generator=torch.Generator().manual_seed(seed))[:pages]
        self.table = perm.to(torch.int32).view(1, -1).to(dev)
        self.kcache = [torch.zeros(2 * pages, PAGE, KV_HEADS, HEAD_DIM, dtype=torch.bfloat16,
                                   device=dev) for _ in range(nl)]
        self.vcache = [torch.zeros_like(k) for k in self.kcache]
        inv = 1.0 / (c["rope_theta"] ** (torch.arange(0, HEAD_DIM, 2, device=dev,
                                                         dtype=torch.float32) / HEAD_DIM))
        ang = torch.arange(TTFT_PROMPT, device=dev, dtype=torch.float32)[:, None] * inv[None]
        self.cos, self.sin = ang.cos(), ang.sin()

    def rmsnorm(self, x, weight):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.c["eps"])).to(
            x.dtype) * weight

    def rope(self, x, p0: int):
        tq = x.shape[0]
        cos = self.cos[p0:p0 + tq, None, :]
        sin = self.sin[p0:p0 + tq, None, :]
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(x.dtype)

    def prefill(self, ids_host, triangle_layers: frozenset, cfg, counts: dict) -> torch.Tensor:
        """One prompt, chunk by chunk; returns the first generated token id (host)."""
        tm, dev, c = self.tm, self.dev, self.c
        kernel = tm.kernel
        ids = ids_host.to(dev, non_blocking=True)
        prompt = ids.shape[0]
        x = None
        for p0 in range(0, prompt, TTFT_CHUNK):
            tq = min(TTFT_CHUNK, prompt - p0)
            seq = p0 + tq
            pos = torch.arange(p0, seq, device=dev)
            slots = (self.table[0, pos // PAGE].long() * PAGE + pos % PAGE)
            x = self.embed[ids[p0:seq]]
            direct = kernel.triangle_direct_eligible(query_len=tq, seq_len=seq, prompt_len=prompt,
                                                     config=cfg)
            dense_name, dense = stock_dense(tq, seq, self.table, dev)
            counts["dense_kind"] = dense_name
            for li in range(c["layers"]):
                lw = self.layers[li]
                hdn = self.rmsnorm(x, self.norm_in[li])
                qkv = hdn @ lw["wqkv"]
                q = qkv[:, :QUERY_HEADS * HEAD_DIM].view(tq, QUERY_HEADS, HEAD_DIM)
                k = qkv[:, QUERY_HEADS * HEAD_DIM:(QUERY_HEADS + KV_HEADS) * HEAD_DIM].view(
                    tq, KV_HEADS, HEAD_DIM)
                v = qkv[:, (QUERY_HEADS + KV_HEADS) * HEAD_DIM:].view(tq, KV_HEADS, HEAD_DIM)
                q = self.rope(self.rmsnorm(q, self.q_norm[li]), p0).contiguous()
                k = self.rope(self.rmsnorm(k, self.k_norm[li]), p0)
                self.kcache[li].view(-1, KV_HEADS, HEAD_DIM)[slots] = k
                self.vcache[li].view(-1, KV_HEADS, HEAD_DIM)[slots] = v
                if li in triangle_layers and direct:
                    attn = torch.empty_like(q)
                    kernel.triangle_direct_paged_attention(
                        query=q, key_cache=self.kcache[li], value_cache=self.vcache[li],
                        block_table=self.table, seq_len=seq, prompt_len=prompt, output=attn,
                        softmax_scale=SCALE, config=cfg)
                    counts["direct"] += 1
                else:
                    attn = dense(q, self.kcache[li], self.vcache[li], self.table)
                    counts["dense"] += 1
                x = x + attn.reshape(tq, -1) @ lw["wo"]
                gu = self.rmsnorm(x, self.norm_post[li]) @ lw["wgu"]
                gate, up = gu.chunk(2, dim=-1)
                x = x + (torch.nn.functional.silu(gate) * up) @ lw["wd"]
        logits = self.rmsnorm(x[-1:], self.norm_final) @ self.lm_head
        return logits.argmax(-1).to("cpu")


def run_ttft(args) -> None:
    """BASELINE config 2 on one GPU: TTFT of one 8320-token prompt (chunk
    2048) with TriangleMix on layers 5, 7, 10, 15-35 against all-dense,
    alternating D-S-S-D (reference ttft_abba.py:73-197).  The timed region
    of a run starts before the token ids' H2D copy and ends after the first
    generated token is on the host (CUDA events on the launching stream)."""
    from __graft_entry__ import load_package

    tm = load_package()
    tm.load_adapter()
    kernel = tm.kernel
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    model = Qwen3Prefill(tm, dev)
    cfg = tm.config.resolve_plugin_config(None).kernel
    layers = kernel.parse_layer_indices(TTFT_LAYERS)
    ids = torch.randint(0, QWEN3_8B["vocab"], (TTFT_PROMPT,),
                        generator=torch.Generator().manual_seed(0)).pin_memory()

    def one(mode: str) -> tuple[float, dict]:
        counts = {"direct": 0, "dense": 0, "dense_kind": None}
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        model.prefill(ids, layers if mode == "triangle" else frozenset(), cfg, counts)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1), counts

    for _ in range(args.warmup):
        one("dense")
        one("triangle")
    times = {"dense": [], "triangle": []}
    counts = {}
    sampler = ClockSampler(0)
    sampler.start()
    for r in range(args.steps):
        order = ("dense", "triangle", "triangle", "dense") if r % 2 == 0 else \
            ("triangle", "dense", "dense", "triangle")
        for mode in order:
            ms, counts[mode] = one(mode)
            times[mode].append(ms)
    clocks = sampler.stop()
    status = tm._native.device_status(0)
    if status:
        raise RuntimeError(f"device status {status:#x}")
    med = {m: sorted(v)[len(v) // 2] for m, v in times.items()}
    line = {"metric": METRIC, "workload": "ttft_qwen3_8b_8320_c2048",
            "value": med["triangle"], "unit": "ms TTFT", "higher_is_better": False,
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "data": "synthetic (random-init Qwen3-8B weights N(0,0.02), uniform random token ids)",
            "dtype": "bf16",
            "config": {"model": "Qwen3-8B geometry (36 layers, hidden 4096, Hq 32, Hkv 8, D 128, "
                                "MLP 12288, vocab 151936, QK-norm, RoPE 1e6)",
                       "prompt": TTFT_PROMPT, "chunk": TTFT_CHUNK, "triangle_layers": TTFT_LAYERS,
                       "thresholds": "b200 profile", "kv_cache": "paged, page 128, random table",
                       "dense_attention": counts["dense"].get("dense_kind")},
            "ttft_ms": {"triangle": med["triangle"], "dense": med["dense"],
                        "speedup": med["dense"] / med["triangle"]},
            "runs_ms": times, "attention_calls_per_prefill": counts, "clocks": clocks,
            "order": "D-S-S-D / S-D-D-S alternating rounds, median per mode"}
    print(json.dumps(line), flush=True)


# Qwen3-8B's architecture for vLLM's dummy-weight loader (random weights, no
# checkpoint): the public model configuration's shape fields.
QWEN3_8B_VLLM_CONFIG = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 4096,
    "intermediate_size": 12288, "num_hidden_layers": 36, "num_attention_heads": 32,
    "num_key_value_heads": 8, "head_dim": 128, "max_position_embeddings": 40960,
    "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "vocab_size": 151936,
    "torch_dtype": "bfloat16", "tie_word_embeddings": False, "hidden_act": "silu",
    "attention_bias": False, "attention_dropout": 0.0, "rope_scaling": None,
    "sliding_window": None, "use_sliding_window": False, "max_window_layers": 36,
    "bos_token_id": 151643, "eos_token_id": 151645}


def ttft_vllm_worker(mode: str, runs: int, warmup: int) -> None:
    """One process of the live-engine TTFT: a vLLM 0.22 engine (in this
    process) with a random-init Qwen3-8B, the plugin registered, TriangleMix
    on (``triangle``) or off (``dense``); prints one JSON line with the TTFT
    of each timed run (wall time of ``generate`` with one output token for
    the 8320-token prompt: five 2048-token prefill steps and the sample)."""
    import tempfile

    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"  # the hook lives in this process
    os.environ.setdefault("VLLM_USE_FLASHINFER_SAMPLER", "0")
    from __graft_entry__ import load_package

    tm = load_package()
    tm.plugin.register()
    model_dir = tempfile.mkdtemp(prefix="qwen3_8b_config_")
    Path(model_dir, "config.json").write_text(json.dumps(QWEN3_8B_VLLM_CONFIG))
    from vllm import LLM, SamplingParams

    section = {"enabled": mode == "triangle", "layers": TTFT_LAYERS, "threshold_profile": "b200"}
    llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, enforce_eager=True,
              dtype="bfloat16", max_model_len=TTFT_PROMPT + 128, block_size=PAGE,
              max_num_batched_tokens=TTFT_CHUNK, enable_chunked_prefill=True,
              enable_prefix_caching=False, gpu_memory_utilization=0.6,
              attention_backend="TRITON_ATTN", seed=0,
              additional_config={"trianglemix": section})
    ids = torch.randint(0, QWEN3_8B["vocab"], (TTFT_PROMPT,),
                        generator=torch.Generator().manual_seed(0)).tolist()
    params = SamplingParams(max_tokens=1, temperature=0.0, detokenize=False)
    prompt = [{"prompt_token_ids": ids}]
    for _ in range(warmup):
        llm.generate(prompt, params, use_tqdm=False)
    router = tm.plugin.registered_router()
    before = dict(router.stats.snapshot()["counters"]) if router else {}
    times = []
    for _ in range(runs):
        t0 = time.perf_counter()
        out = llm.generate(prompt, params, use_tqdm=False)
        times.append((time.perf_counter() - t0) * 1e3)
        assert len(out[0].outputs[0].token_ids) == 1
    after = router.stats.snapshot()["counters"] if router else {}
    per_prefill = {k: (after.get(k, 0) - before.get(k, 0)) / runs for k in sorted(after)
                   if after.get(k, 0) != before.get(k, 0) and not k.endswith("_ns")}
    print("TTFT_VLLM " + json.dumps({"mode": mode, "ttft_ms": times,
                                     "per_prefill": per_prefill,
                                     "status": tm._native.device_status(0)}), flush=True)


def run_ttft_vllm(args) -> None:
    """BASELINE config 2 through a live vLLM engine: TTFT of one 8320-token
    prompt (chunk 2048, block 128) with TriangleMix on layers 5, 7, 10, 15-35
    against vLLM's own attention on every layer.  Rounds of four processes
    in D-S-S-D / S-D-D-S order, each a fresh engine timing ``--steps`` runs
    after ``--warmup`` (reference ttft_abba.py:73-197: alternating process
    order and a bootstrap over rounds).  vLLM 0.22's FlashAttention extension
    is not built in this image, so its attention backend here is the Triton
    one (``TRITON_ATTN``), which the plugin hooks like FlashAttention."""
    import random
    import subprocess

    rounds = max(1, args.rounds)
    per_mode: dict[str, list[float]] = {"dense": [], "triangle": []}
    per_round: list[dict[str, list[float]]] = []
    counts = {}
    for r in range(rounds):
        order = ("dense", "triangle", "triangle", "dense") if r % 2 == 0 else \
            ("triangle", "dense", "dense", "triangle")
        got: dict[str, list[float]] = {"dense": [], "triangle": []}
        for mode in order:
            res = subprocess.run([sys.executable, str(Path(__file__).resolve()),
                                  "--ttft-vllm-worker", mode, "--steps", str(args.steps),
                                  "--warmup", str(args.warmup)],
                                 capture_output=True, text=True, timeout=900)
            lines = [ln for ln in res.stdout.splitlines() if ln.startswith("TTFT_VLLM ")]
            if res.returncode != 0 or not lines:
                raise RuntimeError(f"vLLM worker ({mode}) failed:\n{res.stdout[-2000:]}\n"
                                   f"{res.stderr[-4000:]}")
            rec = json.loads(lines[-1][len("TTFT_VLLM "):])
            if rec["status"]:
                raise RuntimeError(f"device status {rec['status']:#x} in the {mode} worker")
            med = sorted(rec["ttft_ms"])[len(rec["ttft_ms"]) // 2]
            got[mode].append(med)
            per_mode[mode].append(med)
            counts[mode] = rec["per_prefill"]
        per_round.append(got)
    med = {m: sorted(v)[len(v) // 2] for m, v in per_mode.items()}
    # Bootstrap over rounds of the ratio of per-mode means (a round keeps its
    # pair of processes per mode together).
    rng = random.Random(0)
    ratios = []
    for _ in range(2000):
        pick = [per_round[rng.randrange(rounds)] for _ in range(rounds)]
        d = sum(sum(x["dense"]) for x in pick) / sum(len(x["dense"]) for x in pick)
        t = sum(sum(x["triangle"]) for x in pick) / sum(len(x["triangle"]) for x in pick)
        ratios.append(d / t)
    ratios.sort()
    line = {"metric": METRIC, "workload": "ttft_qwen3_8b_8320_c2048_vllm",
            "value": med["triangle"], "unit": "ms TTFT", "higher_is_better": False,
            "n_gpus": 1, "rounds": rounds, "runs_per_process": args.steps, "warmup": args.warmup,
            "data": "synthetic (vLLM dummy-weight Qwen3-8B, uniform random token ids)",
            "dtype": "bf16",
            "config": {"engine": "vLLM 0.22, one process per run set, enforce_eager, prefix "
                                 "caching off, chunked prefill 2048, block 128",
                       "stock_attention": "TRITON_ATTN (vLLM's FlashAttention extension is not "
                                          "built in this image)",
                       "triangle_layers": TTFT_LAYERS, "thresholds": "b200 profile",
                       "prompt": TTFT_PROMPT, "chunk": TTFT_CHUNK},
            "ttft_ms": {"triangle": med["triangle"], "dense": med["dense"],
                        "speedup": med["dense"] / med["triangle"],
                        "speedup_ci95": [ratios[int(0.025 * len(ratios))],
                                         ratios[int(0.975 * len(ratios)) - 1]]},
            "process_medians_ms": per_mode, "attention_calls_per_prefill": counts,
            "order": "D-S-S-D / S-D-D-S rounds of fresh engine processes"}
    print(json.dumps(line), flush=True)


def workload_config(args, seq: int | None = None, tq: int | None = None) -> dict:
    seq = args.seq_len if seq is None else seq
    tq = args.query_tokens if tq is None else tq
    name = "prefill_8k" if seq == 8192 and tq == 8192 else f"prefill_{seq // 1024}k_q{tq}"
    world = args.gpus
    return {"workload": name, "seq_len": seq, "query_tokens": tq, "query_start": seq - tq,
            "prompt_len": seq, "geometry": "Qwen3-8B attention (Hq=32, Hkv=8, D=128, page 128)",
            "parallelism": (f"kv-head partition x{world}: each rank runs its {KV_HEADS // world} "
                            f"KV heads of the one layer" if world > 1 else "one GPU, all 8 KV heads"),
            "layers_per_step": 1,
            "l2": "flushed between timed steps (256 MiB write)"}


class Timer:
    """Steps timed with CUDA events on the launching stream, L2 flushed
    between steps (outside the events), clocks sampled during the timing."""

    def __init__(self, tm, dev, local: int, world: int):
        self.tm, self.dev, self.local, self.world = tm, dev, local, world
        self.stream = torch.cuda.current_stream(dev)
        self.flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier(self):
        if self.world > 1:
            torch.distributed.barrier()

    def max_over_ranks(self, ms: float) -> float:
        if self.world == 1:
            return ms
        t = torch.tensor([ms], device=self.dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def all_ranks(self, ms: float) -> list[float]:
        if self.world == 1:
            return [ms]
        t = torch.tensor([ms], device=self.dev)
        out = [torch.empty_like(t) for _ in range(self.world)]
        torch.distributed.all_gather(out, t)
        return [float(x.item()) for x in out]

    def run(self, step, steps: int, warmup: int) -> tuple[float, dict]:
        """(mean ms per step on this rank, clocks during the timed steps)."""
        for _ in range(warmup):
            self.flush.fill_(1.0)
            step()
        torch.cuda.synchronize(self.dev)
        status = self.tm._native.device_status(self.local)
        if status:
            raise RuntimeError(f"device status {status:#x} after warm-up")
        sampler = ClockSampler(self.local)
        sampler.start()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        self.barrier()
        torch.cuda.synchronize(self.dev)
        for i in range(steps):
            self.flush.fill_(float(i))  # evict L2 between steps (outside the timed events)
            starts[i].record(self.stream)
            step()
            ends[i].record(self.stream)
        torch.cuda.synchronize(self.dev)
        self.barrier()
        clocks = sampler.stop()
        status = self.tm._native.device_status(self.local)
        if status:
            raise RuntimeError(f"device status {status:#x} after timing")
        times = [a.elapsed_time(b) for a, b in zip(starts, ends)]
        return sum(times) / len(times), clocks


def layer_flops(tq: int, seq: int) -> float:
    return 4.0 * HEAD_DIM * QUERY_HEADS * effective_pairs(seq - tq, tq, seq, seq)


def roofline_record(flops: float, kernel_ms: float, workload: str, heads: int,
                    kernel: str) -> dict:
    peaks, peak_kind = load_peaks()
    achieved = flops / (kernel_ms * 1e-3) / 1e12
    rec = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
           "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": None,
           "peak_source": f"{peak_kind} bf16_tflops (burst)", "kernel": kernel,
           "kernel_ms": kernel_ms,
           "algorithmic": "4*128*heads*pairs effective FLOPs per launch"}
    traffic = profiled_traffic(workload, heads)
    if traffic is not None:
        rec["traffic"] = traffic["bytes"]
        rec["traffic_unit"] = "bytes/launch (ncu dram read+write)"
        rec["traffic_source"] = traffic["source"]
    return rec


def measure_layer(tm, timer: Timer, args, tq: int, seq: int, rank: int, world: int,
                  e2e: bool) -> dict:
    """One layer per step: the full 8-head layer on one GPU, or this rank's
    8/N-KV-head slice of it (one tpsa_paged_attention_heads launch)."""
    dev = timer.dev
    q0 = seq - tq
    heads = KV_HEADS // world
    host = make_inputs(tq, seq, 0, rank, world)
    q, k, v, table = (t.to(dev) for t in host)
    out = torch.empty_like(q)
    plan = tm._native.make_plan(tq, q0, seq, seq, heads, 0, SCALE)
    ws = torch.empty(max(plan.workspace_bytes, 256), dtype=torch.uint8, device=dev)
    stream = timer.stream

    def launch(q_, k_, v_, t_, o_):
        tm._native.paged_attention(q_, k_, v_, t_, o_, q0, seq, seq, SCALE,
                                   kv_heads=heads if world > 1 else None, workspace=ws,
                                   stream=stream.cuda_stream)

    ms_rank, clocks = timer.run(lambda: launch(q, k, v, table, out), args.steps, args.warmup)
    per_rank = timer.all_ranks(ms_rank)
    ms = max(per_rank)
    flops = layer_flops(tq, seq)
    rec = {"workload": workload_config(args, seq, tq)["workload"], "ms_per_layer": ms,
           "value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s (effective)",
           "clocks": clocks,
           "roofline": roofline_record(flops * heads / KV_HEADS, ms_rank,
                                       workload_config(args, seq, tq)["workload"], heads,
                                       "tpsa_paged_kernel<false, false>"),
           "plan": {"grid": plan.grid, "items": plan.total_items, "split_tiles": plan.split_tiles,
                    "tiles": plan.total_tiles}}
    if world > 1:
        rec["per_rank_kernel_ms"] = per_rank
    if e2e:
        rec["e2e"] = measure_e2e(tm, timer, args, host, launch, flops, world)
    rec["_out"] = out
    return rec


def measure_e2e(tm, timer: Timer, args, host, launch, flops: float, world: int) -> dict:
    """The same layer through the public API with pinned host buffers: every
    step copies its inputs host -> device and its output back inside the
    timing.  Steps are pipelined as a serving loop runs them: step i + 1's
    inputs go up on a copy stream (into the other of two device buffers) while
    step i computes and its output comes down."""
    dev, stream = timer.dev, timer.stream
    host = tuple(t.pin_memory() for t in host)
    hout = torch.empty_like(host[0]).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = hout.numel() * hout.element_size()
    tq, seq = args.query_tokens, args.seq_len
    q0 = seq - tq
    if world == 1:
        tm.load_adapter()
    copy_stream = torch.cuda.Stream(dev)
    dbufs = [tuple(torch.empty_like(t, device=dev) for t in host) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for ev in free:
        ev.record(stream)

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[b])
            for h, d in zip(host, dbufs[b]):
                d.copy_(h, non_blocking=True)
            ready[b].record(copy_stream)
        stream.wait_event(ready[b])
        dq, dk, dv, dt = dbufs[b]
        if world == 1:
            o = torch.ops.trianglemix_reference.triangle_paged_sparse_attention(
                dq, dk, dv, dt, q0, seq, seq, SCALE)
        else:
            o = torch.empty_like(dq)
            launch(dq, dk, dv, dt, o)
        hout.copy_(o, non_blocking=True)
        free[b].record(stream)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    timer.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    copy_stream.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = timer.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    return {"value": flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s (effective)", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
            "path": ("torch.ops.trianglemix_reference.triangle_paged_sparse_attention"
                     if world == 1 else
                     "C ABI tpsa_paged_attention_heads, each rank its KV-head slice"),
            "pipelining": "step i+1's H2D (copy stream, second device buffer) overlaps "
                          "step i's kernel and D2H"}


def measure_concurrent(tm, timer: Timer, args, rank: int, world: int) -> dict:
    """N concurrent requests (one layer each) at tensor parallelism N: each rank
    runs its 8/N KV heads of all N requests as one varlen launch over one page
    pool, as a serving engine with one KV pool per layer would."""
    dev = timer.dev
    tq, seq = args.query_tokens, args.seq_len
    heads = KV_HEADS // world
    per_req = [make_inputs(tq, seq, j, rank, world) for j in range(world)]
    pages = per_req[0][1].shape[0]
    q = torch.cat([x[0] for x in per_req]).to(dev)
    k = torch.cat([x[1] for x in per_req]).to(dev)
    v = torch.cat([x[2] for x in per_req]).to(dev)
    table = torch.cat([x[3] + j * pages for j, x in enumerate(per_req)]).to(dev)
    out = torch.empty_like(q)
    cu = [tq * j for j in range(world + 1)]
    seqs = [seq] * world
    ws = torch.empty(tm._native.varlen_workspace_size(cu, seqs, seqs, kv_heads=heads),
                     dtype=torch.uint8, device=dev)

    def step():
        tm._native.paged_attention_varlen(q, k, v, table, out, cu, seqs, seqs, SCALE,
                                          kv_heads=heads, workspace=ws,
                                          stream=timer.stream.cuda_stream)

    ms_rank, _ = timer.run(step, args.steps, args.warmup)
    ms = timer.max_over_ranks(ms_rank)
    return {"what": f"{world} concurrent requests of one layer at tensor parallelism {world}: "
                    f"each rank its {heads} KV heads of every request, one varlen launch",
            "ms_per_step": ms, "value": world * layer_flops(tq, seq) / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s (effective, all requests)", "scaling": "weak"}


def run_rank_sweep(args) -> None:
    """One GPU: the launch each rank of an N-GPU KV-head partition runs, for
    N = 1, 2, 4, 8 (ranks 0 and N - 1; the slices are equal in work), at the
    headline context and at 32K/q8K.  Predicts the strong-scaling headline
    of `--gpus N` without N GPUs: the N-GPU step time is the max over ranks
    of these launches."""
    from __graft_entry__ import load_package

    tm = load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    timer = Timer(tm, dev, 0, 1)
    rows = []
    for seq, tq in ((args.seq_len, args.query_tokens), (32768, 8192)):
        base = None
        for world in (1, 2, 4, 8):
            heads = KV_HEADS // world
            per_rank = []
            for rank in sorted({0, world - 1}):
                q, k, v, table = (t.to(dev) for t in make_inputs(tq, seq, 0, rank, world))
                out = torch.empty_like(q)
                plan = tm._native.make_plan(tq, seq - tq, seq, seq, heads, 0, SCALE)
                ws = torch.empty(max(plan.workspace_bytes, 256), dtype=torch.uint8, device=dev)

                def step():
                    tm._native.paged_attention(q, k, v, table, out, seq - tq, seq, seq, SCALE,
                                               kv_heads=heads if world > 1 else None,
                                               workspace=ws)

                ms, clocks = timer.run(step, args.steps, args.warmup)
                per_rank.append(ms)
            ms = max(per_rank)
            base = ms if world == 1 else base
            rows.append({"workload": workload_config(args, seq, tq)["workload"], "n": world,
                         "kv_heads_per_rank": heads, "ms_per_rank": per_rank,
                         "value": layer_flops(tq, seq) / (ms * 1e-3) / 1e12,
                         "efficiency": base / (world * ms), "items": plan.total_items,
                         "split_tiles": plan.split_tiles, "clocks": clocks})
    print(json.dumps({"metric": "KV-head partition: per-rank launch on one B200",
                      "unit": "TFLOP/s (effective, whole layer)", "steps": args.steps,
                      "warmup": args.warmup, "data": "synthetic (seeded N(0,1) bf16)",
                      "rows": rows}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--seq-len", type=int, default=8192)
    ap.add_argument("--query-tokens", type=int, default=None)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-32k", action="store_true",
                    help="skip the second record (the last 8192-token chunk of a 32K prompt)")
    ap.add_argument("--batch", type=int, default=0,
                    help="BASELINE config 4: a packed batch of this many prompts (one GPU)")
    ap.add_argument("--crossover", action="store_true",
                    help="BASELINE config 1: chunked-prefill sweep against the dense baseline "
                         "(one GPU)")
    ap.add_argument("--repeats", type=int, default=5,
                    help="--crossover: alternating-order repeats per chunk")
    ap.add_argument("--ttft", action="store_true",
                    help="BASELINE config 2: Qwen3-8B prefill TTFT, TriangleMix layers against "
                         "all-dense (one GPU)")
    ap.add_argument("--ttft-vllm", action="store_true",
                    help="BASELINE config 2 through a live vLLM engine: D-S-S-D rounds of "
                         "engine processes (one GPU)")
    ap.add_argument("--rounds", type=int, default=2, help="--ttft-vllm: D-S-S-D rounds")
    ap.add_argument("--ttft-vllm-worker", choices=("dense", "triangle"), default=None,
                    help=argparse.SUPPRESS)
    ap.add_argument("--rank-sweep", action="store_true",
                    help="one GPU: time the launch each rank of an N-GPU KV-head partition "
                         "runs, N = 1, 2, 4, 8")
    ap.add_argument("--validate", action="store_true",
                    help="N > 1: all-gather the layer's head slices over NCCL and compare "
                         "them with a full-layer run on rank 0 (outside the timing)")
    args = ap.parse_args()
    if args.query_tokens is None:
        args.query_tokens = min(args.seq_len, 8192)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    if args.crossover:
        if world != 1:
            ap.error("--crossover runs on one GPU")
        run_crossover(args)
        return
    if args.ttft:
        if world != 1:
            ap.error("--ttft runs on one GPU")
        run_ttft(args)
        return
    if args.ttft_vllm_worker:
        ttft_vllm_worker(args.ttft_vllm_worker, args.steps, args.warmup)
        return
    if args.ttft_vllm:
        if world != 1:
            ap.error("--ttft-vllm runs on one GPU")
        run_ttft_vllm(args)
        return
    if args.batch:
        if world != 1:
            ap.error("--batch runs on one GPU")
        run_batch(args)
        return
    if args.rank_sweep:
        if world != 1:
            ap.error("--rank-sweep runs on one GPU")
        run_rank_sweep(args)
        return

    from __graft_entry__ import load_package

    tm = load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    timer = Timer(tm, dev, local, world)
    tq, seq = args.query_tokens, args.seq_len
    # Headline: one layer per step (on N GPUs, split by KV head: strong scaling).
    head = measure_layer(tm, timer, args, tq, seq, rank, world, e2e=not args.no_e2e)
    out = head.pop("_out")
    check = None
    if args.validate and world > 1:
        check = validate_shards(tm, rank, world, dev, out, seq - tq, seq, tq)
    del out
    points = []
    if not args.no_32k and (seq, tq) == (8192, 8192):
        # The "@32K" point of the metric: the last 8192-token chunk of a
        # 32768-token prompt, measured the same way.
        p32 = measure_layer(tm, timer, args, 8192, 32768, rank, world, e2e=False)
        p32.pop("_out")
        points.append(p32)
    concurrent = measure_concurrent(tm, timer, args, rank, world) if world > 1 else None

    line = {"metric": METRIC, "value": head["value"], "unit": "TFLOP/s (effective)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["ms_per_layer"], "ms_per_layer": head["ms_per_layer"],
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16)",
            "config": workload_config(args), "gpu_launches": args.steps,
            "clocks": head["clocks"], "roofline": head["roofline"], "e2e": head.get("e2e"),
            "plan": head["plan"]}
    if world > 1:
        line["per_rank_kernel_ms"] = head["per_rank_kernel_ms"]
        line["concurrent_requests"] = concurrent
    if points:
        line["points"] = points
    if check is not None:
        line["validation"] = check
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(tq, seq, seq - tq, seq, args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
