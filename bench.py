#!/usr/bin/env python
"""bench.py -- BASELINE metric: bs1 MXFP4 decode tok/s (TinyLlama shape), with the
FP4 GEMV's HBM GB/s against the measured peak.

Workload: random-init TinyLlama-shape MXFP4 decoder (22 L,
d 2048, ffn 5632, 32q/4kv, hd 64, V 32000, theta 1e4, eps 1e-5), bf16 KV cache,
16-token seeded prompt, greedy decode.  One STEP = one decode token at batch 1
(one pass of the whole model: 549.5 MB of MXFP4 weights, > the 126 MB L2, so
no flush is needed between steps).  The prompt is prefilled before warm-up; the
default --warmup 7 --steps 120 covers decode positions 16..142, i.e. the
reference's timed tokens of a 128-token generation (llama_run/src/main.rs:554-562).

  value      device-timed decode tok/s (CUDA events on the launching stream
             around K graph replays; max over ranks; N>1 runs N independent
             replicas -- the path does not shard at this shape)
  e2e        the same metric through the public C-ABI call llama_generate with
             HOST prompt/ids (H2D + D2H inside the timed region), 16+128 tokens
             per call, prefill included
  roofline   weight bytes per token / device time per token vs MEASURED_PEAKS
  gemv       config 0: 5632x2048 MXFP4 GEMV, bf16 x, over 64 rotated weight
             copies (394 MB > L2), GB/s vs measured HBM peak
  cpu_baseline  the C oracle (restated reference CPU loops) on the host cores

--impl reference times the reference's own CPU path (the oracle port of its
loops; the Rust/cuda-oxide reference cannot be built here) on the same config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for p in (REPO, REPO / "rust-fp4-blackwell_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = "bs1 MXFP4 decode tok/s (TinyLlama shape)"
UNIT = "tok/s"
N_PROMPT, N_GEN = 16, 128


def tinyllama_cfg(max_seq=2048):
    from fp4x.engine import TINYLLAMA
    return dict(TINYLLAMA, max_seq=max_seq)


def measured_peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def hbm_peak():
    pk = measured_peaks()
    if "hbm_gbs" in pk:
        return float(pk["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons of this process's GPU, polled through NVML
    every 5 ms while the timed region runs (read-only queries; nvidia-smi's 200 ms
    floor would miss a sub-second region).  The device is found by PCI bus id."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.sm, self.bits, self.max_mhz = [], 0, None
        self.err = None
        self._stop = threading.Event()
        self.t = None

    def _handle(self, nv):
        import torch
        pr = torch.cuda.get_device_properties(self.cuda_index)
        for fmt in ("{:08x}:{:02x}:{:02x}.0", "{:04x}:{:02x}:{:02x}.0"):
            try:
                return nv.nvmlDeviceGetHandleByPciBusId(fmt.format(pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id))
            except Exception:
                pass
        return nv.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def __enter__(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv, self.h = nv, self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception as e:  # no NVML: report no samples rather than fail the bench
            self.err = repr(e)
        return self

    def _run(self):
        nv, h = self.nv, self.h
        while not self._stop.is_set():
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                self.bits |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
            except Exception as e:
                self.err = repr(e)
                return
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        reasons = []
        if self.t:
            reasons = [name for name, attr in self.REASONS if self.bits & int(getattr(self.nv, attr, 0))]
        out = {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
               "reasons": reasons, "samples": len(self.sm), "source": "nvml"}
        if self.err:
            out["error"] = self.err
        return out


def traffic_per_token():
    """dram__bytes_read.sum + dram__bytes_write.sum per token of the decode kernel, from
    the ncu capture recorded in profiles/dram_traffic.json (keyed by decode path; the
    file also holds the capture command).  Paths without a capture map to None."""
    try:
        rec = json.loads((REPO / "profiles" / "dram_traffic.json").read_text())
    except Exception:
        return {}
    out = {}
    for path, r in rec.get("decode", {}).items():
        out[path] = (r["dram_bytes_read"] + r["dram_bytes_write"]) / r["tokens"]
    return out

DTYPES = {
    "tensor": "e2m1xe8m0 weights x 8-term e2m1xe8m0 activation on tcgen05 kind::mxf4 (exact products, "
              "fp32 accumulate), bf16 KV",
    "persistent": "e2m1xe8m0 weights, f32 activations (f16 hi/lo mma.sync operands), bf16 KV",
    "graph": "e2m1xe8m0 weights, f32 activations (f16 hi/lo mma.sync operands), bf16 KV",
}


def cpu_baseline_port(cfg, budget_s=20.0, threads=0):
    """Oracle forward (reference CPU loops, OpenMP over rows) on a bounded sample."""
    import oracle
    threads = threads if threads > 0 else host_cores()
    m = oracle.Model(cfg, threads=threads)
    from fp4x import synth
    prompt = synth.prompt_for(cfg)
    t0 = time.perf_counter()
    m.forward(int(prompt[0]), 0)
    first = time.perf_counter() - t0
    n = max(2, min(64, cfg["max_seq"] - 2, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    tok = int(prompt[1])
    for pos in range(1, 1 + n):
        nxt, _ = m.forward(tok, pos)
        tok = int(prompt[pos + 1]) if pos + 1 < len(prompt) else nxt
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} single-token forwards (positions 1..{n}) of the TinyLlama-shape MXFP4 model, "
                      f"C oracle of the reference loops, OpenMP over rows"}


def host_cores() -> int:
    """Host threads this process may run on (torchrun sets OMP_NUM_THREADS=1 for its
    workers, so the OpenMP default is not the box's core count)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference's CPU path on the whole host: one process over every host core
    (rank 0; under torchrun the other ranks exit without work).  N GPU replicas on
    this box would share the same cores, so the line is the host's CPU throughput
    at every N."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    cfg = tinyllama_cfg()
    cores = host_cores()
    m = oracle.Model(cfg, threads=cores)
    from fp4x import synth
    prompt = synth.prompt_for(cfg)
    # prefill (untimed) then W warm-up and K timed decode tokens, as our arm
    tok = int(prompt[0])
    pos = 0
    for pos in range(N_PROMPT):
        nxt, _ = m.forward(int(prompt[pos]), pos)
    tok, pos = nxt, N_PROMPT
    for _ in range(args.warmup):
        tok, _ = m.forward(tok, pos)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok, _ = m.forward(tok, pos)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    v = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights -> MXFP4, seeded uniform prompt ids)",
        "config": {"workload": "config1: TinyLlama-shape MXFP4 decode, bs1, 16-token prompt, greedy",
                   "batch": 1, "prompt": N_PROMPT, "positions": f"{N_PROMPT}..{N_PROMPT + args.warmup + args.steps - 1}"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": "the whole --steps run: single-token forwards of the C restatement of the "
                                   "reference CPU loops (Rust/cuda-oxide reference not buildable here), one "
                                   f"process over all {cores} host cores (OpenMP over rows), rank 0 only"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


C3_LINEARS = {"qkv": (2560, 2048), "o": (2048, 2048), "gate_up": (11264, 2048), "down": (2048, 5632),
              "lm_head": (32000, 2048)}


def run_config3(args):
    """fp4_mma (tcgen05 kind::mxf4) on the TinyLlama linears x M tokens
    (16/64/256 decode batches, 512-token prefill), MXFP4 N(0,1) activations, fp32
    accumulate, bf16 out.  Each (M, linear) is a CUDA graph of calls over rotated weight
    copies (> 300 MB, so weights come from HBM), timed with CUDA events."""
    import torch
    from fp4x import check, lib, ops
    L = lib()
    peak, peak_kind = hbm_peak()
    ms = [int(x) for x in args.c3_m.split(",")]
    names = args.c3_linears.split(",")
    rows, tot_flop, tot_us = [], 0.0, 0.0
    for m in ms:
        for name in names:
            n, k = C3_LINEARS[name]
            wbytes = n * k // 2 + n * k // (16 if args.c3_format == "nvf4" else 32)
            copies = max(2, -(-(300 << 20) // wbytes))
            nv = args.c3_format == "nvf4"
            if nv:  # NVFP4: one quantised matrix, cloned into distinct copies (L2 rotation)
                w0 = ops.quantize_nvfp4(ops.fill_normal(n * k, seed=100, sigma=0.02).view(n, k), 1.0 / 4096.0)
                ws = [(w0[0].clone(), w0[1].clone()) for _ in range(copies)]
                a, sa = ops.quantize_nvfp4(ops.fill_normal(m * k, seed=7, sigma=1.0).view(m, k), 1.0 / 64.0)
                wsb = L.fp4_mma_nvf4_workspace_size(m, n, k)
            else:
                ws = [ops.init_mxfp4(n, k, seed=100 + i) for i in range(copies)]
                a, sa = ops.init_mxfp4(m, k, seed=7, sigma=1.0)
                wsb = L.fp4_mma_workspace_size(m, n, k)
            d = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
            wsp = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())

            def call(p, sc):
                if nv:
                    check(L.fp4_mma_nvf4(s.cuda_stream, m, n, k, a.data_ptr(), sa.data_ptr(), p.data_ptr(),
                                         sc.data_ptr(), 1.0 / 262144.0, d.data_ptr(), wsp.data_ptr(), wsb))
                else:
                    check(L.fp4_mma(s.cuda_stream, m, n, k, a.data_ptr(), sa.data_ptr(), p.data_ptr(), sc.data_ptr(),
                                    d.data_ptr(), wsp.data_ptr(), wsb))
            with torch.cuda.stream(s):
                call(*ws[0])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for p, sc in ws:
                    call(p, sc)
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            st = torch.cuda.current_stream()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(args.steps):
                g.replay()
            e1.record(st)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (args.steps * copies)
            byts = wbytes + m * k // 2 + m * k // (16 if args.c3_format == "nvf4" else 32) + m * n * 2
            flop = 2.0 * m * n * k
            rows.append({"m": m, "linear": name, "n": n, "k": k, "us": round(us, 2), "gbs": round(byts / us / 1e3, 1),
                         "tflops": round(flop / us / 1e6, 1), "split_k": wsb > 0})
            if m == ms[-1]:
                tot_flop += flop
                tot_us += us
            del ws, g
            torch.cuda.empty_cache()
    fmt = "NVFP4 " if args.c3_format == "nvf4" else ""
    line = {"metric": f"fp4_mma {fmt}config3: TinyLlama linears at M={ms[-1]} tokens", "value": tot_flop / tot_us / 1e6,
            "unit": "TFLOP/s", "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
            "dtype": ("e2m1 x e2m1 (UE4M3 block-16 scales), fp32 accumulate, bf16 out" if fmt else
                      "e2m1 x e2m1 (E8M0 block-32 scales), fp32 accumulate, bf16 out"),
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations -> MXFP4)",
            "config": {"workload": "config3", "tokens": ms, "linears": names,
                       "l2": "rotated weight copies > 300 MB per graph"},
            "hbm_peak_gbs": peak, "peak_kind": peak_kind, "table": rows}
    print(json.dumps(line), flush=True)
    return 0


def run_config2(args):
    """batched bf16 flash-decode (llama_attn_decode_bf16 through the
    C ABI): GQA 32q/4kv hd 64 and 32q/8kv hd 128, contexts 512..32768, batch 1/8/64.
    Per shape a CUDA graph of calls over enough rotated KV caches to exceed 300 MB (or
    one cache when it is larger), CUDA-event timed.  Bytes = K + V read + q + out."""
    import torch
    from fp4x import check, lib, ops
    L = lib()
    peak, peak_kind = hbm_peak()
    shapes = [(32, 4, 64), (32, 8, 128)]
    ctxs = [int(x) for x in args.c2_ctx.split(",")]
    batches = [int(x) for x in args.c2_batch.split(",")]
    rows = []
    for (H, KV, hd) in shapes:
        for B in batches:
            for T in ctxs:
                cache = B * T * KV * hd * 2 * 2
                if cache > (24 << 30):
                    continue
                copies = max(1, min(16, -(-(300 << 20) // cache)))
                kvs = []
                for i in range(copies):
                    kc = ops.fill_normal(B * T * KV * hd, seed=10 + 2 * i, dtype=torch.bfloat16).view(B, T, KV, hd)
                    vc = ops.fill_normal(B * T * KV * hd, seed=11 + 2 * i, dtype=torch.bfloat16).view(B, T, KV, hd)
                    kvs.append((kc, vc))
                q = ops.fill_normal(B * H * hd, seed=3, dtype=torch.bfloat16).view(B, H, hd)
                out = torch.empty_like(q)
                nbytes = L.llama_attn_workspace_size(B, H, KV, hd, T)
                ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())

                def call(kc, vc):
                    check(L.llama_attn_decode_bf16(s.cuda_stream, B, H, KV, hd, T, T, q.data_ptr(), kc.data_ptr(),
                                                   vc.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes))
                with torch.cuda.stream(s):
                    call(*kvs[0])
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for kc, vc in kvs:
                        call(kc, vc)
                for _ in range(args.warmup):
                    g.replay()
                torch.cuda.synchronize()
                st = torch.cuda.current_stream()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                for _ in range(args.steps):
                    g.replay()
                e1.record(st)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (args.steps * copies)
                byts = cache + 2 * B * H * hd * 2
                rows.append({"heads": f"{H}q/{KV}kv", "hd": hd, "batch": B, "ctx": T, "us": round(us, 2),
                             "gbs": round(byts / us / 1e3, 1), "frac": round(byts / us / 1e3 / peak, 3),
                             "in_l2": copies * cache <= (100 << 20)})
                del kvs, g
                torch.cuda.empty_cache()
    big = [r for r in rows if not r["in_l2"]]
    line = {"metric": "flash-decode attention config2: HBM fraction (caches > L2)",
            "value": max(r["frac"] for r in big) if big else None, "unit": "fraction of measured HBM GB/s",
            "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
            "dtype": "bf16 q/K/V/out, fp32 softmax", "data": "synthetic N(0,1) bf16",
            "config": {"workload": "config2", "shapes": ["32q/4kv hd64", "32q/8kv hd128"], "ctx": ctxs,
                       "batch": batches, "l2": "rotated caches > 300 MB where a cache is smaller"},
            "hbm_peak_gbs": peak, "peak_kind": peak_kind, "table": rows}
    print(json.dumps(line), flush=True)
    return 0


def run_config4(args):
    """Llama-3-8B-shape MXFP4 decoder, tensor-parallel over the
    torchrun ranks (1 process per GPU; in-graph NVLink peer-memory allreduce after O
    and down, cross-rank argmax), batch 1, greedy decode at a 4096-token context.
    The context is 4096 positions of zero-filled KV cache (attention reads all of
    them; the prompt's values do not change the work), so no 4096-token prefill is
    timed.  Step = one decode token of the whole TP group; value = tokens / max
    over ranks of the device time."""
    import datetime
    import torch
    import torch.distributed as dist
    from fp4x import engine, tp
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    ctx = args.c4_ctx
    cfg = dict(engine.LLAMA3_8B, max_seq=ctx + args.warmup + args.steps + 8)
    m = tp.create_model(cfg) if world > 1 else engine.Model(cfg)
    path = m.path
    m.forward(1, ctx - 1, want_logits=False)  # device state: position ctx - 1 done
    m.decode_steps(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(st)
        m.decode_steps(args.steps)
        e1.record(st)
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e-3
    if world > 1:
        tt = torch.tensor([t], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    wbytes = m.weight_bytes()  # this rank's shard
    m.close()
    if rank == 0:
        peak, peak_kind = hbm_peak()
        per_tok = t / args.steps
        line = {"metric": "config4 Llama-3-8B-shape MXFP4 decode tok/s (batch 1, TP)", "value": args.steps / t,
                "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": per_tok * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": DTYPES.get(path, path), "data": "synthetic (seeded N(0,0.02) weights -> MXFP4)",
                "config": {"workload": "config4", "batch": 1, "context": ctx, "tp": world, "path": path,
                           "kv": "zero-filled cache of ctx positions (prefill not timed)"},
                "roofline": {"bound": "hbm", "kernel": f"decode token ({path} path), rank 0 shard",
                             "achieved": wbytes / per_tok / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": wbytes / per_tok / 1e9 / peak, "bytes_per_launch": wbytes,
                             "peak_kind": peak_kind},
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_batch(args):
    """Batched decode through the llama_batch engine (every linear on the tcgen05
    fp4_mma GEMM, 8-term MXFP4 activations): BASELINE config 4 at batch 64
    (--batch-model llama8b --batch-ctx 4096) or the TinyLlama shape.  Every
    sequence starts at a context of --batch-ctx positions of zero-filled KV cache
    (prefill not timed); step = one token of every sequence; value = tokens of
    all sequences / device time.  Bytes per step = MXFP4 weights + the bf16 K/V
    rows every sequence reads (at the mean position of the timed steps)."""
    import datetime
    import torch
    import torch.distributed as dist
    from fp4x import engine, tp
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    base = engine.LLAMA3_8B if args.batch_model == "llama8b" else engine.TINYLLAMA
    B, ctx = args.batch, args.batch_ctx
    terms = 4 if os.environ.get("FP4X_BATCH_TERMS") == "4" else 8
    cfg = dict(base, max_seq=ctx + args.warmup + args.steps + 8)
    m = tp.create_model(cfg) if world > 1 else engine.Model(cfg)
    b = tp.create_batch(m, B) if world > 1 else engine.Batch(m, B)
    for s in range(B):
        b.set_length(s, ctx, (17 + 31 * s) % cfg["vocab"])
    b.decode(args.warmup)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        if args.profile_region:
            torch.cuda.profiler.start()
        e0.record(st)
        b.decode(args.steps)
        e1.record(st)
        torch.cuda.synchronize()
        if args.profile_region:
            torch.cuda.profiler.stop()
    t = e0.elapsed_time(e1) * 1e-3
    if world > 1:
        tt = torch.tensor([t], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    wbytes = m.weight_bytes()  # this rank's shard
    kvd = cfg["n_kv_heads"] * cfg["head_dim"] // world
    mean_seq = ctx + args.warmup + (args.steps + 1) / 2
    kv_bytes = B * mean_seq * cfg["n_layers"] * kvd * 2 * 2
    per_step = t / args.steps
    peak, peak_kind = hbm_peak()
    b.close()
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {"metric": f"batched MXFP4 decode tok/s ({args.batch_model} shape, batch {B})", "value": B * args.steps / t,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"e2m1xe8m0 weights x {terms}-term e2m1xe8m0 activations on tcgen05 kind::mxf4 -> f32",
            "data": "synthetic (seeded N(0,0.02) weights -> MXFP4)",
            "config": {"workload": "config4-batch" if args.batch_model == "llama8b" else "tinyllama-batch",
                       "batch": B, "context": ctx, "tp": world,
                       "kv": "zero-filled cache of ctx positions per sequence (prefill not timed)",
                       "l2": "weights and KV caches far above L2 (no flush needed)"},
            "roofline": {"bound": "hbm", "kernel": "batched decode step (fp4_mma + attention), rank 0 shard",
                         "achieved": (wbytes + kv_bytes) / per_step / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": (wbytes + kv_bytes) / per_step / 1e9 / peak,
                         "bytes_per_step": wbytes + kv_bytes, "weight_bytes": wbytes, "kv_bytes": kv_bytes,
                         "peak_kind": peak_kind},
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


def tp_section(args, rank, world, torch, dist):
    """BASELINE config 4 over the job's ranks (tensor parallel at TP = world; one
    process per GPU, the library's NVLink peer-memory allreduce after O and down):
      parity  a 2-layer model of the 8B shape (every real dimension): each rank's
              logits slice over 3 positions, gathered on rank 0 and compared with
              the CPU oracle's full logits (rms-floor relative error, greedy token);
      bs1     batch-1 greedy decode at a 4096-token context (zero-filled KV);
      bs64    64 sequences at a 4096-token context through the batched engine.
    Times are CUDA events on the launching stream, max over ranks.  Every rank takes
    the same steps in the same order; rank 0 returns the summary."""
    from fp4x import engine, tp
    import numpy as np
    import datetime
    group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300)) if dist else None
    st = torch.cuda.current_stream()
    out = {"tp": world, "model": "llama3-8b shape, MXFP4, random init", "context": args.tp_ctx}

    def barrier():
        if dist:
            dist.barrier(group=group)

    def make(cfg):
        return tp.create_model(cfg, group=group) if dist else engine.Model(cfg)

    def max_over_ranks(t):
        if dist:
            tt = torch.tensor([t], dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
            t = float(tt.item())
        return t

    # parity at reduced depth
    pcfg = dict(engine.LLAMA3_8B, n_layers=2, max_seq=16)
    toks = [int(t) for t in np.random.default_rng(4).integers(0, pcfg["vocab"], 3)]
    m = make(pcfg)
    v0, _ = m.shard()
    mine = []
    for pos, t in enumerate(toks):
        nxt, lg = m.forward(t, pos)
        mine.append((nxt, v0, lg))
    m.close()
    parts = [None] * world
    if dist:
        dist.all_gather_object(parts, mine, group=group)
    else:
        parts = [mine]
    if rank == 0:
        import oracle
        ref = oracle.Model(pcfg, threads=host_cores())
        worst, same = 0.0, True
        for pos, t in enumerate(toks):
            rn, rl = ref.forward(t, pos)
            full = np.empty_like(rl)
            for pr in parts:
                _, a, lg = pr[pos]
                full[a:a + len(lg)] = lg
            rms = float(np.sqrt(np.mean(rl.astype(np.float64) ** 2)))
            worst = max(worst, float(np.max(np.abs(full.astype(np.float64) - rl) / np.maximum(np.abs(rl), rms))))
            same = same and all(pr[pos][0] == rn for pr in parts)
        ref.close()
        out["parity"] = {"layers": 2, "positions": len(toks), "max_rel_logits": worst, "tol": 1e-2,
                         "greedy_tokens_equal": bool(same), "vs": "CPU oracle (reference loops restated)"}
    barrier()

    # batch 1 at the full depth
    ctx = args.tp_ctx
    cfg = dict(engine.LLAMA3_8B, max_seq=ctx + args.warmup + max(args.tp_steps, args.tp_bsteps) + 8)
    m = make(cfg)
    out["path_bs1"] = m.path
    m.forward(1, ctx - 1, want_logits=False)
    m.decode_steps(args.warmup)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    m.decode_steps(args.tp_steps)
    e1.record(st)
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3)
    out["bs1_tok_s"] = args.tp_steps / t
    out["bs1_ms_per_token"] = 1e3 * t / args.tp_steps
    out["bs1_steps"] = args.tp_steps
    out["weight_bytes_per_rank"] = m.weight_bytes()

    # batch 64
    B = args.tp_batch
    b = tp.create_batch(m, B, group=group) if dist else engine.Batch(m, B)
    for s in range(B):
        b.set_length(s, ctx, (17 + 31 * s) % cfg["vocab"])
    b.decode(args.warmup)
    torch.cuda.synchronize()
    barrier()
    e0.record(st)
    b.decode(args.tp_bsteps)
    e1.record(st)
    torch.cuda.synchronize()
    t = max_over_ranks(e0.elapsed_time(e1) * 1e-3)
    out[f"bs{B}_tok_s"] = B * args.tp_bsteps / t
    out[f"bs{B}_ms_per_step"] = 1e3 * t / args.tp_bsteps
    out[f"bs{B}_steps"] = args.tp_bsteps
    b.close()
    m.close()
    torch.cuda.synchronize()
    barrier()
    if dist:
        dist.destroy_process_group(group)
    return out if rank == 0 else None


def gemv_config0(torch, peak):
    """Config 0 GEMV (fp4_gemv through the C ABI) over 64 rotated weight copies,
    captured in one CUDA graph (no host launch gaps), CUDA-event timed."""
    from fp4x import ops
    n, k, copies = 5632, 2048, 64
    ws = [ops.init_mxfp4(n, k, seed=1000 + i) for i in range(copies)]
    x = ops.fill_normal(k, seed=2, sigma=1.0, dtype=torch.bfloat16)
    y = torch.empty(n, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for p, sc in ws[:4]:
            ops.gemv(p, sc, x, out=y)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for p, sc in ws:
            ops.gemv(p, sc, x, out=y)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = 10
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / (reps * copies) * 1e-3
    # one launch at a time (each bracketed by its own events, weights not in L2 since
    # the 63 other copies ran in between): the kernel without the graph's launch chain
    singles = []
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ws]
    with torch.cuda.stream(s):
        for (a, b), (p, sc) in zip(ev, ws):
            a.record(s)
            ops.gemv(p, sc, x, out=y)
            b.record(s)
    torch.cuda.synchronize()
    singles = sorted(a.elapsed_time(b) * 1e3 for a, b in ev)
    nbytes = n * k // 2 + n * k // 32 + k * 2 + n * 4
    gbs = nbytes / per / 1e9
    del g, ws
    return {"workload": "config0: MXFP4 GEMV 5632x2048, bf16 x, f32 y, 64 rotated weight copies (394 MB > L2) "
                        "in one CUDA graph",
            "bytes_per_launch": nbytes, "us_per_launch": per * 1e6, "achieved_gbs": gbs, "peak_gbs": peak,
            "frac": gbs / peak, "us_single_launch_median": singles[len(singles) // 2],
            "single_launch_note": "each of the 64 copies launched alone between two events on one stream"}


def run_config0(args):
    """BASELINE config 0 alone: fp4_gemv 5632x2048 over 64 rotated weight copies in
    one CUDA graph (the `gemv` key of the default line), printed as its own line."""
    import torch
    peak, peak_kind = hbm_peak()
    with ClockSampler(torch.cuda.current_device()) as clk:
        g = gemv_config0(torch, peak)
    line = {"metric": "config0 fp4_gemv 5632x2048 HBM GB/s", "value": g["achieved_gbs"], "unit": "GB/s",
            "higher_is_better": True, "us_per_launch": g["us_per_launch"],
            "roofline": {"bound": "hbm", "achieved": g["achieved_gbs"], "peak": peak, "unit": "GB/s",
                         "frac": g["frac"], "bytes_per_launch": g["bytes_per_launch"], "peak_kind": peak_kind},
            "dtype": "e2m1xe8m0 weights, bf16 x, f32 accumulate", "data": "synthetic (seeded N(0,0.02) -> MXFP4)",
            "config": {"workload": g["workload"]}, "detail": g, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=7)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--config3", action="store_true", help="fp4_mma sweep of BASELINE config 3 instead of decode")
    ap.add_argument("--c3-m", default="16,64,256,512")
    ap.add_argument("--config2", action="store_true", help="attention sweep of BASELINE config 2 instead of decode")
    ap.add_argument("--config4", action="store_true", help="Llama-3-8B-shape TP decode (torchrun ranks) instead")
    ap.add_argument("--config0", action="store_true", help="the config-0 fp4_gemv measurement alone")
    ap.add_argument("--c4-ctx", type=int, default=4096)
    ap.add_argument("--c2-ctx", default="512,2048,8192,32768")
    ap.add_argument("--c2-batch", default="1,8,64")
    ap.add_argument("--c3-linears", default=",".join(C3_LINEARS))
    ap.add_argument("--c3-format", default="mxf4", choices=["mxf4", "nvf4"],
                    help="operand format of the config-3 sweep (NVFP4: UE4M3 scales per 16)")
    ap.add_argument("--batch", type=int, default=0, help="batched decode of this many sequences instead")
    ap.add_argument("--batch-model", default="llama8b", choices=["llama8b", "tinyllama"])
    ap.add_argument("--batch-ctx", type=int, default=4096)
    ap.add_argument("--no-tp", action="store_true", help="skip the config-4 tensor-parallel section")
    ap.add_argument("--tp-ctx", type=int, default=4096)
    ap.add_argument("--tp-steps", type=int, default=32, help="timed batch-1 tokens of the TP section")
    ap.add_argument("--tp-bsteps", type=int, default=8, help="timed batch steps of the TP section")
    ap.add_argument("--tp-batch", type=int, default=64)
    ap.add_argument("--profile-region", action="store_true",
                    help="bracket the timed region with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    args = ap.parse_args()
    assert args.warmup >= 3, "timing rules: at least 3 warm-up steps"
    if args.impl == "reference":
        return run_reference(args)
    if args.config3:
        return run_config3(args)
    if args.config2:
        return run_config2(args)
    if args.config4:
        return run_config4(args)
    if args.config0:
        return run_config0(args)
    if args.batch:
        return run_batch(args)

    import torch
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    from fp4x import engine, ops, synth
    positions = N_PROMPT + args.warmup + args.steps + 1
    cfg = tinyllama_cfg(max_seq=max(2048, positions + 8))
    model = engine.Model(cfg)
    prompt = synth.prompt_for(cfg, N_PROMPT)
    peak, peak_kind = hbm_peak()

    # prefill the prompt (device-resident loop); the last prompt position yields token 1
    model.generate(prompt, 1)
    model.decode_steps(args.warmup)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(st)
        model.decode_steps(args.steps)  # K tokens of the device-resident loop
        e1.record(st)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t = e0.elapsed_time(e1) * 1e-3
    if dist:
        tt = torch.tensor([t], device="cuda", dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    value = world * args.steps / t
    per_tok = t / args.steps
    wbytes = model.weight_bytes()
    model_path = model.path
    achieved = wbytes / per_tok / 1e9
    kpt = model.kernels_per_token() if model.path == "graph" else 1

    e2e = None
    if not args.no_e2e:
        # public API with host buffers: llama_generate(prompt host -> ids host), 16 + 128 tokens
        model.reset()
        model.generate(prompt, N_GEN)  # warm
        reps = 2
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            model.reset()
            model.generate(prompt, N_GEN)
        torch.cuda.synchronize()
        te = time.perf_counter() - t0
        if dist:
            tt = torch.tensor([te], device="cuda", dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            te = float(tt.item())
        e2e = {"value": world * reps * N_GEN / te, "unit": UNIT,
               "h2d_bytes_per_step": (N_PROMPT * 4 + 20) / N_GEN, "d2h_bytes_per_step": 4,
               "call": "llama_generate(host prompt[16] -> host ids[128]) incl. prefill, KV reset between calls"}

    gemv = None
    if rank == 0:
        gemv = gemv_config0(torch, peak)
    model.close()
    torch.cuda.synchronize()

    tpres = None
    if not args.no_tp:
        try:
            tpres = tp_section(args, rank, world, torch, dist)
        except Exception as e:  # the config-1 line above is still reported
            tpres = {"tp": world, "error": f"{type(e).__name__}: {e}"[:300]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_port(tinyllama_cfg(max_seq=128))

    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_tok * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPES[model_path],
        "data": "synthetic (seeded N(0,0.02) weights -> MXFP4, seeded uniform prompt ids)",
        "config": {"workload": "config1: TinyLlama-shape MXFP4 decode, bs1, 16-token prompt, greedy",
                   "n_layers": 22, "dim": 2048, "ffn": 5632, "heads": "32q/4kv", "head_dim": 64, "vocab": 32000,
                   "positions": f"{N_PROMPT}..{N_PROMPT + args.warmup + args.steps - 1}",
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "no flush: 549.5 MB of weights per step > 126 MB L2"},
        "roofline": {"bound": "hbm", "kernel": f"decode token ({model_path} path)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic_per_token().get(model_path), "bytes_per_launch": wbytes,
                     "peak_kind": peak_kind,
                     "traffic_source": "profiles/dram_traffic.json: ncu dram bytes of one launch / its tokens"},
        "gemv": gemv,
        "tp": tpres,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": kpt * args.steps if model_path == "graph" else 1,
        "clocks": {"sm_mhz": clocks["sm_mhz"], "sm_max_mhz": clocks["sm_max_mhz"], "reasons": clocks["reasons"]},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
