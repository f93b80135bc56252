#!/usr/bin/env python
"""Decode throughput of the 7B-shaped 4-bit Llama decoder on B200.

Workload (one "step" = one decode step of every sequence in the batch):
32 layers, d_model 4096, 32 heads x 128, SwiGLU 11008, RMSNorm, RoPE,
vocab 32000, every linear Q4_0 (block 32, f16 scales) from N(0, 0.02)
synthetic weights, a 2048-token random-id prompt per sequence, then decode
steps at batch 32 (headline) and batch 1. KV cache bf16, paged. Prompts are
prefilled in one pass per sequence (prefill GEMM + flash attention).

Prints one JSON line (rank 0). With torchrun (N > 1) the ranks run one
tensor-parallel decoder (heads, FFN rows and vocabulary split over the N GPUs,
NCCL all-reduce of the residual stream twice per layer): the batch is the same
at every N, value = tokens/s of the job, timed as the max over ranks (strong
scaling). --impl reference times the CPU oracle port of the reference path
(rank 0 only).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s (7B-shape 4-bit) at 1/2/4/8 B200; dequant-GEMV HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes / algorithmic bytes of decode_attn_kernel, from an ncu capture of
# the same kernel on batch 32, ctx 8192 (1.07446 GB read + 7.79 MB written for
# 1.07427 GB of K/V/q/out): applied to the bench's launch to give its traffic
ATTN_TRAFFIC_RATIO = (1.074456e9 + 7.78624e6) / 1.074266112e9
CFG_7B = dict(vocab_size=32000, dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, ffn_dim=11008)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vortex", choices=["vortex", "reference"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--e2e-steps", type=int, default=16)
    ap.add_argument("--no-batch1", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-layers", type=int, default=1)
    ap.add_argument("--no-gemv-sweep", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------- helpers

def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        # NCCL's banner and warnings go to stderr: stdout carries the JSON line only
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        import datetime

        import torch
        import torch.distributed as dist
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        return rank, ws, local
    return 0, 1, 0


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU baseline (oracle port)

_CPU_WEIGHTS = {}


def _cpu_weights(seed: int):
    """The sampled layer's four fused Q4_0 linears and the LM head as blocks
    (quantized once per process: the quantization is setup, not the sample)."""
    if seed not in _CPU_WEIGHTS:
        import numpy as np

        from oracle import oracle as O
        rng = np.random.default_rng(seed)
        d, f, V = CFG_7B["dim"], CFG_7B["ffn_dim"], CFG_7B["vocab_size"]
        shapes = [(3 * d, d), (d, d), (2 * f, d), (d, f)]
        mats = [(O.quantize_blocks(O.GGML_Q4_0, rng.normal(0, 0.02, n * k).astype(np.float32)), n, k)
                for n, k in shapes]
        lm = (O.quantize_blocks(O.GGML_Q4_0, rng.normal(0, 0.02, V * d).astype(np.float32)), V, d)
        _CPU_WEIGHTS[seed] = (mats, lm)
    return _CPU_WEIGHTS[seed]


def cpu_layer_sample(n_threads: int, batch: int = 1, seed: int = 7):
    """Time one Llama-style layer of a decode step for `batch` sequences at
    context 2048 on the CPU oracle (f64, dequantize-then-matvec per reference
    order) plus the LM head, split across n_threads by output rows. Returns
    (seconds for one decode step of the full 32-layer model, description)."""
    import concurrent.futures as cf

    import numpy as np

    from oracle import oracle as O
    rng = np.random.default_rng(seed + 1)
    mats, lm = _cpu_weights(seed)
    bpr = lambda k: k // 32 * 18

    def gemv_rows(args):
        blocks, n, k, x, r0, r1 = args
        O.gemv_blocks(O.GGML_Q4_0, blocks[r0 * bpr(k):r1 * bpr(k)], r1 - r0, k, x)

    def gemv(pool, blocks, n, k):
        x = rng.standard_normal((batch, k))
        step = (n + n_threads - 1) // n_threads
        list(pool.map(gemv_rows, [(blocks, n, k, x, r, min(n, r + step)) for r in range(0, n, step)]))

    ctx, hd, H = 2048, 128, 32
    K = rng.standard_normal((ctx, hd))
    Vv = rng.standard_normal((ctx, hd))
    q = rng.standard_normal(hd)
    with cf.ThreadPoolExecutor(max_workers=n_threads) as pool:
        t0 = time.perf_counter()
        for blocks, n, k in mats:
            gemv(pool, blocks, n, k)
        list(pool.map(lambda h: O.paged_attention(q, K, Vv, hd), range(batch * H)))
        t_layer = time.perf_counter() - t0
        t0 = time.perf_counter()
        gemv(pool, *lm)
        t_lm = time.perf_counter() - t0
    per_step = CFG_7B["n_layers"] * t_layer + t_lm
    return per_step, f"one layer (4 fused Q4_0 GEMVs over {batch} rows + 32-head attention at ctx 2048 for " \
                     f"{batch} sequences) + LM head, {n_threads} thread(s), extrapolated x32 layers"


def run_reference(args, rank, ws):
    if rank != 0:
        return
    n_threads = os.cpu_count() or 1
    # warmup samples
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_layer_sample(n_threads, args.batch)
    times = []
    t_all = time.perf_counter()
    steps = max(1, min(args.steps, 4))
    for _ in range(steps):
        per_step, desc = cpu_layer_sample(n_threads, args.batch)
        times.append(per_step)
    per_step = statistics.median(times)
    value = args.batch / per_step
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "7B-shape Llama decoder decode, Q4_0 linears, CPU oracle port of the reference "
                                   "path (sampled layer, extrapolated)", "global_batch": args.batch,
                       "seq_len": args.prompt_len, "parallelism": "cpu threads"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n_threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t_all}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

def time_attention(dec, seq_ids, hd_heads, reps=20):
    """Average duration of the decode attention kernel (layer 0) on the
    decoder's cache at its current lengths, CUDA events on the launch stream."""
    import ctypes

    import numpy as np
    import torch

    from vortex_b200 import _native as N
    kv = ctypes.c_void_p()
    N.check(N.lib().vxb_decoder_kv(dec.ptr, ctypes.byref(kv)))
    H, hd = hd_heads
    n = len(seq_ids)
    q = torch.randn(n, H, hd, device="cuda").bfloat16()
    out = torch.empty_like(q)
    ids = np.ascontiguousarray(seq_ids, dtype=np.int64)
    s = torch.cuda.Stream()
    L = N.lib()
    with torch.cuda.stream(s):
        for _ in range(3):
            N.check(L.vxb_decode_attention(kv, 0, n, ids.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(q.data_ptr()),
                                           H, ctypes.c_float(1.0 / hd ** 0.5), ctypes.c_void_p(out.data_ptr()), None,
                                           ctypes.c_void_p(s.cuda_stream)))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            L.vxb_decode_attention(kv, 0, n, ids.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(q.data_ptr()), H,
                                   ctypes.c_float(1.0 / hd ** 0.5), ctypes.c_void_p(out.data_ptr()), None,
                                   ctypes.c_void_p(s.cuda_stream))
        e1.record(s)
    torch.cuda.synchronize()
    lens = []
    for sid in seq_ids:
        ln = ctypes.c_int64()
        N.check(L.vxb_kv_seq_len(kv, 0, int(sid), ctypes.byref(ln)))
        lens.append(ln.value)
    return e0.elapsed_time(e1) / reps * 1e-3, lens


def run_decode(dec, seq_ids, prompt, steps, warmup, ws, torch):
    """Prefill every sequence's prompt in one pass (K2 GEMM + K3 flash
    attention; timed separately), warm up, then time `steps` decode steps with
    CUDA events on the decoder's stream. Returns (decode seconds, next tokens,
    prefill seconds)."""
    import numpy as np
    B = len(seq_ids)
    nxt = torch.empty(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    barrier(ws)
    t0 = time.perf_counter()
    first = [dec.prefill(s, prompt[i]) for i, s in enumerate(seq_ids)]
    t_prefill = time.perf_counter() - t0
    nxt.copy_(torch.tensor(first, dtype=torch.int32))
    tok = nxt.clone()
    for _ in range(warmup):
        tok.copy_(nxt)
        dec.step_device(seq_ids, tok, nxt)
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()  # bounds a profiler capture to the timed region
    e0.record(stream)
    for _ in range(steps):
        tok.copy_(nxt)
        dec.step_device(seq_ids, tok, nxt)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    barrier(ws)
    return e0.elapsed_time(e1) * 1e-3, nxt, t_prefill


def main():
    args = parse()
    rank, ws, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, ws)
        return
    import numpy as np
    import torch

    from vortex_b200 import decoder as D

    torch.cuda.set_device(local)
    B = args.batch
    max_seq = args.prompt_len + args.warmup + args.steps + args.e2e_steps + 8
    t_setup = time.perf_counter()
    comm = None
    if ws > 1:
        from vortex_b200 import comm as C
        comm = C.Comm(ws, rank, C.share_unique_id(rank), device=local)
    dec = D.Decoder(max_batch=B, max_seq=max_seq, comm=comm, **CFG_7B)
    dec.init_random(seed=1234, sigma=0.02)
    rng = np.random.default_rng(2024)
    prompt = rng.integers(0, CFG_7B["vocab_size"], size=(B, args.prompt_len))
    seq_ids = list(range(B))

    sampler = ClockSampler(local)
    sampler.start()
    t_dev, nxt, t_prefill = run_decode(dec, seq_ids, prompt, args.steps, args.warmup, ws, torch)
    t_prefill = max_over_ranks(t_prefill, ws)
    clocks = sampler.stop()
    t_max = max_over_ranks(t_dev, ws)
    value = B * args.steps / t_max

    # end to end through the host-buffer C ABI call (tokens H2D, next tokens D2H)
    host_tok = nxt.cpu().numpy().astype(np.int32)
    barrier(ws)
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        host_tok = dec.step(seq_ids, host_tok)
    t_e2e = max_over_ranks(time.perf_counter() - t0, ws)
    e2e = B * args.e2e_steps / t_e2e
    h2d = B * 4 + CFG_7B["n_layers"] * B * 16 + B * 4
    d2h = B * 4

    # dominant kernel at this workload: decode attention (KV bytes >> weights),
    # this rank's heads
    hbm, peak_src = measured_peaks()
    hd = CFG_7B["dim"] // CFG_7B["n_heads"]
    hq_loc, hkv_loc = CFG_7B["n_heads"] // ws, CFG_7B["n_kv_heads"] // ws
    t_attn, lens = time_attention(dec, seq_ids, (hq_loc, hd))
    attn_bytes = sum(lens) * hkv_loc * hd * 2 * 2 + 2 * B * hq_loc * hd * 2
    achieved = attn_bytes / t_attn / 1e9

    # batch 1 on a freed slot
    b1 = None
    if not args.no_batch1:
        dec.free_seq(seq_ids[-1])
        sid = [10_000]
        t1, _, _ = run_decode(dec, sid, prompt[:1], args.steps, args.warmup, ws, torch)
        b1 = max_over_ranks(t1, ws)
    barrier(ws)

    # dequant-GEMV sweep (weights 4096x4096, 11008x4096, 4096x11008; Q4_0 and
    # Q8_0; batch 1, 4, 16), each over rotating weight copies > 2x L2; one GPU
    # (with N > 1 the other ranks would idle at the barrier meanwhile)
    gemv = None
    if rank == 0 and ws == 1 and not args.no_gemv_sweep:
        from vortex_b200 import kernel_bench as KB
        rows = KB.gemv_sweep()
        gemv = {"unit": "GB/s", "peak": hbm, "peak_source": peak_src,
                "bytes": "N*K*(18 or 34)/32 + 2*B*K + 4*B*N per launch",
                "cases": [{"fmt": r["fmt"], "N": r["N"], "K": r["K"], "batch": r["batch"], "us": round(r["us"], 2),
                           "achieved": round(r["GBps"], 1), "frac": round(r["GBps"] / hbm, 3)} for r in rows]}
        gemv["best_frac"] = max(c["frac"] for c in gemv["cases"])

    cpu = None  # the CPU baseline runs at N = 1 only
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        per_step, desc = cpu_layer_sample(1, B)
        cpu = {"value": B / per_step, "unit": "tokens/s", "cores": 1, "kind": "port", "sample": desc}

    # our kernels per step (NCCL's own kernels not counted): embedding; per
    # layer RMSNorm, QKV GEMV, RoPE + KV append, decode attention, O GEMV,
    # RMSNorm, gate/up GEMV, SwiGLU, down GEMV (+ two one-shot all-reduces with
    # tp > 1); final RMSNorm, LM-head GEMV, argmax (argmax key, all-reduce,
    # key -> token with tp > 1)
    launches_per_step = 1 + CFG_7B["n_layers"] * (9 + (2 if ws > 1 else 0)) + (3 if ws == 1 else 5)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "7B-shape Llama decoder decode (32 layers, d4096, 32x128 heads, SwiGLU 11008, "
                                   "vocab 32000, Q4_0 linears, bf16 paged KV), random weights N(0,0.02)",
                       "global_batch": B, "seq_len": args.prompt_len,
                       "prompt_len": args.prompt_len, "decode_steps": args.steps,
                       "parallelism": f"tp{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (3.7 GB weights + KV per step)"},
            "prefill": {"tokens_per_s": B * args.prompt_len / t_prefill, "seconds": t_prefill,
                        "sequences": B, "prompt_len": args.prompt_len,
                        "note": "host wall time of vxb_decoder_prefill per sequence (K2 GEMM + K3 flash)"},
            "batch1_tokens_per_s": (args.steps / b1) if b1 else None,
            "batch1_ms_per_step": (b1 / args.steps * 1e3) if b1 else None,
            "roofline": {"kernel": "decode_attn_kernel (layer 0, batch %d)" % B, "bound": "hbm",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": peak_src, "traffic": attn_bytes * ATTN_TRAFFIC_RATIO,
                         "algorithmic_bytes": attn_bytes, "launch_us": t_attn * 1e6},
            "cpu_baseline": cpu,
            "gemv": gemv,
            "clocks": clocks,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "setup_s": time.perf_counter() - t_setup,
        }
        print(json.dumps(line), flush=True)
    barrier(ws)
    dec.close()  # its CUDA graphs hold NCCL calls: release them before the communicator
    if comm is not None:
        comm.close()
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
