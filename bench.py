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
all-reduce of the residual stream twice per layer): the batch is the same
at every N, value = tokens/s of the job, timed as the max over ranks (strong
scaling). Besides the headline the line carries:
  tp_parity    logits of a small tensor-parallel-splittable decoder on the N
               ranks against oracle logits stored in tests/golden (any N);
  decode_attn  the decode-attention configuration (32 sequences, 32 query /
               8 KV heads, ctx 1k/8k/32k, bf16 and int8 KV), heads split over
               the N ranks, GB/s against the HBM peak;
  flash        the causal flash-attention prefill configuration (B=4, H=32,
               S=4096, d=128), TFLOP/s against the bf16 peak, algorithmic
               and as executed on the tensor pipe (N = 1);
  prefill_gemm the K2 GEMM on the decoder's projection shapes at 2048 rows
               (N = 1);
  gemv         the dequant-GEMV sweep (N = 1).
--impl reference times the CPU oracle port of the reference path (rank 0).
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
FALLBACK_BF16_TFLOPS = 1590.0
# DRAM bytes / algorithmic bytes of decode_attn_kernel on the decode step's
# own per-layer shape (32 sequences x 32 heads, ctx 2048, bf16): one ncu
# capture read 1,074,086,144 + wrote 3,865,344 bytes for 1,074,266,112
# algorithmic bytes; applied to the bench's launch to give its traffic
ATTN_TRAFFIC_RATIO = (1074920192 + 6536448) / 1074266112
ATTN_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of decode_attn_kernel at 32 sequences x "
                       "32 heads, ctx 2048, bf16 (profiles/decode_attn_b32_ctx2048_mha_bf16.md), scaled by "
                       "algorithmic bytes")
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
    ap.add_argument("--cpu-sample-layers", type=int, default=1, help="layer-steps in the CPU baseline sample")
    ap.add_argument("--no-gemv-sweep", action="store_true")
    ap.add_argument("--no-flash", action="store_true")
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


def measured_tflops():
    """Dense bf16 peak: the burst figure (kernels timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


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


def cpu_layer_step(pool, n_threads: int, batch: int, part: int, seed: int = 7):
    """One layer-step of a decode step for `batch` sequences at context 2048
    on the CPU oracle (f64, dequantize-then-matvec per reference order): one
    Llama-style layer's four fused Q4_0 GEMVs and its 32-head attention, plus
    part `part` (of 32) of the LM head's rows. All 32 layers of the model have
    the same shapes, so 32 layer-steps (parts 0..31) are exactly the work of
    one full decode step. Rows are split across n_threads. Returns seconds."""
    import numpy as np

    from oracle import oracle as O
    rng = np.random.default_rng(seed + 1 + part)
    mats, lm = _cpu_weights(seed)
    bpr = lambda k: k // 32 * 18

    def gemv_rows(args):
        blocks, n, k, x, r0, r1 = args
        O.gemv_blocks(O.GGML_Q4_0, blocks[r0 * bpr(k):r1 * bpr(k)], r1 - r0, k, x)

    def gemv(blocks, n, k, r_lo=0, r_hi=None):
        r_hi = n if r_hi is None else r_hi
        x = rng.standard_normal((batch, k))
        step = (r_hi - r_lo + n_threads - 1) // n_threads
        list(pool.map(gemv_rows, [(blocks, n, k, x, r, min(r_hi, r + step)) for r in range(r_lo, r_hi, step)]))

    ctx, hd, H = 2048, 128, 32
    K = rng.standard_normal((ctx, hd))
    Vv = rng.standard_normal((ctx, hd))
    q = rng.standard_normal(hd)
    t0 = time.perf_counter()
    for blocks, n, k in mats:
        gemv(blocks, n, k)
    list(pool.map(lambda h: O.paged_attention(q, K, Vv, hd), range(batch * H)))
    V = lm[1]
    gemv(*lm, r_lo=part * V // 32, r_hi=(part + 1) * V // 32)
    return time.perf_counter() - t0


def cpu_decode_sample(n_threads: int, batch: int, layer_steps: int = 1):
    """Tokens/s of the CPU oracle on `layer_steps` consecutive layer-steps
    (each 1/32 of a decode step, see cpu_layer_step)."""
    import concurrent.futures as cf
    with cf.ThreadPoolExecutor(max_workers=n_threads) as pool:
        t = sum(cpu_layer_step(pool, n_threads, batch, i % 32) for i in range(layer_steps))
    tokens = batch * layer_steps / 32.0
    return tokens / t, (f"{layer_steps} layer-step(s) of the decode step for {batch} sequences at ctx 2048 "
                        f"(each: one layer's 4 fused Q4_0 GEMVs + 32-head attention per sequence, and 1/32 of the "
                        f"LM head rows; 32 layer-steps = one decode step), {n_threads} thread(s)")


def cpu_flash_sample():
    """C3 on the CPU oracle: flash_attention_forward (src/flash_attention.rs:
    53-159, its auto tile) for one (batch, head) of S=4096, d=128, causal,
    one thread; the reference runs heads serially, so the configuration's 128
    heads take 128 times as long. Returns (TFLOP/s, description)."""
    import numpy as np

    from oracle import oracle as O
    S, d = 4096, 128
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal(S * d) for _ in range(3))
    t = O.flash_auto_tile(S, d)
    t0 = time.perf_counter()
    O.flash_attention_forward(q, k, v, d, t, t, True)
    dt = time.perf_counter() - t0
    flops_head = 4 * d * S * (S + 1) // 2
    return flops_head / dt / 1e12, "one (batch, head) of B=4 H=32 S=4096 d=128 causal, 1 thread " \
                                   "(the configuration is 128 such heads run serially: time x128)"


def cpu_attn_sample(ctx: int = 1024, n: int = 32, Hq: int = 32, Hkv: int = 8, D: int = 128):
    """C4 at ctx 1024 on the CPU oracle: paged_attention (src/kv_cache.rs:
    95-112) for every (sequence, query head), one thread, full size. Returns
    (GB/s on the same algorithmic bytes as the GPU figure, description)."""
    import numpy as np

    from oracle import oracle as O
    rng = np.random.default_rng(4)
    K = rng.standard_normal((n, Hkv, ctx * D))
    V = rng.standard_normal((n, Hkv, ctx * D))
    q = rng.standard_normal((n, Hq, D))
    G = Hq // Hkv
    t0 = time.perf_counter()
    for i in range(n):
        for h in range(Hq):
            O.paged_attention(q[i, h], K[i, h // G], V[i, h // G], D)
    dt = time.perf_counter() - t0
    byts = n * ctx * Hkv * D * 2 * 2 + 2 * 2 * n * Hq * D
    return byts / dt / 1e9, f"{n} sequences x {Hq} query heads ({Hkv} KV heads) at ctx {ctx}, bf16-sized bytes, " \
                            "1 thread, full size"


def run_reference(args, rank, ws):
    """The reference path's CPU implementation (the oracle port) with every
    host thread: a step is one layer-step (1/32 of a decode step for the
    batch), so value = batch/32 tokens per step over the measured time and
    steps/warmup are the driver's own."""
    if rank != 0:
        return
    import concurrent.futures as cf
    n_threads = os.cpu_count() or 1
    B = args.batch
    with cf.ThreadPoolExecutor(max_workers=n_threads) as pool:
        for i in range(args.warmup):
            cpu_layer_step(pool, n_threads, B, i % 32)
        t_all = time.perf_counter()
        times = [cpu_layer_step(pool, n_threads, B, i % 32) for i in range(args.steps)]
        wall = time.perf_counter() - t_all
    total = sum(times)
    value = B * args.steps / 32.0 / total
    desc = (f"{args.steps} layer-steps (each 1/32 of the decode step for {B} sequences at ctx 2048: one layer's "
            f"4 fused Q4_0 GEMVs + 32-head attention per sequence + 1/32 of the LM head rows), {n_threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": bench_config(args, ws),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": n_threads, "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": wall}
    print(json.dumps(line), flush=True)


def bench_config(args, ws):
    return {"workload": "7B-shape Llama decoder decode (32 layers, d4096, 32x128 heads, SwiGLU 11008, "
                        "vocab 32000, Q4_0 linears, bf16 paged KV), random weights N(0,0.02)",
            "global_batch": args.batch, "seq_len": args.prompt_len, "prompt_len": args.prompt_len,
            "parallelism": f"tp{ws}" if ws > 1 else "single",
            "l2": "inputs larger than L2 (3.7 GB weights + KV per step)"}


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
    setup_s = time.perf_counter() - t_setup
    dec.close()  # its CUDA graphs hold NCCL calls: released before any later collective use

    tp = tp_parity(comm, ws)
    attn = decode_attn_sweep(ws, hbm, peak_src)

    flash = None  # single-GPU configurations
    prefill_gemm = None
    if rank == 0 and ws == 1 and not args.no_flash:
        from vortex_b200 import kernel_bench as KB
        tfl, tsrc = measured_tflops()
        r = KB.flash_case(4, 32, 4096, True)
        # the tensor pipe runs whole 128x128 tiles up to the diagonal and P.V
        # twice (P as bf16 hi + lo): S, P_hi.V, P_lo.V per tile
        nt = (4096 + 127) // 128
        tiles = nt * (nt + 1) // 2
        executed = 4 * 32 * tiles * 3 * 2 * 128 * 128 * 128
        flash = {"config": "B=4 H=32 S=4096 d=128 causal, q/k/v bf16 N(0,1), scale 1/sqrt(128)", "unit": "TFLOP/s",
                 "us": r["us"], "achieved": r["TFLOPs"], "peak": tfl, "peak_source": tsrc + " bf16 burst",
                 "frac": r["TFLOPs"] / tfl, "flops": r["flops"],
                 "flops_formula": "4*B*H*d*S(S+1)/2 (visible score pairs only)",
                 "tensor_executed_tflops": executed / (r["us"] * 1e-6) / 1e12,
                 "tensor_frac_executed": executed / (r["us"] * 1e-6) / 1e12 / tfl,
                 "executed_formula": "B*H*T*3*2*128^3, T = 528 causal 128x128 tiles per head (S, P_hi.V, P_lo.V)"}
        # K2 prefill GEMM on the decoder's projection shapes (2048 prompt
        # rows, Q4_0): the weights enter as two exact bf16 terms, so the
        # tensor pipe runs twice the algorithmic FLOPs; the time includes the
        # per-call weight expansion
        gemm_rows = []
        for n_, k_ in ((12288, 4096), (4096, 4096), (22016, 4096), (4096, 11008)):
            g_ = KB.gemm_case("Q4_0", 2048, n_, k_, reps=5)
            gemm_rows.append({"M": 2048, "N": n_, "K": k_, "us": round(g_["us"], 1),
                              "achieved": round(g_["TFLOPs"], 1), "frac": round(g_["TFLOPs"] / tfl, 3),
                              "tensor_frac_executed": round(2 * g_["TFLOPs"] / tfl, 3)})
        prefill_gemm = {"config": "Y[2048, N] = X deq(W)^T, Q4_0 W ~ N(0, 0.02), X bf16 N(0, 1), f32 out",
                        "unit": "TFLOP/s", "peak": tfl, "peak_source": tsrc + " bf16 burst",
                        "flops_formula": "2*M*N*K (executed on the tensor pipe: twice, hi and lo weight terms)",
                        "cases": gemm_rows}

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

    cpu = None  # the CPU baselines run at N = 1 only
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        v, desc = cpu_decode_sample(1, B, args.cpu_sample_layers)
        cpu = {"value": v, "unit": "tokens/s", "cores": 1, "kind": "port", "sample": desc}
        if flash is not None:
            v, desc = cpu_flash_sample()
            flash["cpu_baseline"] = {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": desc}
        if attn is not None:
            v, desc = cpu_attn_sample()
            attn["cpu_baseline"] = {"value": v, "unit": "GB/s", "cores": 1, "kind": "port", "sample": desc}

    # our kernels per step (NCCL's own kernels not counted): embedding; per
    # layer RMSNorm, QKV GEMV, RoPE + KV append, decode attention, O GEMV,
    # RMSNorm, gate/up GEMV, SwiGLU, down GEMV (+ two one-shot all-reduces with
    # tp > 1); final RMSNorm, LM-head GEMV, argmax (argmax key, all-reduce,
    # key -> token with tp > 1)
    launches_per_step = 1 + CFG_7B["n_layers"] * (9 + (2 if ws > 1 else 0)) + (3 if ws == 1 else 5)
    if rank == 0:
        cfg = bench_config(args, ws)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t_max / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": cfg,
            "prefill": {"tokens_per_s": B * args.prompt_len / t_prefill, "seconds": t_prefill,
                        "sequences": B, "prompt_len": args.prompt_len,
                        "note": "host wall time of vxb_decoder_prefill per sequence (K2 GEMM + K3 flash)"},
            "batch1_tokens_per_s": (args.steps / b1) if b1 else None,
            "batch1_ms_per_step": (b1 / args.steps * 1e3) if b1 else None,
            "roofline": {"kernel": "decode_attn_kernel (layer 0, batch %d)" % B, "bound": "hbm",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_source": peak_src, "traffic": attn_bytes * ATTN_TRAFFIC_RATIO,
                         "traffic_source": ATTN_TRAFFIC_SOURCE,
                         "algorithmic_bytes": attn_bytes, "launch_us": t_attn * 1e6},
            "cpu_baseline": cpu,
            "tp_parity_err": tp["err"] if tp else None,
            "tp_parity": tp,
            "decode_attn": attn,
            "flash": flash,
            "prefill_gemm": prefill_gemm,
            "gemv": gemv,
            "clocks": clocks,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "setup_s": setup_s,
        }
        print(json.dumps(line), flush=True)
    barrier(ws)
    if comm is not None:
        comm.close()
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def tp_parity(comm, ws):
    """Logits of the small fixture decoder (vocab 1024, d 1024, 2 layers, 8
    heads x 128, SwiGLU 2048, Q4_0; it splits over 1/2/4/8 ranks) on these
    ranks, prefill + teacher-forced decode, against the oracle logits stored
    in tests/golden/tp_decoder_logits.npz (normwise error, max over every
    position; the gate is 1e-2). Every rank runs it; rank 0 reports."""
    import numpy as np

    from vortex_b200 import decoder as D
    fx = np.load(os.path.join(ROOT, "tests", "golden", "tp_decoder_logits.npz"))
    cfg = json.loads(str(fx["cfg"]))
    dec = D.Decoder(max_batch=len(fx["seq_ids"]), max_seq=32, comm=comm, **cfg)
    dec.load_float_weights(D.synthetic_weights(cfg, int(fx["seed"])))
    ids = [int(s) for s in fx["seq_ids"]]
    pre, steps = dec.score(ids, fx["prompts"], fx["tokens"])
    dec.close()

    def nerr(y, r):
        return float(np.max(np.abs(y.astype(np.float64) - r)) / np.max(np.abs(r)))

    errs = [nerr(pre[i], fx["prefill_logits"][i]) for i in range(len(ids))]
    errs += [nerr(steps[t, i], fx["logits"][t, i]) for t in range(steps.shape[0]) for i in range(len(ids))]
    err = max_over_ranks(max(errs), ws)
    return {"err": err, "gate": 1e-2, "ranks": ws, "positions": len(errs),
            "model": "vocab 1024, d 1024, 2 layers, 8x128 heads, SwiGLU 2048, Q4_0; 4 sequences, 8-token prompts, "
                     "4 teacher-forced decode steps; normwise max|y-r|/max|r| against the oracle"}


def decode_attn_sweep(ws, hbm, peak_src):
    """The decode-attention configuration: 32 sequences, 32 query / 8 KV heads,
    head_dim 128, ctx 1k/8k/32k, bf16 and int8 KV; the heads are split over
    the ranks (each rank 32/N query and 8/N KV heads), time = max over ranks,
    GB/s = the whole configuration's algorithmic bytes / that time; frac
    against the N GPUs' combined peak (N x the one-GPU copy bandwidth)."""
    from vortex_b200 import kernel_bench as KB
    cases = []
    for dt in ("bf16", "int8"):
        for ctx in (1024, 8192, 32768):
            r = KB.attn_case(ctx, dt, n=32, Hq=32 // ws, Hkv=8 // ws)
            t = max_over_ranks(r["us"], ws)
            per_tok = 8 * 128 * 2 * 2 if dt == "bf16" else 8 * 128 * 2 + 8 * 2 * 4
            byts = 32 * ctx * per_tok + 2 * 2 * 32 * 32 * 128
            cases.append({"dtype": dt, "ctx": ctx, "us": round(t, 2), "achieved": round(byts / t / 1e3, 1),
                          "frac": round(byts / t / 1e3 / (hbm * ws), 3), "bytes": byts})
    return {"config": "32 sequences x 32 query heads / 8 KV heads (GQA), head_dim 128, one new token each; "
                      f"heads split over {ws} GPU(s)", "unit": "GB/s", "peak": hbm * ws,
            "peak_source": peak_src + (f" (x{ws} GPUs)" if ws > 1 else ""),
            "bytes": "32*ctx*(8*128*2*2 bf16 | 8*(128+4)*2 int8) + q/out", "cases": cases}


if __name__ == "__main__":
    main()
