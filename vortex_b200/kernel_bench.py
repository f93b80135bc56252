"""Kernel-level timing of the decode GEMV and the decode attention.

    python -m vortex_b200.kernel_bench gemv [--fmt Q4_0] [--n 11008] [--k 4096] [--batch 1]
    python -m vortex_b200.kernel_bench attn [--ctx 8192] [--dtype bf16] [--batch 32] [--hq 32] [--hkv 8]
    python -m vortex_b200.kernel_bench flash [--b 4] [--h 32] [--s 4096] [--non-causal]
    python -m vortex_b200.kernel_bench flash_bwd [--b 4] [--h 32] [--s 4096]
    python -m vortex_b200.kernel_bench gemm [--m 2048] [--n 12288 ...] [--k 4096 ...]

Each case streams its operands from HBM: the GEMV rotates over enough distinct
weight copies to exceed twice the L2 (126 MB), the attention reads a KV cache
far larger than L2. Launches are captured back to back in one CUDA graph and
timed with CUDA events on the capturing stream; the figure is the average
device time of one launch. GB/s counts algorithmic bytes: weights (codes +
f16 scales) + bf16 activations + outputs for the GEMV, K and V of every cached
token (+ scales for int8) + q/out for the attention.
"""
from __future__ import annotations

import argparse
import json

L2_BYTES = 126 * 2 ** 20


def _graph_time(torch, fn, launches_per_call: int, reps: int = 20):
    """Capture fn() once into a graph, replay `reps` times; seconds per launch."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # first call outside capture (one-time setup such as workspace growth)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e-3 / (reps * launches_per_call)
    del g
    return t


def gemv_bytes(fmt: int, N: int, K: int, B: int) -> int:
    from . import quant as Q
    return Q.block_bytes(fmt, N * K) + 2 * B * K + 4 * B * N


def gemv_case(fmt, N: int, K: int, batches=(1, 4, 16), reps: int = 20, seed: int = 0, min_copies: int = 2):
    """Time y = deq(W) x for each batch size over rotating weight copies
    (W ~ N(0, 0.02), x ~ N(0, 1) bf16, y f32)."""
    import torch

    from . import quant as Q
    f = Q._fmt(fmt)
    wbytes = Q.block_bytes(f, N * K)
    copies = max(min_copies, -(-2 * L2_BYTES // wbytes) + 1)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    ws = []
    for _ in range(copies):
        w = torch.randn(N, K, device="cuda", generator=gen) * 0.02
        ws.append(Q.TiledWeight.from_float(w, f))
        del w
    out = []
    for B in batches:
        x = torch.randn(B, K, device="cuda", generator=gen).bfloat16()
        y = torch.empty(B, N, device="cuda")

        def run():
            for tw in ws:
                tw.gemv(x, out=y)

        t = _graph_time(torch, run, copies, reps)
        byts = gemv_bytes(f, N, K, B)
        out.append({"fmt": "Q4_0" if f == Q.Q4_0 else "Q8_0", "N": N, "K": K, "batch": B, "us": t * 1e6,
                    "GBps": byts / t / 1e9, "bytes": byts, "copies": copies})
    del ws
    torch.cuda.empty_cache()
    return out


def gemv_sweep(shapes=((4096, 4096), (11008, 4096), (4096, 11008)), fmts=("Q4_0", "Q8_0"), batches=(1, 4, 16),
               reps: int = 20):
    res = []
    for fmt in fmts:
        for N, K in shapes:
            res.extend(gemv_case(fmt, N, K, batches, reps))
    return res


def attn_case(ctx: int, dtype: str = "bf16", n: int = 32, Hq: int = 32, Hkv: int = 8, D: int = 128, reps: int = 10,
              seed: int = 0):
    """Decode attention over a paged cache: n sequences of ctx tokens, Hq
    query heads over Hkv KV heads (GQA), head_dim D, one query token each.
    When one cache is smaller than twice the L2, launches rotate over enough
    distinct caches to exceed it."""
    import torch

    from . import kv_cache as KV
    kd = KV.BF16 if dtype == "bf16" else KV.I8
    bs = 16
    per_tok = Hkv * D * 2 * (2 if kd == KV.BF16 else 1) + (Hkv * 2 * 4 if kd == KV.I8 else 0)
    kv_bytes = n * ctx * per_tok
    copies = max(1, -(-2 * L2_BYTES // kv_bytes))
    gen = torch.Generator(device="cuda").manual_seed(seed)
    caches = []
    for _ in range(copies):
        cache = KV.PagedKVCache(1, Hkv, D, bs, max_blocks=n * (-(-ctx // bs)) + 8, max_seqs=n + 1, kv_dtype=kd)
        for i in range(n):
            k = torch.randn(ctx, Hkv, D, device="cuda", generator=gen).bfloat16()
            v = torch.randn(ctx, Hkv, D, device="cuda", generator=gen).bfloat16()
            cache.append_seq(0, i, k, v)
            del k, v
        caches.append(cache)
    q = torch.randn(n, Hq, D, device="cuda", generator=gen).bfloat16()
    ids = list(range(n))
    o = caches[0].attention(0, ids, q)
    per = max(5, copies)

    def run():
        for j in range(per):
            caches[j % copies].attention(0, ids, q, out=o)

    t = _graph_time(torch, run, per, reps)
    byts = kv_bytes + 2 * 2 * n * Hq * D
    res = {"dtype": dtype, "ctx": ctx, "batch": n, "Hq": Hq, "Hkv": Hkv, "D": D, "us": t * 1e6,
           "GBps": byts / t / 1e9, "bytes": byts, "copies": copies}
    del caches
    torch.cuda.empty_cache()
    return res


def flash_case(B: int = 4, H: int = 32, S: int = 4096, causal: bool = True, reps: int = 10, seed: int = 0):
    """Flash-attention forward, q/k/v bf16 [B, S, H, 128] ~ N(0, 1), scale
    1/sqrt(128). FLOPs count only the visible (unmasked) score pairs:
    4 * B * H * d * S(S+1)/2 causal, 4 * B * H * d * S^2 otherwise."""
    import torch

    from . import attention as A
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(B, S, H, 128, device="cuda", generator=gen).bfloat16() for _ in range(3))
    o, lse = A.flash_attention(q, k, v, causal=causal)

    def run():
        A.flash_attention(q, k, v, causal=causal, out=o, lse=lse)

    t = _graph_time(torch, run, 1, reps)
    pairs = S * (S + 1) // 2 if causal else S * S
    flops = 4 * B * H * 128 * pairs
    return {"B": B, "H": H, "S": S, "d": 128, "causal": causal, "us": t * 1e6, "TFLOPs": flops / t / 1e12,
            "flops": flops}


def flash_bwd_case(B: int = 4, H: int = 32, S: int = 4096, causal: bool = True, reps: int = 5, seed: int = 0):
    """Flash-attention backward on the prefill shape. FLOPs count the
    algorithmic products over visible pairs: S, dP, dV, dK, dQ = 5 x 2 x d
    per pair (the recomputation of S and dP in the dQ pass is not counted)."""
    import torch

    from . import attention as A
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v, do = (torch.randn(B, S, H, 128, device="cuda", generator=gen).bfloat16() for _ in range(4))
    o, lse = A.flash_attention(q, k, v, causal=causal)
    A.flash_attention_backward(q, k, v, o, do, lse, causal=causal)

    def run():
        A.flash_attention_backward(q, k, v, o, do, lse, causal=causal)

    t = _graph_time(torch, run, 1, reps)
    pairs = S * (S + 1) // 2 if causal else S * S
    flops = 10 * B * H * 128 * pairs
    return {"B": B, "H": H, "S": S, "d": 128, "causal": causal, "us": t * 1e6, "TFLOPs": flops / t / 1e12,
            "flops": flops}


def gemm_case(fmt="Q4_0", M: int = 2048, N: int = 11008, K: int = 4096, reps: int = 10, seed: int = 0):
    """Prefill GEMM Y[M, N] = X[M, K] deq(W)^T, W ~ N(0, 0.02), X ~ N(0, 1)
    bf16, Y f32. FLOPs = 2 M N K (algorithmic; the kernel runs the hi and lo
    halves, twice that on the tensor pipe). The time includes the per-call
    weight expansion."""
    import torch

    from . import quant as Q
    gen = torch.Generator(device="cuda").manual_seed(seed)
    tw = Q.TiledWeight.from_float(torch.randn(N, K, device="cuda", generator=gen) * 0.02, Q._fmt(fmt))
    x = torch.randn(M, K, device="cuda", generator=gen).bfloat16()
    y = tw.gemm(x)

    def run():
        tw.gemm(x, out=y)

    t = _graph_time(torch, run, 1, reps)
    flops = 2 * M * N * K
    return {"fmt": fmt, "M": M, "N": N, "K": K, "us": t * 1e6, "TFLOPs": flops / t / 1e12, "flops": flops}


def main():
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemv")
    g.add_argument("--fmt", default=None, help="Q4_0 or Q8_0 (default: both)")
    g.add_argument("--n", type=int, default=None)
    g.add_argument("--k", type=int, default=None)
    g.add_argument("--batch", type=int, nargs="*", default=[1, 4, 16])
    g.add_argument("--reps", type=int, default=20)
    m = sub.add_parser("gemm")
    m.add_argument("--fmt", default="Q4_0")
    m.add_argument("--m", type=int, default=2048)
    m.add_argument("--n", type=int, nargs="*", default=[12288, 4096, 22016, 4096])
    m.add_argument("--k", type=int, nargs="*", default=[4096, 4096, 4096, 11008])
    m.add_argument("--reps", type=int, default=10)
    f = sub.add_parser("flash")
    f.add_argument("--b", type=int, default=4)
    f.add_argument("--h", type=int, default=32)
    f.add_argument("--s", type=int, default=4096)
    f.add_argument("--non-causal", action="store_true")
    f.add_argument("--reps", type=int, default=10)
    fb = sub.add_parser("flash_bwd")
    fb.add_argument("--b", type=int, default=4)
    fb.add_argument("--h", type=int, default=32)
    fb.add_argument("--s", type=int, default=4096)
    fb.add_argument("--reps", type=int, default=5)
    a = sub.add_parser("attn")
    a.add_argument("--ctx", type=int, nargs="*", default=[1024, 8192, 32768])
    a.add_argument("--dtype", nargs="*", default=["bf16", "int8"])
    a.add_argument("--batch", type=int, default=32)
    a.add_argument("--hq", type=int, default=32)
    a.add_argument("--hkv", type=int, default=8)
    a.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    import torch
    torch.cuda.set_device(0)
    if args.what == "gemv":
        fmts = [args.fmt] if args.fmt else ["Q4_0", "Q8_0"]
        shapes = [(args.n, args.k)] if args.n and args.k else [(4096, 4096), (11008, 4096), (4096, 11008)]
        for r in gemv_sweep(shapes, fmts, args.batch, args.reps):
            print(json.dumps(r), flush=True)
    elif args.what == "gemm":
        for n, k in zip(args.n, args.k):
            print(json.dumps(gemm_case(args.fmt, args.m, n, k, args.reps)), flush=True)
    elif args.what == "flash_bwd":
        print(json.dumps(flash_bwd_case(args.b, args.h, args.s, True, args.reps)), flush=True)
    elif args.what == "flash":
        print(json.dumps(flash_case(args.b, args.h, args.s, not args.non_causal, args.reps)), flush=True)
    else:
        for dt in args.dtype:
            for c in args.ctx:
                print(json.dumps(attn_case(c, dt, n=args.batch, Hq=args.hq, Hkv=args.hkv, reps=args.reps)),
                      flush=True)


if __name__ == "__main__":
    main()
