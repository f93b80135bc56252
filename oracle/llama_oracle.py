"""Llama-style decoder restatement -- TEST INFRASTRUCTURE ONLY.

f64 restatement of the reference's Llama-style block (stdlib/ai/transformer.vx:
layer_norm 413-439, rope_embed 442-466, attention 522-587, feed_forward
591-603, transformer_block 958-1111, forward 1120-1156, argmax 1163-1177)
driven one token per step with a KV cache (as the .vx kv_cache_* helpers,
734-846), using the C oracle for the arithmetic. Weights are the dequantized
GGUF blocks the device holds. Where the device stores a value in bf16 (the
inputs of every projection, q/k/v after RoPE, the attention output), the
oracle rounds the same value to bf16 (tensor_engine::f32_to_bf16 rule), so
both sides see identical operands at those points.
"""
from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np

from . import oracle as O


def bf16(x):
    return O.bf16_bits_to_f32_array(O.f32_array_to_bf16_bits(np.asarray(x, dtype=np.float32))).astype(np.float64)


class LlamaOracle:
    def __init__(self, cfg: dict, layers: list, emb, final_w, final_b, out_blocks, fmt):
        """layers: dicts with keys wq wk wv wo w1 w2 w3 (GGUF block bytes) and
        ln1_w ln1_b ln2_w ln2_b (float arrays)."""
        self.cfg = cfg
        self.fmt = fmt
        d, f, V = cfg["dim"], cfg["ffn_dim"], cfg["vocab_size"]
        kvd = cfg["n_kv_heads"] * (d // cfg["n_heads"])

        def deq(blocks, n, k):
            return O.dequantize_blocks(fmt, blocks, n * k).astype(np.float64).reshape(n, k)

        # one matrix per thread (the C oracle releases the interpreter lock)
        with cf.ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as pool:
            shapes = dict(wq=(d, d), wk=(kvd, d), wv=(kvd, d), wo=(d, d), w1=(f, d), w2=(d, f), w3=(f, d))
            futs = [{key: pool.submit(deq, l[key], *nk) for key, nk in shapes.items()} for l in layers]
            fout = pool.submit(deq, out_blocks, V, d)
            self.L = []
            for l, fu in zip(layers, futs):
                m = {key: fu[key].result() for key in shapes}
                m.update(ln1_w=np.asarray(l["ln1_w"], np.float64), ln1_b=np.asarray(l["ln1_b"], np.float64),
                         ln2_w=np.asarray(l["ln2_w"], np.float64), ln2_b=np.asarray(l["ln2_b"], np.float64))
                self.L.append(m)
            self.wout = fout.result()
        self.emb = np.asarray(emb, np.float64)
        self.fw = np.asarray(final_w, np.float64)
        self.fb = np.asarray(final_b, np.float64)
        self.cache = {}  # seq -> per layer [(k, v)]
        self.eps = cfg.get("norm_eps", 1e-5)
        self.kv_int8 = bool(cfg.get("kv_int8", False))

    @staticmethod
    def _int8(x, heads, hd):
        """int8 cache entry per (token, head): calibrate_minmax + codes
        (src/quantize.rs:96-137, 585-591), dequantized with the f32 scale."""
        out = np.empty_like(x)
        for h in range(heads):
            row = x[h * hd:(h + 1) * hd]
            packed, scales, _ = O.quantize(row, O.INT8, None)
            out[h * hd:(h + 1) * hd] = packed.view(np.int8).astype(np.float64) * float(np.float32(scales[0]))
        return out

    def step(self, seq: int, token: int) -> np.ndarray:
        return self.step_batch([seq], [token])[0]

    def step_batch(self, seqs, tokens, logits: bool = True):
        """One token for each sequence of `seqs` (distinct ids, each at its own
        position). The projections of all sequences are one f64 matrix
        product per weight (the same per-column sums as a matvec); norms, RoPE
        and attention run per sequence. Returns the logits [len(seqs), vocab]
        (None with logits=False, which skips the output projection)."""
        c = self.cfg
        d, H, Hkv = c["dim"], c["n_heads"], c["n_kv_heads"]
        hd = d // H
        G = H // Hkv
        B = len(seqs)
        kvs = [self.cache.setdefault(s, [[] for _ in self.L]) for s in seqs]
        pos = [len(kv[0]) for kv in kvs]
        X = self.emb[np.asarray(tokens, dtype=np.int64)].T.copy()  # [d, B]

        def norm_cols(X, w, b):
            return bf16(np.stack([O.rmsnorm_bias(X[:, i], w, b, self.eps) for i in range(B)], axis=1))

        for li, L in enumerate(self.L):
            Hn = norm_cols(X, L["ln1_w"], L["ln1_b"])
            Q, K, V = L["wq"] @ Hn, L["wk"] @ Hn, L["wv"] @ Hn
            A = np.zeros((d, B))
            for i in range(B):
                q = bf16(O.rope_embed(Q[:, i], pos[i], d))
                k = bf16(O.rope_embed(K[:, i], pos[i], d))
                v = bf16(V[:, i])
                if self.kv_int8:
                    k, v = self._int8(k, Hkv, hd), self._int8(v, Hkv, hd)
                kvs[i][li].append((k, v))
                Kc = np.array([e[0] for e in kvs[i][li]]).reshape(-1, Hkv, hd)
                Vc = np.array([e[1] for e in kvs[i][li]]).reshape(-1, Hkv, hd)
                for j in range(H):
                    kh = j // G
                    A[j * hd:(j + 1) * hd, i] = O.paged_attention(q[j * hd:(j + 1) * hd], Kc[:, kh].reshape(-1),
                                                                  Vc[:, kh].reshape(-1), hd)
            X = X + L["wo"] @ bf16(A)
            H2 = norm_cols(X, L["ln2_w"], L["ln2_b"])
            Gt = L["w1"] @ H2
            U = L["w3"] @ H2
            X = X + L["w2"] @ bf16(Gt * (1.0 / (1.0 + np.exp(-Gt))) * U)
        if not logits:
            return None
        Hf = norm_cols(X, self.fw, self.fb)
        return (self.wout @ Hf).T


def argmax_first(logits: np.ndarray) -> int:
    """argmax (stdlib/ai/transformer.vx:1163-1177): first index of the maximum."""
    return int(np.argmax(logits))
