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

        self.L = []
        for l in layers:
            self.L.append(dict(
                wq=deq(l["wq"], d, d), wk=deq(l["wk"], kvd, d), wv=deq(l["wv"], kvd, d), wo=deq(l["wo"], d, d),
                w1=deq(l["w1"], f, d), w2=deq(l["w2"], d, f), w3=deq(l["w3"], f, d),
                ln1_w=np.asarray(l["ln1_w"], np.float64), ln1_b=np.asarray(l["ln1_b"], np.float64),
                ln2_w=np.asarray(l["ln2_w"], np.float64), ln2_b=np.asarray(l["ln2_b"], np.float64)))
        self.emb = np.asarray(emb, np.float64)
        self.fw = np.asarray(final_w, np.float64)
        self.fb = np.asarray(final_b, np.float64)
        self.wout = deq(out_blocks, V, d)
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
        c = self.cfg
        d, H, Hkv = c["dim"], c["n_heads"], c["n_kv_heads"]
        hd = d // H
        G = H // Hkv
        kv = self.cache.setdefault(seq, [[] for _ in self.L])
        pos = len(kv[0])
        x = self.emb[token].copy()
        for li, L in enumerate(self.L):
            h = bf16(O.rmsnorm_bias(x, L["ln1_w"], L["ln1_b"], self.eps))
            q = bf16(O.rope_embed(L["wq"] @ h, pos, d))
            k = bf16(O.rope_embed(L["wk"] @ h, pos, d))
            v = bf16(L["wv"] @ h)
            if self.kv_int8:
                k, v = self._int8(k, Hkv, hd), self._int8(v, Hkv, hd)
            kv[li].append((k, v))
            K = np.array([e[0] for e in kv[li]]).reshape(-1, Hkv, hd)
            Vv = np.array([e[1] for e in kv[li]]).reshape(-1, Hkv, hd)
            a = np.zeros(d)
            for j in range(H):
                kh = j // G
                a[j * hd:(j + 1) * hd] = O.paged_attention(q[j * hd:(j + 1) * hd], K[:, kh].reshape(-1),
                                                            Vv[:, kh].reshape(-1), hd)
            a = bf16(a)
            x = x + L["wo"] @ a
            h2 = bf16(O.rmsnorm_bias(x, L["ln2_w"], L["ln2_b"], self.eps))
            g = L["w1"] @ h2
            u = L["w3"] @ h2
            act = bf16(g * (1.0 / (1.0 + np.exp(-g))) * u)
            x = x + L["w2"] @ act
        hf = bf16(O.rmsnorm_bias(x, self.fw, self.fb, self.eps))
        return self.wout @ hf


def argmax_first(logits: np.ndarray) -> int:
    """argmax (stdlib/ai/transformer.vx:1163-1177): first index of the maximum."""
    return int(np.argmax(logits))
