"""Llama-style quantized decoder over libvxb.so (host-side mirror of the
transformer forward / generate interface, stdlib/ai/transformer.vx:958-1177,
and of the transformer_* builtins' call pattern, src/transformer.rs:940-1034).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .quant import context


class DecoderConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int), ("dim", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("max_batch", ctypes.c_int), ("max_seq", ctypes.c_int), ("norm_eps", ctypes.c_float),
                ("weight_fmt", ctypes.c_int), ("kv_dtype", ctypes.c_int), ("kv_block_size", ctypes.c_int)]


LLAMA_7B = dict(vocab_size=32000, dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, ffn_dim=11008,
                norm_eps=1e-5, weight_fmt=N.Q4_0, kv_dtype=N.BF16, kv_block_size=16)

# weight slots of vxb_decoder_set_weight
WQ, WK, WV, WO, W1, W2, W3, LN1_W, LN1_B, LN2_W, LN2_B = range(11)
EMBED, FINAL_W, FINAL_B, OUTPUT = range(4)

# Llama-style GGUF tensor names (llama.cpp convention) of the linear slots
GGUF_LINEARS = {"attn_q": WQ, "attn_k": WK, "attn_v": WV, "attn_output": WO, "ffn_gate": W1, "ffn_down": W2,
                "ffn_up": W3}


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns, round to nearest even by adding 0x7FFF plus
    the kept lowest bit (the tensor_engine::f32_to_bf16 rule)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def gguf_decoder_weights(f, cfg: dict) -> list:
    """(layer, slot, host array) for every weight of a decoder with config cfg
    (vocab_size, dim, n_layers, n_heads, n_kv_heads, ffn_dim, weight_fmt) from
    an open GGUFFile with llama.cpp tensor names: blk.{i}.attn_q/attn_k/attn_v/
    attn_output/ffn_gate/ffn_down/ffn_up.weight as blocks of the decoder's
    weight format (dims [in, out]), blk.{i}.attn_norm/ffn_norm.weight (+
    optional .bias) and output_norm.weight (+ .bias) as F32 or F16 (a missing
    bias is zero), token_embd.weight F32/F16 [vocab, dim] (stored as bf16) and
    output.weight blocks [vocab, dim]. Raises ValueError naming the tensor on a
    missing tensor, a wrong type or wrong dims."""
    from . import gguf as G
    d, ffn, V, L = cfg["dim"], cfg["ffn_dim"], cfg["vocab_size"], cfg["n_layers"]
    kvd = cfg["n_kv_heads"] * (d // cfg["n_heads"])
    fmt = cfg["weight_fmt"]
    have = {t["name"]: t for t in f.tensors()}

    def info(name, dims, types):
        t = have.get(name)
        if t is None:
            raise ValueError(f"GGUF tensor '{name}' is missing")
        if t["type"] not in types:
            raise ValueError(f"GGUF tensor '{name}' has ggml type {t['type']}, expected one of {sorted(types)}")
        if t["dims"] != dims:
            raise ValueError(f"GGUF tensor '{name}' has dims {t['dims']}, expected {dims}")
        return t

    def floats(name, n, optional=False):
        if optional and name not in have:
            return np.zeros(n, dtype=np.float32)
        t = info(name, [n], (G.GGML_F32, G.GGML_F16))
        raw = f.tensor_bytes(name)
        return (raw.view(np.float32) if t["type"] == G.GGML_F32 else raw.view(np.float16).astype(np.float32)).copy()

    out = []
    shapes = {WQ: [d, d], WK: [d, kvd], WV: [d, kvd], WO: [d, d], W1: [d, ffn], W2: [ffn, d], W3: [d, ffn]}
    for i in range(L):
        for stem, slot in GGUF_LINEARS.items():
            name = f"blk.{i}.{stem}.weight"
            info(name, shapes[slot], (fmt,))
            out.append((i, slot, f.tensor_bytes(name)))
        out.append((i, LN1_W, floats(f"blk.{i}.attn_norm.weight", d)))
        out.append((i, LN1_B, floats(f"blk.{i}.attn_norm.bias", d, optional=True)))
        out.append((i, LN2_W, floats(f"blk.{i}.ffn_norm.weight", d)))
        out.append((i, LN2_B, floats(f"blk.{i}.ffn_norm.bias", d, optional=True)))
    t = info("token_embd.weight", [d, V], (G.GGML_F32, G.GGML_F16))
    raw = f.tensor_bytes("token_embd.weight")
    emb = raw.view(np.float32) if t["type"] == G.GGML_F32 else raw.view(np.float16).astype(np.float32)
    out.append((-1, EMBED, _bf16_bits(emb.reshape(V, d))))
    out.append((-1, FINAL_W, floats("output_norm.weight", d)))
    out.append((-1, FINAL_B, floats("output_norm.bias", d, optional=True)))
    info("output.weight", [d, V], (fmt,))
    out.append((-1, OUTPUT, f.tensor_bytes("output.weight")))
    return out


LINEAR_KEYS = ("wq", "wk", "wv", "wo", "w1", "w2", "w3")
SLOT_OF = dict(wq=WQ, wk=WK, wv=WV, wo=WO, w1=W1, w2=W2, w3=W3, ln1_w=LN1_W, ln1_b=LN1_B, ln2_w=LN2_W,
               ln2_b=LN2_B)


def synthetic_weights(cfg: dict, seed: int, sigma: float = 0.02) -> dict:
    """Host weights of a random Llama-style decoder from one seeded numpy
    generator: every linear f32 [out, in] ~N(0, sigma) (wq wk wv wo w1 w2 w3
    per layer, then the output projection [vocab, dim]), norm weights
    1 + N(0, 0.1) and biases N(0, 0.1) (f32), the embedding as bf16 bit
    patterns of N(0, 1) values. Returns {"layers": [dict], "emb_bits",
    "final_w", "final_b", "out"}; the same seed gives the same arrays on any
    machine (numpy's PCG64 stream)."""
    rng = np.random.default_rng(seed)
    d, f, V = cfg["dim"], cfg["ffn_dim"], cfg["vocab_size"]
    kvd = cfg["n_kv_heads"] * (d // cfg["n_heads"])
    lin = lambda n, k: (rng.standard_normal((n, k), dtype=np.float32) * np.float32(sigma))
    shapes = dict(wq=(d, d), wk=(kvd, d), wv=(kvd, d), wo=(d, d), w1=(f, d), w2=(d, f), w3=(f, d))
    layers = []
    for _ in range(cfg["n_layers"]):
        l = {key: lin(*shapes[key]) for key in LINEAR_KEYS}
        for key in ("ln1", "ln2"):
            l[key + "_w"] = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
            l[key + "_b"] = (0.1 * rng.standard_normal(d)).astype(np.float32)
        layers.append(l)
    emb_bits = _bf16_bits(rng.standard_normal((V, d), dtype=np.float32))
    fw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    fb = (0.1 * rng.standard_normal(d)).astype(np.float32)
    return {"layers": layers, "emb_bits": emb_bits, "final_w": fw, "final_b": fb, "out": lin(V, d)}


class Decoder:
    """comm (optional): a vortex_b200.comm.Comm; the decoder is then this
    rank's tensor-parallel part, and every rank makes the same calls."""

    def __init__(self, max_batch: int, max_seq: int, device=None, comm=None, **cfg):
        self.ctx = comm.ctx if comm is not None else context(device)
        L = N.lib()
        c = dict(LLAMA_7B)
        c.update(cfg)
        self.cfg = DecoderConfig(**{k: c[k] for k, _ in DecoderConfig._fields_ if k in c},
                                 max_batch=max_batch, max_seq=max_seq)
        p = ctypes.c_void_p()
        if comm is None:
            N.check(L.vxb_decoder_create(self.ctx.ptr, ctypes.addressof(self.cfg), ctypes.byref(p)), self.ctx.ptr)
        else:
            N.check(L.vxb_decoder_create_tp(self.ctx.ptr, ctypes.addressof(self.cfg), comm.ptr, ctypes.byref(p)),
                    self.ctx.ptr)
        self.comm = comm
        self.ptr = p
        self.vocab = self.cfg.vocab_size

    def close(self):
        if getattr(self, "ptr", None):
            N.lib().vxb_decoder_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != N.VXB_OK:
            raise N.VxbError(rc, N.last_error(self.ctx.ptr))

    def init_random(self, seed: int = 42, sigma: float = 0.02):
        self._check(N.lib().vxb_decoder_init_random(self.ptr, seed, sigma))

    def set_weight(self, layer: int, which: int, data: np.ndarray):
        a = np.ascontiguousarray(data)
        self._check(N.lib().vxb_decoder_set_weight(self.ptr, layer, which, a.ctypes.data_as(ctypes.c_void_p),
                                                   a.nbytes))

    def load_float_weights(self, w: dict):
        """Quantize host f32 weights (synthetic_weights layout) into the
        decoder's block format with the host packer (the reference's
        quantize rules) and load them; norms and the embedding as given."""
        from . import quant as Q
        fmt = self.cfg.weight_fmt
        for li, l in enumerate(w["layers"]):
            for key, slot in SLOT_OF.items():
                a = l[key]
                self.set_weight(li, slot, Q.pack_blocks(fmt, a) if key in LINEAR_KEYS else a)
        self.set_weight(-1, EMBED, w["emb_bits"])
        self.set_weight(-1, FINAL_W, w["final_w"])
        self.set_weight(-1, FINAL_B, w["final_b"])
        self.set_weight(-1, OUTPUT, Q.pack_blocks(fmt, w["out"]))

    def load_gguf(self, source):
        """Load every weight from a Llama-style GGUF (a path, bytes or an open
        gguf.GGUFFile; tensor names and formats as gguf_decoder_weights)."""
        from . import gguf as G
        f = source if isinstance(source, G.GGUFFile) else G.GGUFFile(source)
        c = self.cfg
        cfg = dict(vocab_size=c.vocab_size, dim=c.dim, n_layers=c.n_layers, n_heads=c.n_heads,
                   n_kv_heads=c.n_kv_heads, ffn_dim=c.ffn_dim, weight_fmt=c.weight_fmt)
        for layer, which, a in gguf_decoder_weights(f, cfg):
            self.set_weight(layer, which, a)

    def step(self, seq_ids, tokens, want_logits: bool = False):
        ids = np.ascontiguousarray(seq_ids, dtype=np.int64)
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(ids.size, dtype=np.int32)
        logits = np.zeros((ids.size, self.vocab), dtype=np.float32) if want_logits else None
        self._check(N.lib().vxb_decoder_step(self.ptr, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                             tok.ctypes.data_as(ctypes.c_void_p), nxt.ctypes.data_as(ctypes.c_void_p),
                                             logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None))
        return (nxt, logits) if want_logits else nxt

    def prefill(self, seq_id: int, tokens, want_logits: bool = False):
        """Whole prompt of a new sequence in one pass (K2 GEMM + K3 flash
        attention); returns the greedy next token (and the last logits)."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        self._check(N.lib().vxb_decoder_prefill(self.ptr, int(seq_id), tok.ctypes.data_as(ctypes.c_void_p), tok.size,
                                                nxt.ctypes.data_as(ctypes.c_void_p),
                                                logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None))
        return (int(nxt[0]), logits) if want_logits else int(nxt[0])

    def score(self, seq_ids, prompts, tokens):
        """Teacher-forced scoring: prefill prompts[i] into the new sequence
        seq_ids[i], then feed tokens[s, i] for every step s. Returns the
        logits after each prompt [n, vocab] and after each fed token
        [steps, n, vocab] (f32)."""
        pre = np.stack([self.prefill(s, prompts[i], want_logits=True)[1] for i, s in enumerate(seq_ids)])
        steps = [self.step(seq_ids, tokens[t], want_logits=True)[1] for t in range(len(tokens))]
        return pre, np.stack(steps) if steps else np.zeros((0, len(seq_ids), self.vocab), np.float32)

    def step_device(self, seq_ids, d_tokens, d_next, stream=None):
        import torch
        ids = np.ascontiguousarray(seq_ids, dtype=np.int64)
        s = stream if stream is not None else torch.cuda.current_stream()
        self._check(N.lib().vxb_decoder_step_device(self.ptr, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                                    ctypes.c_void_p(d_tokens.data_ptr()),
                                                    ctypes.c_void_p(d_next.data_ptr()) if d_next is not None else None,
                                                    ctypes.c_void_p(s.cuda_stream)))

    def free_seq(self, seq_id: int):
        self._check(N.lib().vxb_decoder_free_seq(self.ptr, int(seq_id)))

    def fork(self, src_seq: int, dst_seq: int, n_tokens: int):
        """A new sequence continuing from the first n_tokens of src_seq
        (shared prompt prefix: its KV blocks are shared, not recomputed)."""
        self._check(N.lib().vxb_decoder_fork(self.ptr, int(src_seq), int(dst_seq), int(n_tokens)))

    def stream_handle(self) -> int:
        p = ctypes.c_void_p()
        self._check(N.lib().vxb_decoder_stream(self.ptr, ctypes.byref(p)))
        return p.value or 0
