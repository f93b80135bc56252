"""Decoder.load_gguf on the GPU: a decoder loaded from a Llama-style GGUF
holds the same weights as one loaded slot by slot from the arrays the file was
written from (identical logits and tokens). The name/slot mapping itself is
checked on CPU in test_gguf_decoder_cpu.py."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.test_decoder_gpu import _build, _load

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def test_decoder_load_gguf_matches_array_load(cuda_ok):
    """A decoder loaded from a Llama-style GGUF (Decoder.load_gguf) holds the
    same weights as one loaded slot by slot from the arrays the file was
    written from: identical logits and tokens, step by step."""
    from vortex_b200 import _native as N
    from vortex_b200 import decoder as D
    from vortex_b200 import gguf
    cfg = dict(vocab_size=512, dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, norm_eps=1e-5)
    layers, emb_bits, fw, fb, out = _build(cfg, 9, O.GGML_Q4_0)
    d, f, V = cfg["dim"], cfg["ffn_dim"], cfg["vocab_size"]
    kvd = cfg["n_kv_heads"] * (d // cfg["n_heads"])
    linears = {"wq": ("attn_q", [d, d]), "wk": ("attn_k", [d, kvd]), "wv": ("attn_v", [d, kvd]),
               "wo": ("attn_output", [d, d]), "w1": ("ffn_gate", [d, f]), "w2": ("ffn_down", [f, d]),
               "w3": ("ffn_up", [d, f])}
    ts = []
    for i, l in enumerate(layers):
        for key, (stem, dims) in linears.items():
            ts.append((f"blk.{i}.{stem}.weight", (dims, bytes(l[key])), gguf.GGML_Q4_0))
        ts += [(f"blk.{i}.attn_norm.weight", l["ln1_w"], gguf.GGML_F32),
               (f"blk.{i}.attn_norm.bias", l["ln1_b"], gguf.GGML_F32),
               (f"blk.{i}.ffn_norm.weight", l["ln2_w"], gguf.GGML_F32),
               (f"blk.{i}.ffn_norm.bias", l["ln2_b"], gguf.GGML_F32)]
    ts += [("token_embd.weight", O.bf16_bits_to_f32_array(emb_bits).reshape(V, d), gguf.GGML_F32),
           ("output_norm.weight", fw, gguf.GGML_F32), ("output_norm.bias", fb, gguf.GGML_F32),
           ("output.weight", ([d, V], bytes(out)), gguf.GGML_Q4_0)]
    data = gguf.write_gguf(None, {"general.architecture": "llama"}, ts)
    a = D.Decoder(max_batch=4, max_seq=32, weight_fmt=N.Q4_0, kv_dtype=N.BF16, **cfg)
    _load(a, layers, emb_bits, fw, fb, out)
    b = D.Decoder(max_batch=4, max_seq=32, weight_fmt=N.Q4_0, kv_dtype=N.BF16, **cfg)
    b.load_gguf(data)
    seqs = [3, 8]
    toks = np.array([5, 17], dtype=np.int32)
    for _ in range(4):
        na, la = a.step(seqs, toks, want_logits=True)
        nb, lb = b.step(seqs, toks, want_logits=True)
        assert np.array_equal(la, lb) and np.array_equal(na, nb)
        toks = na
    a.close()
    b.close()
