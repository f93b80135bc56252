"""GGUF -> decoder weight slots (vortex_b200.decoder.gguf_decoder_weights): a
Llama-style GGUF written with llama.cpp tensor names maps to the decoder's
slots with the oracle's block codes (bit-exact), f32 norms, zero biases where
the file has none, the embedding as bf16 by the tensor_engine::f32_to_bf16
rule, and errors that name the offending tensor. CPU only."""
import numpy as np
import pytest

from oracle import oracle as O

CFG = dict(vocab_size=96, dim=64, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=128)


def _tensors(fmt, rng, with_bias):
    from vortex_b200 import gguf
    d, f, V = CFG["dim"], CFG["ffn_dim"], CFG["vocab_size"]
    kvd = CFG["n_kv_heads"] * (d // CFG["n_heads"])
    shapes = {"attn_q": (d, d), "attn_k": (kvd, d), "attn_v": (kvd, d), "attn_output": (d, d),
              "ffn_gate": (f, d), "ffn_down": (d, f), "ffn_up": (f, d)}
    ts, ref = [], {}
    for i in range(CFG["n_layers"]):
        for stem, (n, k) in shapes.items():
            w = rng.normal(0, 0.05, (n, k)).astype(np.float32)
            ts.append((f"blk.{i}.{stem}.weight", w, fmt))
            ref[f"blk.{i}.{stem}.weight"] = O.quantize_blocks(fmt, w.astype(np.float64))
        for nm in ("attn_norm", "ffn_norm"):
            w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
            ts.append((f"blk.{i}.{nm}.weight", w, gguf.GGML_F32))
            ref[f"blk.{i}.{nm}.weight"] = w
            if with_bias:
                b = (0.1 * rng.standard_normal(d)).astype(np.float32)
                ts.append((f"blk.{i}.{nm}.bias", b, gguf.GGML_F16))
                ref[f"blk.{i}.{nm}.bias"] = b.astype(np.float16).astype(np.float32)
    emb = rng.standard_normal((V, d)).astype(np.float32)
    ts.append(("token_embd.weight", emb, gguf.GGML_F32))
    ref["token_embd.weight"] = O.f32_array_to_bf16_bits(emb)
    fw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    ts.append(("output_norm.weight", fw, gguf.GGML_F32))
    ref["output_norm.weight"] = fw
    out = rng.normal(0, 0.05, (V, d)).astype(np.float32)
    ts.append(("output.weight", out, fmt))
    ref["output.weight"] = O.quantize_blocks(fmt, out.astype(np.float64))
    return ts, ref


@pytest.mark.parametrize("fmt", [2, 8])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gguf_maps_to_decoder_slots(fmt, with_bias):
    from vortex_b200 import decoder as D
    from vortex_b200 import gguf
    ts, ref = _tensors(fmt, np.random.default_rng(fmt + with_bias), with_bias)
    f = gguf.GGUFFile(gguf.write_gguf(None, {"general.architecture": "llama"}, ts))
    got = D.gguf_decoder_weights(f, dict(CFG, weight_fmt=fmt))
    names = {D.WQ: "attn_q", D.WK: "attn_k", D.WV: "attn_v", D.WO: "attn_output", D.W1: "ffn_gate",
             D.W2: "ffn_down", D.W3: "ffn_up"}
    norms = {D.LN1_W: "attn_norm.weight", D.LN1_B: "attn_norm.bias", D.LN2_W: "ffn_norm.weight",
             D.LN2_B: "ffn_norm.bias"}
    seen = set()
    for layer, slot, a in got:
        seen.add((layer, slot))
        if layer >= 0 and slot in names:
            assert a.dtype == np.uint8 and a.tobytes() == bytes(ref[f"blk.{layer}.{names[slot]}.weight"])
        elif layer >= 0:
            key = f"blk.{layer}.{norms[slot]}"
            want = ref.get(key, np.zeros(CFG["dim"], np.float32))
            assert a.dtype == np.float32 and np.array_equal(a, want), key
        elif slot == D.EMBED:
            assert a.dtype == np.uint16 and a.shape == (CFG["vocab_size"], CFG["dim"])
            assert np.array_equal(a, ref["token_embd.weight"])
        elif slot == D.FINAL_W:
            assert np.array_equal(a, ref["output_norm.weight"])
        elif slot == D.FINAL_B:
            assert np.array_equal(a, np.zeros(CFG["dim"], np.float32))
        else:
            assert slot == D.OUTPUT and a.tobytes() == bytes(ref["output.weight"])
    assert len(seen) == CFG["n_layers"] * 11 + 4 == len(got)


def test_gguf_decoder_weights_errors_name_the_tensor():
    from vortex_b200 import decoder as D
    from vortex_b200 import gguf
    ts, _ = _tensors(2, np.random.default_rng(0), False)
    cfg = dict(CFG, weight_fmt=2)
    f = gguf.GGUFFile(gguf.write_gguf(None, {}, [t for t in ts if t[0] != "output.weight"]))
    with pytest.raises(ValueError, match="'output.weight' is missing"):
        D.gguf_decoder_weights(f, cfg)
    f = gguf.GGUFFile(gguf.write_gguf(None, {}, ts))
    with pytest.raises(ValueError, match="'blk.0.attn_q.weight' has ggml type 2"):
        D.gguf_decoder_weights(f, dict(cfg, weight_fmt=8))
    with pytest.raises(ValueError, match="'blk.0.attn_k.weight' has dims"):
        D.gguf_decoder_weights(f, dict(cfg, n_kv_heads=4))
