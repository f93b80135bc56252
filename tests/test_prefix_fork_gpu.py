"""Prefix reuse on the paged KV cache (vxb_kv_fork) and in the decoder
(vxb_decoder_fork): a forked sequence shares its source's full blocks,
copies the partly filled last block, and from then on both sequences append
independently. The reference declares a prefix_cache map it never fills
(src/kv_cache.rs:37, 44); the allocator semantics otherwise follow
PagedKVCache (src/kv_cache.rs:41-93).

Checks: block tables and block accounting (shared blocks counted once, freed
with their last holder), gathered K/V bit-identical to the source prefix,
attention over the forked sequence against the oracle, and decoder logits of
a forked continuation against the f64 oracle stepping an independent copy of
the prefix (normwise <= 1e-2)."""
import copy

import numpy as np
import pytest

from oracle import oracle as O
from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("dtype", ["bf16", "int8"])
def test_kv_fork_shares_full_blocks(cuda_ok, dtype):
    from vortex_b200 import kv_cache as KV
    kd = KV.BF16 if dtype == "bf16" else KV.I8
    c = KV.PagedKVCache(2, 2, 128, 16, max_blocks=64, max_seqs=8, kv_dtype=kd)
    g = torch.Generator(device="cuda").manual_seed(3)
    for layer in range(2):
        k = torch.randn(37, 2, 128, device="cuda", generator=g).bfloat16()
        v = torch.randn(37, 2, 128, device="cuda", generator=g).bfloat16()
        c.append_seq(layer, 1, k, v)
    base = [c.get_kv(l, 1) for l in range(2)]
    c.fork(1, 2, 37)  # two shared blocks + a private copy of the partial third
    c.fork(1, 3, 32)  # exactly two shared blocks
    for l in range(2):
        t1, t2, t3 = c.block_table(l, 1), c.block_table(l, 2), c.block_table(l, 3)
        assert t2[:2] == t1[:2] and t3 == t1[:2] and t2[2] != t1[2]
        k2, v2 = c.get_kv(l, 2)
        k3, v3 = c.get_kv(l, 3)
        assert torch.equal(k2, base[l][0]) and torch.equal(v2, base[l][1])
        assert torch.equal(k3, base[l][0][:32]) and torch.equal(v3, base[l][1][:32])
    assert c.stats()["used_blocks"] == 2 * (3 + 1)
    # the sequences diverge: a new token each
    news = {}
    for s in (1, 2, 3):
        k = torch.randn(1, 2, 128, device="cuda", generator=g).bfloat16()
        v = torch.randn(1, 2, 128, device="cuda", generator=g).bfloat16()
        news[s] = (k, v)
        c.append_kv(0, [s], k, v)
    k1, _ = c.get_kv(0, 1)
    assert torch.equal(k1[:37], base[0][0])  # the shared prefix is untouched
    k3, _ = c.get_kv(0, 3)
    assert k3.shape[0] == 33 and torch.equal(k3[:32], base[0][0][:32])
    # attention over the forked sequence = the oracle over its own keys/values
    q = torch.randn(1, 4, 128, device="cuda", generator=g).bfloat16()
    out = c.attention(0, [2], q).float().cpu().numpy()[0]
    k2, v2 = (t.cpu().numpy().astype(np.float64) for t in c.get_kv(0, 2))
    qf = q.float().cpu().numpy().astype(np.float64)[0]
    for h in range(4):
        kh = h // 2
        want = O.paged_attention(qf[h], k2[:, kh].ravel(), v2[:, kh].ravel(), 128)
        assert rel_err(out[h], want) <= 1e-2
    c.free_seq(1)
    assert c.stats()["used_blocks"] == 2 * (2 + 1) + 1  # seq 2's blocks (3) + seq 3's new block (1)
    assert torch.equal(c.get_kv(1, 2)[0], base[1][0])
    c.free_seq(2)
    c.free_seq(3)
    assert c.stats()["used_blocks"] == 0


def test_decoder_fork_matches_oracle(cuda_ok):
    from oracle.llama_oracle import LlamaOracle
    from tests.parity import norm_err
    from tests.test_decoder_gpu import _build, _load
    from vortex_b200 import _native as N
    from vortex_b200 import decoder as D
    cfg = dict(vocab_size=512, dim=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn_dim=512, norm_eps=1e-5)
    layers, emb_bits, fw, fb, out = _build(cfg, 13, O.GGML_Q4_0)
    dec = D.Decoder(max_batch=4, max_seq=64, weight_fmt=N.Q4_0, **cfg)
    _load(dec, layers, emb_bits, fw, fb, out)
    orc = LlamaOracle(dict(cfg), layers, O.bf16_bits_to_f32_array(emb_bits), fw, fb, out, O.GGML_Q4_0)
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, 512, size=21)
    for t in prompt:  # token by token, so both sides hold the same 21 positions
        dec.step([7], np.array([t]))
        orc.step(7, int(t))
    dec.fork(7, 8, 21)
    orc.cache[8] = copy.deepcopy(orc.cache[7])
    toks = {7: 5, 8: 300}
    for step in range(4):
        ids = [7, 8]
        nxt, logits = dec.step(ids, np.array([toks[7], toks[8]]), want_logits=True)
        for i, s in enumerate(ids):
            ref = orc.step(s, toks[s])
            assert norm_err(logits[i], ref) <= 1e-2, (step, s)
        toks = {7: int(nxt[0]), 8: int(nxt[1])}
    dec.close()
