"""Flash-attention backward (f4) on the device against the oracle's
restatement of flash_attention_backward (src/flash_attention.rs:227-317).

The oracle runs in f64 on the same bf16 inputs, with the forward output and
lse the device produced (the backward's own inputs). Gradients are f32;
gate: floored max relative error <= 1e-2 per head (denominator max(|r|,
1e-3 max|r|)), as the forward's bf16 outputs."""
import numpy as np
import pytest

from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("B,S,H,Hkv,causal", [(1, 64, 1, 1, False), (2, 100, 2, 2, True), (1, 256, 4, 2, True),
                                               (1, 200, 2, 1, False), (2, 384, 2, 2, True)])
def test_flash_backward_matches_oracle(cuda_ok, B, S, H, Hkv, causal):
    from oracle import oracle as O
    from vortex_b200 import attention as A
    g = torch.Generator(device="cuda").manual_seed(S + H)
    q = torch.randn(B, S, H, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, Hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, 128, device="cuda", generator=g).bfloat16()
    do = torch.randn(B, S, H, 128, device="cuda", generator=g).bfloat16()
    o, lse = A.flash_attention(q, k, v, causal=causal)
    dq, dk, dv = A.flash_attention_backward(q, k, v, o, do, lse, causal=causal)
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    qn, kn, vn, on, don, ln = f(q), f(k), f(v), f(o), f(do), lse.cpu().numpy().astype(np.float64)
    dqn, dkn, dvn = (t.cpu().numpy() for t in (dq, dk, dv))
    G = H // Hkv
    for b in range(B):
        gk_sum = np.zeros((Hkv, S, 128))
        gv_sum = np.zeros((Hkv, S, 128))
        for h in range(H):
            hk = h // G
            rq, rk, rv = O.flash_attention_backward(qn[b, :, h], kn[b, :, hk], vn[b, :, hk], on[b, :, h],
                                                    don[b, :, h], ln[b, h], 128, 32, 32, causal)
            assert rel_err(dqn[b, :, h], rq) <= 1e-2, ("dq", b, h, rel_err(dqn[b, :, h], rq))
            gk_sum[hk] += rk.reshape(S, 128)
            gv_sum[hk] += rv.reshape(S, 128)
        for hk in range(Hkv):
            assert rel_err(dkn[b, :, hk], gk_sum[hk]) <= 1e-2, ("dk", b, hk, rel_err(dkn[b, :, hk], gk_sum[hk]))
            assert rel_err(dvn[b, :, hk], gv_sum[hk]) <= 1e-2, ("dv", b, hk, rel_err(dvn[b, :, hk], gv_sum[hk]))


def test_flash_backward_builtin(cuda_ok):
    """The builtin adapter (per head, non-causal as the reference's adapter)."""
    from oracle import oracle as O
    from tests.parity import bf16_round
    from vortex_b200 import builtins as Bi
    rng = np.random.default_rng(2)
    n, H = 48, 2
    q, k, v, do = (bf16_round(rng.standard_normal((n, H * 128))).astype(np.float64) for _ in range(4))
    out = O.multi_head_flash_attention(q, k, v, H, 128, False).reshape(n, H * 128)
    out_b = bf16_round(out).astype(np.float64)
    gq, gk, gv = (np.array(t) for t in Bi.flash_attention_backward(q.tolist(), k.tolist(), v.tolist(),
                                                                   out_b.tolist(), do.tolist(), H, True))
    for h in range(H):
        sl = slice(h * 128, (h + 1) * 128)
        _, lse, _ = O.flash_attention_forward(q[:, sl], k[:, sl], v[:, sl], 128, 32, 32, False)
        rq, rk, rv = O.flash_attention_backward(q[:, sl], k[:, sl], v[:, sl], out_b[:, sl], do[:, sl], lse, 128, 32,
                                                32, False)
        assert rel_err(gq[:, sl], rq) <= 1e-2
        assert rel_err(gk[:, sl], rk) <= 1e-2
        assert rel_err(gv[:, sl], rv) <= 1e-2
