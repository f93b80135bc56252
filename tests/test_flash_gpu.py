"""K3 flash-attention forward (tcgen05) against the oracle's restatement of
flash_attention_forward / attention rows (src/flash_attention.rs:53-219).

The oracle runs in f64 on the same bf16-rounded inputs. Output is bf16, so the
gate is the floored max relative error <= 1e-2 (denominator max(|r|,
1e-3 * max|r|)); lse (f32) within 1e-3 relative.
"""
import numpy as np
import pytest

from tests.parity import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _inputs(B, S, H, Hkv, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, S, H, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, S, Hkv, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, S, Hkv, 128, device="cuda", generator=g).bfloat16()
    return q, k, v


def _oracle_rows(q, k, v, b, h, Hkv, H, rows, causal):
    from oracle import oracle as O
    hk = h // (H // Hkv)
    qh = q[b, :, h, :].float().cpu().numpy().astype(np.float64)
    kh = k[b, :, hk, :].float().cpu().numpy().astype(np.float64)
    vh = v[b, :, hk, :].float().cpu().numpy().astype(np.float64)
    return O.attention_rows(qh, kh, vh, 128, causal, rows)


@pytest.mark.parametrize("S,H,Hkv,causal", [(128, 2, 2, True), (256, 2, 2, False), (200, 2, 1, True),
                                             (384, 4, 2, True), (512, 2, 2, True), (512, 2, 2, False)])
def test_flash_full_check_small(cuda_ok, S, H, Hkv, causal):
    from vortex_b200 import attention as A
    B = 2 if S <= 256 else 1
    q, k, v = _inputs(B, S, H, Hkv, seed=S + H + 7 * causal)
    o, lse = A.flash_attention(q, k, v, causal=causal)
    torch.cuda.synchronize()
    rows = np.arange(S)
    for b in range(B):
        for h in range(H):
            ro, rl = _oracle_rows(q, k, v, b, h, Hkv, H, rows, causal)
            got = o[b, :, h, :].float().cpu().numpy()
            assert rel_err(got, ro) <= 1e-2, (b, h, rel_err(got, ro))
            gl = lse[b, h].cpu().numpy()
            assert np.max(np.abs(gl - rl) / np.maximum(1.0, np.abs(rl))) <= 1e-3


def test_flash_matches_reference_flash_path(cuda_ok):
    """Same result as the reference's tiled flash_attention_forward (oracle
    restatement, its own tile sizes) on one head."""
    from oracle import oracle as O
    from vortex_b200 import attention as A
    S = 256
    q, k, v = _inputs(1, S, 1, 1, seed=3)
    o, lse = A.flash_attention(q, k, v, causal=True)
    qh, kh, vh = (t[0, :, 0, :].float().cpu().numpy().astype(np.float64) for t in (q, k, v))
    t = O.flash_auto_tile(S, 128)
    ro, rl, _ = O.flash_attention_forward(qh, kh, vh, 128, t, t, True)
    assert rel_err(o[0, :, 0, :].float().cpu().numpy(), ro.reshape(S, 128)) <= 1e-2
    assert np.max(np.abs(lse[0, 0].cpu().numpy() - rl)) <= 1e-3 * np.max(np.abs(rl))


def test_flash_c3_shape_sampled_rows(cuda_ok):
    """The prefill benchmark shape (S=4096, d=128, causal) on one batch and two
    heads: the first and last 64 query rows and 64 random rows, each against
    the exact attention over all its visible keys."""
    from vortex_b200 import attention as A
    S, H = 4096, 2
    q, k, v = _inputs(1, S, H, H, seed=11)
    o, lse = A.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    rng = np.random.default_rng(5)
    rows = np.unique(np.concatenate([np.arange(64), np.arange(S - 64, S), rng.integers(64, S - 64, 64)]))
    for h in range(H):
        ro, rl = _oracle_rows(q, k, v, 0, h, H, H, rows, True)
        got = o[0, rows, h, :].float().cpu().numpy()
        assert rel_err(got, ro) <= 1e-2, (h, rel_err(got, ro))
        assert np.max(np.abs(lse[0, h, rows].cpu().numpy() - rl) / np.maximum(1.0, np.abs(rl))) <= 1e-3


def test_flash_c3_all_heads_sampled_rows(cuda_ok):
    """The prefill benchmark configuration itself (B=4, H=32, S=4096, d=128,
    causal, Q/K/V ~N(0,1) bf16): every one of the 128 (batch, head) pairs is
    checked on the first and last 64 query rows plus 256 random rows, each
    against the exact attention over all its visible keys (oracle in f64,
    heads spread over host threads)."""
    import concurrent.futures as cf
    import os

    from oracle import oracle as O
    from vortex_b200 import attention as A
    B, S, H = 4, 4096, 32
    q, k, v = _inputs(B, S, H, H, seed=4096)
    o, lse = A.flash_attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    on, ln = o.float().cpu().numpy(), lse.cpu().numpy()
    rng = np.random.default_rng(128)
    picks = [np.unique(np.concatenate([np.arange(64), np.arange(S - 64, S), rng.integers(64, S - 64, 256)]))
             for _ in range(B * H)]

    def check(bh):
        b, h = divmod(bh, H)
        rows = picks[bh]
        ro, rl = O.attention_rows(qn[b, :, h].astype(np.float64), kn[b, :, h].astype(np.float64),
                                  vn[b, :, h].astype(np.float64), 128, True, rows)
        e = rel_err(on[b, rows, h], ro)
        le = float(np.max(np.abs(ln[b, h, rows] - rl) / np.maximum(1.0, np.abs(rl))))
        return bh, e, le

    with cf.ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1)) as pool:
        results = list(pool.map(check, range(B * H)))
    assert len(results) == 128
    worst = max(results, key=lambda r: r[1])
    assert worst[1] <= 1e-2, worst
    assert max(r[2] for r in results) <= 1e-3


def test_flash_multi_head_layout(cuda_ok):
    """multi_head_flash_attention's [N, H*d] interleaved-head layout."""
    from oracle import oracle as O
    from vortex_b200 import attention as A
    n, H = 160, 2
    g = torch.Generator(device="cuda").manual_seed(9)
    q, k, v = (torch.randn(n, H * 128, device="cuda", generator=g).bfloat16() for _ in range(3))
    o = A.multi_head_flash_attention(q, k, v, H, 128, causal=True)
    ref = O.multi_head_flash_attention(*(t.float().cpu().numpy() for t in (q, k, v)), H, 128, True)
    assert rel_err(o.float().cpu().numpy(), ref.reshape(n, H * 128)) <= 1e-2


def test_flash_rejects_unsupported_head_dim(cuda_ok):
    from vortex_b200 import _native as N
    from vortex_b200 import attention as A
    q = torch.zeros(1, 64, 2, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(N.VxbError) as e:
        A.flash_attention(q, q, q)
    assert e.value.code == N.VXB_EUNSUPPORTED
