"""Tensor-parallel decoder on 2 GPUs (one process per GPU, NCCL): the same
model (random init, or full host weights sliced per rank by set_weight) gives
the same logits and greedy tokens as the single-GPU decoder. Skipped with
fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CFG = dict(vocab_size=512, dim=256, n_layers=2, n_heads=4, n_kv_heads=2, ffn_dim=512, norm_eps=1e-5)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _host_weights(seed):
    """Full model as GGUF Q4_0 blocks / f32 / bf16 host arrays."""
    from oracle import oracle as O
    from vortex_b200 import decoder as D
    rng = np.random.default_rng(seed)
    c = CFG
    hd = c["dim"] // c["n_heads"]
    kvd = c["n_kv_heads"] * hd
    q = lambda n, k: O.quantize_blocks(O.GGML_Q4_0, rng.normal(0, 0.05, n * k).astype(np.float32))
    w = []
    for l in range(c["n_layers"]):
        w += [(l, D.WQ, q(c["dim"], c["dim"])), (l, D.WK, q(kvd, c["dim"])), (l, D.WV, q(kvd, c["dim"])),
              (l, D.WO, q(c["dim"], c["dim"])), (l, D.W1, q(c["ffn_dim"], c["dim"])),
              (l, D.W2, q(c["dim"], c["ffn_dim"])), (l, D.W3, q(c["ffn_dim"], c["dim"]))]
        for which in (D.LN1_W, D.LN2_W):
            w.append((l, which, (1 + 0.1 * rng.standard_normal(c["dim"])).astype(np.float32)))
        for which in (D.LN1_B, D.LN2_B):
            w.append((l, which, (0.01 * rng.standard_normal(c["dim"])).astype(np.float32)))
    emb = O.f32_array_to_bf16_bits(rng.normal(0, 1.0, c["vocab_size"] * c["dim"]).astype(np.float32))
    w += [(-1, D.EMBED, emb), (-1, D.FINAL_W, np.ones(c["dim"], np.float32)),
          (-1, D.FINAL_B, np.zeros(c["dim"], np.float32)), (-1, D.OUTPUT, q(c["vocab_size"], c["dim"]))]
    return w


def _run(dec, steps, B):
    rng = np.random.default_rng(1)
    toks = rng.integers(0, CFG["vocab_size"], size=B)
    out = []
    for _ in range(steps):
        nxt, logits = dec.step(list(range(B)), toks, want_logits=True)
        out.append((nxt.copy(), logits.copy()))
        toks = nxt
    return out


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist

    from vortex_b200 import comm as C
    from vortex_b200 import decoder as D
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = C.share_unique_id(rank)
        comm = C.Comm(world, rank, uid, device=rank)
        dec = D.Decoder(max_batch=3, max_seq=16, comm=comm, **CFG)
        if mode == "random":
            dec.init_random(seed=5, sigma=0.05)
        else:
            for layer, which, data in _host_weights(7):
                dec.set_weight(layer, which, data)
        res = _run(dec, 4, 3)
        dec.close()
        comm.close()
        q.put((rank, res))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["random", "host_weights"])
def test_tp2_decoder_matches_single_gpu(cuda_ok, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from tests.parity import norm_err
    from vortex_b200 import decoder as D
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
    ref_dec = D.Decoder(max_batch=3, max_seq=16, **CFG)
    if mode == "random":
        ref_dec.init_random(seed=5, sigma=0.05)
    else:
        for layer, which, data in _host_weights(7):
            ref_dec.set_weight(layer, which, data)
    ref = _run(ref_dec, 4, 3)
    ref_dec.close()
    for (n0, l0), (n1, l1), (nr, lr) in zip(got[0], got[1], ref):
        assert np.array_equal(n0, n1)  # every rank decides the same token
        np.testing.assert_array_equal(l0, l1)
        assert norm_err(l0, lr) <= 1e-4, norm_err(l0, lr)
        for b in range(lr.shape[0]):
            top2 = np.sort(lr[b])[-2:]
            if top2[1] - top2[0] > 1e-3 * np.max(np.abs(lr[b])):  # no near tie
                assert n0[b] == nr[b]


def _ar_worker(rank, world, port, q):
    import torch.distributed as dist

    from vortex_b200 import comm as C
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        comm = C.Comm(world, rank, C.share_unique_id(rank), device=rank)
        res = []
        for n in (1, 4097, 131072, 400000):  # the last one (1.6 MB) goes through NCCL
            for it in range(3):  # reuse of both peer-buffer slots
                g = torch.Generator(device="cuda").manual_seed(1000 * n + 10 * it + rank)
                t = torch.randn(n, device="cuda", generator=g)
                comm.allreduce_sum(t)
                torch.cuda.synchronize()
                res.append(t.cpu().numpy())
        comm.close()
        q.put((rank, res))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_allreduce_sum_peer_memory_and_nccl_paths(cuda_ok):
    """vxb_allreduce_sum on 2 GPUs: both ranks hold the elementwise f32 sum of
    the two inputs (rank order), for one-shot (<= 512 KiB) and NCCL sizes."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
    k = 0
    for n in (1, 4097, 131072, 400000):
        for it in range(3):
            ins = []
            for r in range(2):
                g = torch.Generator(device="cuda").manual_seed(1000 * n + 10 * it + r)
                ins.append(torch.randn(n, device="cuda", generator=g).cpu().numpy())
            want = ins[0] + ins[1]
            np.testing.assert_array_equal(got[0][k], got[1][k])
            if n <= 262144:
                np.testing.assert_array_equal(got[0][k], want)
            else:
                np.testing.assert_allclose(got[0][k], want, rtol=1e-6, atol=1e-6)
            k += 1


def _fixture():
    from tests.golden import make_tp_fixture as M
    return M, np.load(M.PATH)


def _fixture_err(dec, fx):
    """Largest normwise logits error of a decoder against the oracle fixture
    (prefill logits and every teacher-forced decode step)."""
    from tests.parity import norm_err
    ids = [int(s) for s in fx["seq_ids"]]
    pre, steps = dec.score(ids, fx["prompts"], fx["tokens"])
    errs = [norm_err(pre[i], fx["prefill_logits"][i]) for i in range(len(ids))]
    errs += [norm_err(steps[t, i], fx["logits"][t, i]) for t in range(steps.shape[0]) for i in range(len(ids))]
    return max(errs)


def test_fixture_decoder_matches_oracle_single_gpu(cuda_ok):
    """The tensor-parallel fixture model on one GPU (prefill + teacher-forced
    decode) against the oracle's logits: normwise <= 1e-2."""
    from vortex_b200 import decoder as D
    from vortex_b200.decoder import synthetic_weights
    M, fx = _fixture()
    dec = D.Decoder(max_batch=4, max_seq=32, **M.CFG)
    dec.load_float_weights(synthetic_weights(M.CFG, M.SEED))
    err = _fixture_err(dec, fx)
    dec.close()
    assert err <= 1e-2, err


def _fixture_worker(rank, world, port, q):
    import torch.distributed as dist

    from vortex_b200 import comm as C
    from vortex_b200 import decoder as D
    from vortex_b200.decoder import synthetic_weights
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, fx = _fixture()
        comm = C.Comm(world, rank, C.share_unique_id(rank), device=rank)
        dec = D.Decoder(max_batch=4, max_seq=32, comm=comm, **M.CFG)
        dec.load_float_weights(synthetic_weights(M.CFG, M.SEED))
        err = _fixture_err(dec, fx)
        dec.close()
        comm.close()
        q.put((rank, err))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_fixture_decoder_matches_oracle_tp2(cuda_ok):
    """The same model split over 2 GPUs (heads, FFN rows, vocabulary) against
    the oracle's logits on every rank."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fixture_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        assert got[r] <= 1e-2, (r, got[r])
