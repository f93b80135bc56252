"""Host side of the tensor-parallel communicator on CPU: two gloo ranks share
a 128-byte unique id through share_unique_id (rank 0 makes it, every rank
receives the same bytes). No GPU and no NCCL call: the id maker is a fake."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from vortex_b200 import comm as C
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = C.share_unique_id(rank, make=lambda: bytes(range(128)))
        q.put((rank, uid))
    finally:
        dist.destroy_process_group()


def test_share_unique_id_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] == bytes(range(128))


def test_share_unique_id_rejects_malformed_id():
    """A maker returning something other than 128 bytes is refused (single
    gloo rank)."""
    import torch.distributed as dist

    from vortex_b200 import _native as N
    from vortex_b200 import comm as C
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        with pytest.raises(N.VxbError):
            C.share_unique_id(0, make=lambda: b"short")
    finally:
        dist.destroy_process_group()
