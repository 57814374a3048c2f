"""Setting up the peer-memory exchange of the block stack is collective: if
any rank fails (e.g. cannot map a peer's region), every rank falls back to
the NCCL all-to-all path together, without a rank left waiting in a barrier.
CPU, gloo, world size 2; the failure is made on the host."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _FakeRegion:
    def __init__(self):
        self.closed_with = None

    def close(self, barrier=True):
        self.closed_with = barrier


def _worker(rank, world, port, fail_ranks, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from joyomni_stack import mmdit
        from joyomni_stack.mmdit import Stack, StackConfig, LayerKV
        fake = _FakeRegion()

        def fake_peer_kv(self, n, cos, sin, device):
            if rank in fail_ranks:
                raise RuntimeError("cannot map a peer region (injected)")
            self.region = fake
            return ["peer"] * n

        mmdit.Stack._peer_kv = fake_peer_kv
        cfg = StackConfig(hidden=256, heads=2, ffn=512, layers=2, img_tokens=20, txt_tokens=4, grid=(1, 4, 5),
                          cache_chunks=1, seed=3)
        st = Stack(cfg, torch.device("cpu"))
        nccl_path = all(isinstance(kv, LayerKV) and kv.peer is None for kv in st.kv)
        q.put((rank, nccl_path, st.region is None, fake.closed_with, getattr(st, "exchange_error", "")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_ranks", [(1,), (0, 1), ()])
def test_peer_exchange_setup_is_agreed(fail_ranks):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_ranks, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, nccl_path, no_region, closed_with, err in res:
        if fail_ranks:
            assert nccl_path and no_region, (rank, err)
            assert "peer" in err or "injected" in err
            if rank not in fail_ranks:
                assert closed_with is False       # unmapped after the common barrier
        else:
            assert not nccl_path and not no_region
