"""Ulysses exchange logic on CPU with gloo, world size 2 (and 3 for uneven
shards): sequence->head->sequence round trip, and attention computed head-
sharded equals attention on the full sequence."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from joyomni_stack.ulysses import SeqParallel, split_sizes


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, img, txt, heads, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        Dh = 8
        L = img + txt
        full = torch.randn(3, L, heads, Dh)          # q, k, v for the whole sequence (img then txt)
        sp = SeqParallel.create(img, txt, heads)
        a, b = sp.img_range
        c, d = sp.txt_range
        local = torch.cat((full[:, a:b], full[:, img + c: img + d]), 1)   # this rank's tokens
        # round trip
        back = sp.heads_to_seq(sp.seq_to_heads(local[0]))
        ok_rt = torch.equal(back, local[0])
        # attention: head-sharded over the gathered (rank-ordered) sequence
        qh, kh, vh = (sp.seq_to_heads(local[i]) for i in range(3))
        o = torch.nn.functional.scaled_dot_product_attention(qh.permute(1, 0, 2)[None], kh.permute(1, 0, 2)[None],
                                                             vh.permute(1, 0, 2)[None])
        o = sp.heads_to_seq(o[0].permute(1, 0, 2).contiguous())
        ref = torch.nn.functional.scaled_dot_product_attention(full[0].permute(1, 0, 2)[None],
                                                               full[1].permute(1, 0, 2)[None],
                                                               full[2].permute(1, 0, 2)[None])[0].permute(1, 0, 2)
        ref_local = torch.cat((ref[a:b], ref[img + c: img + d]), 0)
        err = (o - ref_local).abs().max().item()
        q.put((rank, ok_rt, err, sp.local_len))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,img,txt,heads", [(2, 37, 5, 4), (3, 40, 7, 6), (2, 3, 1, 2)])
def test_ulysses_exchange_and_attention(world, img, txt, heads):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, img, txt, heads, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(r[3] for r in res) == sorted(split_sizes(img, world)[r] + split_sizes(txt, world)[r]
                                               for r in range(world))
    for rank, ok_rt, err, _ in res:
        assert ok_rt, f"rank {rank}: round trip differs"
        assert err < 1e-5, f"rank {rank}: attention error {err}"


def test_split_sizes():
    assert split_sizes(10530, 8) == [1317, 1317] + [1316] * 6
    assert sum(split_sizes(512, 3)) == 512
