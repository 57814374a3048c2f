"""Ulysses exchange logic on CPU with gloo, world size 2 (and 3 for uneven
shards): sequence->head->sequence round trip, attention computed head-
sharded equals attention on the full sequence, and the segment table of the
scattering attention epilogue rebuilds each rank's rows exactly as the
head->sequence all-to-all does."""
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
        # the attention epilogue's scatter rule (jo_attention_fwd_scatter with
        # the segment table gathered_segment_starts): row i of rank r's
        # head-sharded output goes to the owner k of row i at token
        # i - starts[k], heads r * H/P .. -- emulated here with every rank's
        # head-sharded output, it must rebuild exactly what heads_to_seq gives
        hs = qh.contiguous()
        every = [torch.empty_like(hs) for _ in range(world)]
        dist.all_gather(every, hs)
        starts = sp.gathered_segment_starts()
        mine = torch.full((sp.local_len, heads, Dh), float("nan"))
        hpr = heads // world
        for r in range(world):
            for i in range(starts[rank], starts[rank + 1]):
                mine[i - starts[rank], r * hpr:(r + 1) * hpr] = every[r][i]
        ok_sc = starts[-1] == sp.total_len and torch.equal(mine, sp.heads_to_seq(hs))
        q.put((rank, ok_rt and ok_sc, err, sp.local_len))
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
