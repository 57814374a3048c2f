"""torchrun worker for test_ulysses_two_gpus_matches_one: runs 2 layers x 2
chunks with Ulysses over all ranks (NCCL), gathers the image output on rank 0
and compares it with a single-GPU run of the same seeded model."""
import os

import torch
import torch.distributed as dist

from joyomni_stack import SeqParallel, Stack, StackConfig


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))
    cfg = StackConfig(hidden=512, heads=4, ffn=1376, layers=2, img_tokens=130, txt_tokens=24, grid=(1, 10, 13),
                      cache_chunks=2, seed=11)
    st = Stack(cfg, dev)
    from joyomni_stack import split_sizes
    isz = split_sizes(cfg.img_tokens, world)

    def gather_img(t):
        parts = [torch.empty((isz[r], t.shape[1]), device=dev, dtype=t.dtype) for r in range(world)]
        for r in range(world):
            buf = t.contiguous() if r == rank else parts[r]
            dist.broadcast(buf, src=r)
            parts[r] = buf
        return torch.cat(parts, 0)

    # (a) one block forward from identical inputs (no cache)
    x0, txt0 = st.inputs(1)
    vec = st.timestep_vec(1000)
    b_img, _ = st.blocks[0].forward(x0.to(torch.bfloat16), txt0, vec, st.cos, st.sin, st.kv[0], st.sp)
    b_full = gather_img(b_img)
    x, txt = st.inputs(1)
    for _ in range(2):
        x = st.denoise_chunk(x, txt)
    sizes = [st.sp.shard_len(r) for r in range(world)]
    full = gather_img(x)
    if rank == 0:
        def rel(a, b):
            a, b = a.float(), b.float()
            return ((a - b).pow(2).mean().sqrt() / b.pow(2).mean().sqrt()).item()
        sp1 = SeqParallel(None, 1, 0, cfg.img_tokens, cfg.txt_tokens, cfg.heads)
        st1 = Stack(cfg, dev, sp=sp1)
        y0, t0 = st1.inputs(1)
        b1, _ = st1.blocks[0].forward(y0.to(torch.bfloat16), t0, st1.timestep_vec(1000), st1.cos, st1.sin,
                                      st1.kv[0], st1.sp)
        y, t1 = st1.inputs(1)
        for _ in range(2):
            y = st1.denoise_chunk(y, t1)
        rb, rc = rel(b_full, b1), rel(full, y)
        print("block_rel", rb, "chunks_rel", rc, "sizes", sizes, flush=True)
        if rb <= 1e-2 and rc <= 1e-1:
            print("ULYSSES_OK", flush=True)
    st.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
