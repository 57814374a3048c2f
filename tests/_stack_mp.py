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
    x, txt = st.inputs(1)
    for _ in range(2):
        x = st.denoise_chunk(x, txt)
    sizes = [st.sp.shard_len(r) for r in range(world)]
    from joyomni_stack import split_sizes
    isz = split_sizes(cfg.img_tokens, world)
    parts = [torch.empty((isz[r], cfg.hidden), device=dev) for r in range(world)]
    dist.all_gather(parts, x.contiguous()) if len(set(isz)) == 1 else [
        dist.broadcast(parts[r].copy_(x) if r == rank else parts[r], src=r) for r in range(world)]
    full = torch.cat(parts, 0)
    if rank == 0:
        sp1 = SeqParallel(None, 1, 0, cfg.img_tokens, cfg.txt_tokens, cfg.heads)
        st1 = Stack(cfg, dev, sp=sp1)
        y, t1 = st1.inputs(1)
        for _ in range(2):
            y = st1.denoise_chunk(y, t1)
        rel = ((full - y).pow(2).mean().sqrt() / y.pow(2).mean().sqrt()).item()
        print("rel", rel, "sizes", sizes, flush=True)
        if rel <= 1e-3:
            print("ULYSSES_OK", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
