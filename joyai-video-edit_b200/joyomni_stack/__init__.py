"""Caller harness for BASELINE configs 4 and 5: a synthetic MMDiT double-stream
block stack whose joyomni_ops calls run on this repository's sm_100a kernels,
with Ulysses sequence parallelism across GPUs (ulysses.py)."""
from .ulysses import SeqParallel, shard_range, split_sizes  # noqa: F401


def __getattr__(name):
    # mmdit imports joyomni_ops (CUDA library); load it lazily so the Ulysses
    # plumbing can be used and tested without the library.
    if name in ("StackConfig", "Stack", "Block", "LayerKV", "rope_tables"):
        from . import mmdit
        return getattr(mmdit, name)
    raise AttributeError(name)
