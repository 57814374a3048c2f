"""Synthetic MMDiT double-stream block stack routed through joyomni_ops.

This is the caller harness of BASELINE configs 4 and 5: the block arithmetic of
the reference's ``MMDoubleStreamBlock.forward`` (deploy/xvideo/models/dit/dit.py:314-481)
with every joyomni_ops call served by the sm_100a kernels of this repository,
random-initialised weights and synthetic inputs.  Per block and stream:

  mod  = modulate_table + vec -> shift1, scale1, gate1, shift2, scale2, gate2   (dit.py:112-125)
  x_q  = per_token_fp8(LayerNorm(x) * (1 + scale1) + shift1)      fused entry  (dit.py:351-357 + fp8_linear.py:143-166)
  qkv  = fp8_scaled_mm(x_q, W_qkv) + b                                          (fp8_linear.py:167)
  q, k = RMSNorm_head + 3D RoPE, in place in the qkv buffer (image stream);     (dit.py:364-370)
         RMSNorm_head only (text stream)                                        (dit.py:384-385)
  attn = attention(q_img|q_txt, [k_cache | k_img | k_txt], [v ...])              (dit.py:387-420)
         (tcgen05 kernel of this repository, or torch SDPA with cfg.attention = "sdpa")
  x    = x + gate1 * fp8_linear(attn, W_proj)     residual in the GEMM epilogue  (dit.py:463-466)
  x    = x + gate2 * fp8_linear(gelu_tanh(fp8_linear(mod2(LN(x)), W_up)), W_down)  (dit.py:467-476)
         (GELU in the up-projection epilogue, gated residual in the down-projection epilogue)

Differences from the reference model that the synthetic configuration asks
for or that are harness simplifications: BASELINE's dims (hidden 5120, 40
heads, FFN 13824, RoPE split 44/42/42); the KV cache stores post-RoPE keys of
the image tokens of the last 2 chunks (or pre-RoPE keys, kv_cache_pre_rope),
written from the last denoising step, or with store_pass=True from an extra
forward on the clean latent as the reference does; the latent <-> token projections and
the Euler update act directly in token space.  Sequence parallelism (Ulysses,
ulysses.py) is new; with P = 1 it degenerates to plain single-GPU execution.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.nn.functional as F

import joyomni_ops as jo

from .ulysses import SeqParallel, shard_range, split_sizes

NORM_EPS = 1e-6
FP8 = torch.float8_e4m3fn


@dataclass
class StackConfig:
    hidden: int = 5120
    heads: int = 40
    ffn: int = 13824
    layers: int = 40
    img_tokens: int = 10530          # 3 latent frames x 45 x 78 patches
    txt_tokens: int = 512
    grid: tuple = (3, 45, 78)        # (t, h, w) of the image tokens, row-major
    rope_axes: tuple = (44, 42, 42)
    rope_theta: float = 10000.0
    cache_chunks: int = 2
    seed: int = 5
    # attention kernel: "joyomni" (tcgen05 kernel of this repository) or "sdpa"
    # (torch cuDNN / flash); JOYOMNI_ATTENTION overrides the default
    attention: str = field(default_factory=lambda: os.environ.get("JOYOMNI_ATTENTION", "joyomni"))
    # KV cache of pre-RoPE keys (the reference's kv_cache_pre_rope=True,
    # dit.py:360-363): keys are cached after the per-head RMSNorm only and
    # rotated at their window positions when the cache is assembled.
    kv_cache_pre_rope: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def rope_tables(cfg: StackConfig, device, t0: int = 0, fp32: bool = False) -> tuple:
    """cos/sin [T*H*W, head_dim/2] for the row-major (t, h, w) grid with
    temporal positions t0 .. t0+T-1: per axis f_j = 1/theta^(2j/d), angle =
    pos * f_j (fp32); the de-duplicated half of the repeat_interleaved tables
    (rope.py:31-52, sgl_fused_ops.py:87-94), rounded to bf16 for the fused
    QK-norm + RoPE kernel, or kept in fp32 (fp32=True) for rotating cached
    pre-RoPE keys (apply_rotary_emb's fp32 tables, dit.py:955-973)."""
    T, H, W = cfg.grid
    tt, hh, ww = torch.meshgrid(torch.arange(T) + t0, torch.arange(H), torch.arange(W), indexing="ij")
    cs, sn = [], []
    for pos, d in zip((tt, hh, ww), cfg.rope_axes):
        f = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2)[: d // 2].float() / d))
        ang = torch.outer(pos.reshape(-1).float(), f)
        cs.append(ang.cos())
        sn.append(ang.sin())
    dt = torch.float32 if fp32 else torch.bfloat16
    return (torch.cat(cs, 1).to(dt).to(device).contiguous(),
            torch.cat(sn, 1).to(dt).to(device).contiguous())


class Fp8Weight:
    """Per-output-channel FP8 weight in the reference's layout
    (deploy/xvideo/models/dit/fp8_linear.py:100-110): column-major [K, N] e4m3
    codes with scale = max(absmax_k |W[n, :]|, 1e-8) / 448, bias in bf16."""

    def __init__(self, n: int, k: int, gen: torch.Generator, device, std: float = 0.02):
        w = torch.randn((n, k), generator=gen, device=device, dtype=torch.bfloat16) * std
        amax = w.abs().amax(dim=1).float().clamp_min(1e-8)
        self.scale = (amax / 448.0).contiguous()
        self.codes = (w.float() / self.scale[:, None]).clamp(-448, 448).to(FP8)   # [N, K] row-major
        self.b = (torch.randn(n, generator=gen, device=device, dtype=torch.bfloat16) * 0.01).contiguous()
        del w

    @property
    def t(self):  # column-major [K, N] view, as fp8_scaled_mm wants
        return self.codes.t()

    def __call__(self, xq, xs, gelu=False, out=None):
        f = jo.fp8_scaled_mm_gelu if gelu else jo.fp8_scaled_mm
        return f(xq, self.t, xs, self.scale, torch.bfloat16, self.b, out=out)

    def scatter(self, xq, xs, dst_ptrs, ranks, heads_per_rank, head_dim, tok0, dst_tokens):
        """QKV projection with the sequence-parallel all-to-all in its epilogue:
        every (token, head) is stored in the owning rank's q / k / v buffer."""
        jo.fp8_scaled_mm_scatter(xq, self.t, xs, self.scale, torch.bfloat16, self.b, dst_ptrs, 3, ranks,
                                 heads_per_rank, head_dim, tok0, dst_tokens)

    def residual(self, xq, xs, res, gate, out=None):
        """res + gate * (x @ W + b), gated residual fused in the GEMM epilogue."""
        return jo.fp8_scaled_mm_residual(xq, self.t, xs, self.scale, torch.bfloat16, self.b, res, gate, out=out)


def attend(q, k, v, backend: str):
    """Non-causal attention of head-sharded q [Lq, h, 128] over k, v [Lk, h, 128]
    (the block's FA4 / SDPA call, dit.py:150-178, 419), returning [Lq, h, 128].
    backend "joyomni": this repository's tcgen05 kernel (joyomni_ops.attention,
    strided views read in place); "sdpa": torch SDPA (cuDNN / flash), bf16."""
    if backend == "joyomni":
        return jo.attention(q, k, v)
    with torch.nn.attention.sdpa_kernel([torch.nn.attention.SDPBackend.CUDNN_ATTENTION,
                                         torch.nn.attention.SDPBackend.FLASH_ATTENTION,
                                         torch.nn.attention.SDPBackend.EFFICIENT_ATTENTION]):
        o = F.scaled_dot_product_attention(q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None],
                                           v.permute(1, 0, 2)[None])
    return o[0].permute(1, 0, 2)


def quant(x):
    q = torch.empty(x.shape, dtype=FP8, device=x.device)
    s = torch.empty((x.shape[0], 1), dtype=torch.float32, device=x.device)
    jo.sgl_per_token_quant_fp8(x, q, s)
    return q, s


def norm_mod_quant(x, shift, scale):
    q = torch.empty(x.shape, dtype=FP8, device=x.device)
    s = torch.empty((x.shape[0], 1), dtype=torch.float32, device=x.device)
    jo.norm_modulate_quant_fp8(x, None, None, scale, shift, "layer", NORM_EPS, q, s)
    return q, s


class Stream:
    """Weights of one stream (image or text) of one block."""

    def __init__(self, cfg: StackConfig, gen, device):
        D, Fh, Dh = cfg.hidden, cfg.ffn, cfg.head_dim
        self.mod = (torch.randn((6, D), generator=gen, device=device) / math.sqrt(D)).to(torch.bfloat16)
        self.qkv = Fp8Weight(3 * D, D, gen, device)
        self.proj = Fp8Weight(D, D, gen, device)
        self.up = Fp8Weight(Fh, D, gen, device)
        self.down = Fp8Weight(D, Fh, gen, device)
        self.q_norm = (1 + 0.1 * torch.randn(Dh, generator=gen, device=device)).to(torch.bfloat16)
        self.k_norm = (1 + 0.1 * torch.randn(Dh, generator=gen, device=device)).to(torch.bfloat16)


class LayerKV:
    """Head-sharded K/V of one layer: [current | cache slot 0 | cache slot 1] along
    tokens, so the all-to-all writes the current chunk's keys straight into the
    buffer and the attention keys are one contiguous prefix."""

    def __init__(self, cfg: StackConfig, sp: SeqParallel, device, k=None, v=None):
        self.cap = cfg.cache_chunks * cfg.img_tokens
        n = sp.total_len + self.cap
        self.k = k if k is not None else torch.empty((n, sp.local_heads, cfg.head_dim), dtype=torch.bfloat16,
                                                     device=device)
        self.v = v if v is not None else torch.empty_like(self.k)
        self.peer = None        # PeerExchange of the layer (P > 1, peer mode)
        self.keep_q = False     # tests: keep the last forward's head-sharded q in .last_q
        self.last_q = None      # (and, on the peer / local exchange path, the raw keys in .last_k_raw)
        self.last_k_raw = None
        # pre-RoPE mode: normalised, unrotated keys of the cache slots (kpre) and
        # of the current chunk's image tokens (stage, refreshed every forward)
        self.pre_rope = cfg.kv_cache_pre_rope
        self.kpre = torch.empty((self.cap, sp.local_heads, cfg.head_dim), dtype=torch.bfloat16, device=device) \
            if self.pre_rope else None
        self.stage = torch.empty((cfg.img_tokens, sp.local_heads, cfg.head_dim), dtype=torch.bfloat16,
                                 device=device) if self.pre_rope else None
        self.slot_age = []      # pre-RoPE mode: ring slots, oldest first
        self.valid = 0          # cached image tokens
        self.next_slot = 0
        self.cur = sp.total_len
        self.img_len = cfg.img_tokens

    def keys(self):
        n = self.cur + self.valid
        return self.k[:n], self.v[:n]

    def commit(self, sp: SeqParallel, tables=None):
        """Store the current chunk's image-token K/V into the ring (oldest slot).
        Pre-RoPE mode: the slot gets the normalised, unrotated keys of the stage
        buffer, and every cached slot is re-rotated at its window position
        (tables(age) -> fp32 cos/sin; see assemble)."""
        base = self.cur + self.next_slot * self.img_len
        off = 0
        for start, length in sp.gathered_img_segments():
            if not self.pre_rope:
                self.k[base + off: base + off + length].copy_(self.k[start:start + length])
            self.v[base + off: base + off + length].copy_(self.v[start:start + length])
            off += length
        if self.pre_rope:
            s0 = self.next_slot * self.img_len
            self.kpre[s0:s0 + self.img_len].copy_(self.stage)
            if self.next_slot in self.slot_age:
                self.slot_age.remove(self.next_slot)
            self.slot_age.append(self.next_slot)
        self.next_slot = (self.next_slot + 1) % (self.cap // self.img_len)
        self.valid = min(self.cap, self.valid + self.img_len)
        if self.pre_rope and tables is not None:
            self.assemble(tables)

    def assemble(self, tables):
        """Pre-RoPE mode: rotate every cached slot's keys at the position it
        holds in the attention window, oldest slot at chunk position 0 (the
        shifted temporal ids of the reference's cache assembly, dit.py:189-225,
        955-973; graph_runner.py:137-142 rotates at commit the same way)."""
        for age, slot in enumerate(self.slot_age):
            c, s_ = tables(age)
            r0 = slot * self.img_len
            jo.rope_apply(self.kpre[r0:r0 + self.img_len], c, s_,
                          out=self.k[self.cur + r0: self.cur + r0 + self.img_len])

    def fill_random(self, gen, chunks: int, tables=None):
        """Pre-fill `chunks` cache slots with N(0,1) K/V; in
        pre-RoPE mode the unrotated keys, then rotated into the window."""
        n = chunks * self.img_len
        if self.pre_rope:
            self.kpre[:n].normal_(generator=gen)
            self.slot_age = list(range(chunks))
        else:
            self.k[self.cur:self.cur + n].normal_(generator=gen)
        self.v[self.cur:self.cur + n].normal_(generator=gen)
        self.valid = n
        self.next_slot = chunks % (self.cap // self.img_len)
        if self.pre_rope and tables is not None:
            self.assemble(tables)


@dataclass
class PeerExchange:
    """Per-layer view of the peer exchange: the head-sharded q buffer, the
    gathered-order segments (offset, image rows, text rows, first image token)
    of every rank, the full RoPE tables, the 3 x P destination addresses
    (q, k, v of every rank) handed to the scattering QKV projection, and the
    attention output buffers of every rank that the scattering attention
    epilogue writes."""
    region: object
    q: torch.Tensor
    seg: list
    cos: torch.Tensor
    sin: torch.Tensor
    dst: list
    o: Optional[torch.Tensor] = None     # this rank's [tokens, heads, Dh] attention output (all heads)
    odst: Optional[list] = None          # every rank's attention output buffer (device addresses)
    oseg: Optional[list] = None          # rank segment starts of the gathered order (P + 1)


class Block:
    def __init__(self, cfg: StackConfig, gen, device):
        self.cfg = cfg
        self.img = Stream(cfg, gen, device)
        self.txt = Stream(cfg, gen, device)
        self.timer = None       # a list: CUDA events at phase boundaries (bench breakdown)

    def _mark(self, name: str):
        if self.timer is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.timer.append((name, ev))

    def forward(self, img, txt, vec, cos, sin, kv: LayerKV, sp: SeqParallel):
        cfg = self.cfg
        H, Dh, D = cfg.heads, cfg.head_dim, cfg.hidden
        Li, Lt = img.shape[0], txt.shape[0]
        im = (self.img.mod + vec).unbind(0)
        tm = (self.txt.mod + vec).unbind(0)

        if kv.peer is not None:
            return self._forward_peer(img, txt, im, tm, kv, sp)
        if kv.pre_rope:
            raise NotImplementedError("the pre-RoPE KV cache needs the peer / local exchange (JOYOMNI_SP_EXCHANGE=peer)")

        # ---- QKV of both streams into one [L_local, 3, H, Dh] buffer --------
        qkv = torch.empty((Li + Lt, 3 * D), dtype=torch.bfloat16, device=img.device)
        xq, xs = norm_mod_quant(img, im[0], im[1])
        self.img.qkv(xq, xs, out=qkv[:Li])
        tq, ts = norm_mod_quant(txt, tm[0], tm[1])
        self.txt.qkv(tq, ts, out=qkv[Li:])
        v5 = qkv.view(1, Li + Lt, 3, H, Dh)
        jo.qk_norm_rope_strided(v5[:, :Li, 0], v5[:, :Li, 1], NORM_EPS, self.img.q_norm, self.img.k_norm, cos, sin)
        jo.qk_norm_rope_strided(v5[:, Li:, 0], v5[:, Li:, 1], NORM_EPS, self.txt.q_norm, self.txt.k_norm)

        # ---- attention over [current | cached] keys, head-sharded ------------
        q = v5[0, :, 0] if sp.world == 1 else sp.seq_to_heads(v5[0, :, 0])     # strided view when P = 1
        sp.seq_to_heads(v5[0, :, 1], out=kv.k[:kv.cur])
        sp.seq_to_heads(v5[0, :, 2], out=kv.v[:kv.cur])
        if kv.keep_q:
            kv.last_q = q.clone()
        k_all, v_all = kv.keys()
        o = sp.heads_to_seq(attend(q, k_all, v_all, cfg.attention)).reshape(Li + Lt, D)

        # ---- projections + FFN with gated residuals ------------------------
        img = self._tail(self.img, im, img, o[:Li])
        txt = self._tail(self.txt, tm, txt, o[Li:])
        return img, txt

    def _forward_peer(self, img, txt, im, tm, kv: "LayerKV", sp: SeqParallel):
        """The QKV projection's epilogue scatters q, k, v by head into the owning
        ranks' buffers (peer memory for P > 1; with P = 1 straight into this
        rank's q buffer and K/V cache, which saves the two copies), then every
        rank normalises / rotates its heads of all tokens, one launch per rank
        segment of the gathered token order."""
        cfg = self.cfg
        Dh, D = cfg.head_dim, cfg.hidden
        Li = img.shape[0]
        ex = kv.peer
        self._mark("start")
        xq, xs = norm_mod_quant(img, im[0], im[1])
        self.img.qkv.scatter(xq, xs, ex.dst, sp.world, sp.local_heads, Dh, ex.seg[sp.rank][0], ex.q.shape[0])
        tq, ts = norm_mod_quant(txt, tm[0], tm[1])
        self.txt.qkv.scatter(tq, ts, ex.dst, sp.world, sp.local_heads, Dh, ex.seg[sp.rank][0] + Li, ex.q.shape[0])
        self._mark("norm_quant_qkv_scatter_gemm")
        if ex.region is not None:
            ex.region.sync()
        self._mark("exchange_sync")
        q = ex.q
        if kv.keep_q:
            kv.last_k_raw = kv.k[:kv.cur].clone()
        if kv.pre_rope:
            # the normalised, unrotated keys of the image tokens (the reference's
            # rmsnorm_qk_bf16 on img_k, dit.py:360-363), for the cache commit
            for off, ni, nt, i0 in ex.seg:
                jo.rmsnorm(kv.k[off:off + ni].reshape(-1, Dh), self.img.k_norm, NORM_EPS,
                           out=kv.stage[i0:i0 + ni].view(-1, Dh))
        for off, ni, nt, i0 in ex.seg:
            jo.qk_norm_rope_strided(q[off:off + ni][None], kv.k[off:off + ni][None], NORM_EPS, self.img.q_norm,
                                    self.img.k_norm, ex.cos[i0:i0 + ni], ex.sin[i0:i0 + ni])
            if nt:
                jo.qk_norm_rope_strided(q[off + ni:off + ni + nt][None], kv.k[off + ni:off + ni + nt][None],
                                        NORM_EPS, self.txt.q_norm, self.txt.k_norm)
        if kv.keep_q:
            kv.last_q = q.clone()
        self._mark("qk_norm_rope")
        k_all, v_all = kv.keys()
        L = Li + txt.shape[0]
        if self.cfg.attention == "joyomni" and ex.o is not None:
            # The attention epilogue stores every output row into the owning
            # rank's buffer (peer memory for P > 1): the output all-to-all.
            jo.attention_scatter(q, k_all, v_all, ex.odst, ex.oseg, sp.rank * sp.local_heads, cfg.heads,
                                 ex.o.shape[0])
            self._mark("attention")
            # One sync orders both hazards of the shared buffers: every rank's
            # rows have landed before this rank's projection reads its buffer,
            # and no rank's next-layer QKV scatter overwrites the q buffer (or
            # next attention the output buffer) that a slower rank still reads.
            if ex.region is not None:
                ex.region.sync()
            o = ex.o[:L].reshape(L, D)
        else:
            o = attend(q, k_all, v_all, self.cfg.attention)
            self._mark("attention")
            # Every layer shares the one head-sharded q buffer in the peer region:
            # a faster rank's next-layer scatter may only start once this rank's
            # attention has finished reading q.  heads_to_seq is an NCCL all-to-all
            # that no rank leaves before every rank has entered it (after its
            # attention), which gives that ordering.
            o = sp.heads_to_seq(o).reshape(L, D)
        self._mark("output_exchange")
        img = self._tail(self.img, im, img, o[:Li])
        txt = self._tail(self.txt, tm, txt, o[Li:])
        self._mark("proj_ffn_gemms")
        return img, txt

    @staticmethod
    def _tail(st: Stream, m, x, attn):
        aq, as_ = quant(attn)
        x = st.proj.residual(aq, as_, x, m[2])                      # x + gate1 * proj(attn)
        hq, hs = norm_mod_quant(x, m[3], m[4])
        h = st.up(hq, hs, gelu=True)
        h2q, h2s = quant(h)
        return st.down.residual(h2q, h2s, x, m[5], out=x)            # x + gate2 * down(h), in place


class Stack:
    """cfg.layers blocks, per-layer head-sharded KV cache, chunk-causal loop."""

    def __init__(self, cfg: StackConfig, device, sp: Optional[SeqParallel] = None, layers: Optional[int] = None):
        self.cfg = cfg
        self.device = device
        self.sp = sp or SeqParallel.create(cfg.img_tokens, cfg.txt_tokens, cfg.heads)
        gen = torch.Generator(device=device).manual_seed(cfg.seed)
        n = cfg.layers if layers is None else layers
        self.blocks: List[Block] = [Block(cfg, gen, device) for _ in range(n)]
        # pre-RoPE mode: the current chunk sits at window position cache_chunks
        # (after the cached chunks, oldest at 0); cached keys are rotated at theirs
        t_cur = cfg.cache_chunks * cfg.grid[0] if cfg.kv_cache_pre_rope else 0
        cos, sin = rope_tables(cfg, device, t0=t_cur)
        self._win_tables = {}
        a, b = self.sp.img_range
        self.cos, self.sin = cos[a:b].contiguous(), sin[a:b].contiguous()
        self.region = None
        # P > 1: the QKV projections scatter into the owning ranks' buffers over
        # peer memory (JOYOMNI_SP_EXCHANGE=nccl selects the NCCL all-to-all path).
        self.kv = None
        if os.environ.get("JOYOMNI_SP_EXCHANGE", "peer") == "peer":
            self.kv = self._peer_kv_agreed(n, cos, sin, device)
        if self.kv is None:
            self.kv = [LayerKV(cfg, self.sp, device) for _ in range(n)]

    def forward(self, img, txt, vec):
        for blk, kv in zip(self.blocks, self.kv):
            img, txt = blk.forward(img, txt, vec, self.cos, self.sin, kv, self.sp)
        return img, txt

    def window_tables(self, age: int):
        """fp32 cos/sin of the image grid at window chunk position `age`."""
        if age not in self._win_tables:
            self._win_tables[age] = rope_tables(self.cfg, self.device, t0=age * self.cfg.grid[0], fp32=True)
        return self._win_tables[age]

    def commit_kv(self):
        for kv in self.kv:
            kv.commit(self.sp, self.window_tables)
        if self.region is not None and self.sp.world > 1:
            # the next chunk's scatters must not overtake a slower rank's commit copies
            self.region.sync()

    def _peer_kv_agreed(self, n: int, cos, sin, device) -> Optional[List["LayerKV"]]:
        """The peer exchange when every rank could set it up (IPC export / map),
        else None on every rank (the NCCL path): the ranks agree on the outcome
        with a MIN all-reduce, so no rank scatters into a rank that cannot."""
        try:
            kvs, err = self._peer_kv(n, cos, sin, device), None
        except Exception as e:  # noqa: BLE001
            kvs, err = None, e
        if self.sp.world > 1:
            import torch.distributed as dist
            ok = torch.tensor([1.0 if kvs is not None else 0.0], device=device)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.sp.group)
            if ok.item() < 1.0:
                self.exchange_error = repr(err)[:300] if err is not None else "a peer rank failed"
                if torch.cuda.is_available():
                    torch.cuda.synchronize()
                dist.barrier(group=self.sp.group)      # every rank, including the failed one
                if self.region is not None:
                    self.region.close(barrier=False)
                self.region = None
                return None
        elif kvs is None:
            raise err
        return kvs

    def _peer_kv(self, n: int, cos, sin, device) -> List["LayerKV"]:
        from .peer import LocalRegion, PeerRegion, RegionLayout
        cfg, sp = self.cfg, self.sp
        hpr, Dh = sp.local_heads, cfg.head_dim
        rows = sp.total_len + cfg.cache_chunks * cfg.img_tokens
        lay = RegionLayout()
        lay.add("q", (sp.total_len, hpr, Dh))
        # attention output of this rank's tokens, all heads (identical size on
        # every rank: the largest shard)
        ocap = max(sp.shard_len(r) for r in range(sp.world))
        lay.add("o", (ocap, cfg.heads, Dh))
        for i in range(n):
            lay.add(f"k{i}", (rows, hpr, Dh))
            lay.add(f"v{i}", (rows, hpr, Dh))
        # P = 1: the same layout in one local allocation, no peers to map
        self.region = PeerRegion(lay, sp.group, sp.world, sp.rank, device) if sp.world > 1 else \
            LocalRegion(lay, device)
        isz, tsz = split_sizes(cfg.img_tokens, sp.world), split_sizes(cfg.txt_tokens, sp.world)
        seg, off = [], 0
        for r in range(sp.world):
            seg.append((off, isz[r], tsz[r], shard_range(cfg.img_tokens, sp.world, r)[0]))
            off += isz[r] + tsz[r]
        q = self.region.tensor("q")
        # JOYOMNI_ATTN_SCATTER=0 keeps the NCCL all-to-all after attention (comparison)
        scatter_out = os.environ.get("JOYOMNI_ATTN_SCATTER", "1") != "0"
        o = self.region.tensor("o") if scatter_out else None
        odst = [self.region.ptr(r, "o") for r in range(sp.world)] if scatter_out else None
        oseg = sp.gathered_segment_starts()
        assert oseg[:-1] == [s[0] for s in seg]
        kvs = []
        for i in range(n):
            kv = LayerKV(cfg, sp, device, k=self.region.tensor(f"k{i}"), v=self.region.tensor(f"v{i}"))
            kv.peer = PeerExchange(self.region if sp.world > 1 else None, q, seg, cos, sin,
                                   [self.region.ptr(r, name) for name in ("q", f"k{i}", f"v{i}")
                                    for r in range(sp.world)], o, odst, oseg)
            kvs.append(kv)
        return kvs

    def close(self):
        """Unmap the peer regions (collective over the Ulysses group)."""
        if self.region is not None:
            self.region.close()

    def inputs(self, seed: int):
        """This rank's shard of a chunk's synthetic inputs (identical global
        tensors on every rank): image latents in token space (fp32), text tokens
        and the timestep embedding, all N(0, 1)."""
        cfg = self.cfg
        g = torch.Generator(device="cpu").manual_seed(seed)
        img = torch.randn((cfg.img_tokens, cfg.hidden), generator=g)
        txt = torch.randn((cfg.txt_tokens, cfg.hidden), generator=g)
        a, b = self.sp.img_range
        c, d = self.sp.txt_range
        return (img[a:b].to(self.device), txt[c:d].to(torch.bfloat16).to(self.device))

    def timestep_vec(self, t: float):
        g = torch.Generator(device="cpu").manual_seed(int(t) * 7919 + 1)
        return torch.randn(self.cfg.hidden, generator=g).to(torch.bfloat16).to(self.device)

    # ---- whole-step CUDA graph ---------------------------------------------
    def capture(self, txt: torch.Tensor) -> bool:
        """Capture one 40-layer forward (all joyomni_ops kernels, attention and, with
        P > 1, the NCCL all-to-alls) into a CUDA graph over static input buffers
        (the reference captures its denoise steps the same way,
        deploy/xvideo/serving/graph_runner.py:97-183).  Every kernel here launches on
        the current stream and allocates nothing itself, so the step is
        capturable; returns False (eager execution stays in use) if capture fails."""
        D = self.cfg.hidden
        a, b = self.sp.img_range
        dev = self.device
        self._gx = torch.zeros((b - a, D), dtype=torch.bfloat16, device=dev)
        self._gtxt = txt.clone()
        self._gvec = torch.zeros(D, dtype=torch.bfloat16, device=dev)
        saved = [(kv.valid, kv.next_slot) for kv in self.kv]
        try:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self.forward(self._gx, self._gtxt, self._gvec)
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._gout, _ = self.forward(self._gx, self._gtxt, self._gvec)
            self._graph = g
            ok = True
        except Exception as e:  # noqa: BLE001
            self._graph = None
            self.capture_error = repr(e)[:300]
            ok = False
        for kv, (v, n) in zip(self.kv, saved):
            kv.valid, kv.next_slot = v, n
        return ok

    def _step(self, xb: torch.Tensor, txt: torch.Tensor, vec: torch.Tensor):
        g = getattr(self, "_graph", None)
        if g is None:
            return self.forward(xb, txt, vec)[0]
        self._gx.copy_(xb)
        self._gvec.copy_(vec)
        if txt.data_ptr() != self._gtxt.data_ptr():
            self._gtxt.copy_(txt)
        g.replay()
        return self._gout

    def denoise_chunk(self, x: torch.Tensor, txt: torch.Tensor, timesteps=(1000, 750, 500),
                      store_pass: bool = False):
        """3 denoising steps (Euler in fp32 over sigmas t/1000 -> next, last -> 0);
        the chunk's image K/V from the last step enter the cache afterwards.  Uses
        the captured step graph when capture() succeeded.

        store_pass=True adds the reference's extra forward on the clean latent at
        timestep 0 whose K/V are the ones cached (pipeline.py:411-448,
        graph_runner.py:156-163).  The reference skips the text stream in that
        pass (skip_text_stream=True, pipeline.py:447); here it runs the same full
        step (graph), so its cost is an upper bound by the text tokens' share."""
        sig = [t / 1000.0 for t in timesteps] + [0.0]
        for i, t in enumerate(timesteps):
            v = self._step(x.to(torch.bfloat16), txt, self.timestep_vec(t))
            x = x + (sig[i + 1] - sig[i]) * v.float()
        if store_pass:
            self._step(x.to(torch.bfloat16), txt, self.timestep_vec(0))
        self.commit_kv()
        jo.check_gemm_fault(self.device)     # a GEMM that gave up on a wait returned partial output
        return x
