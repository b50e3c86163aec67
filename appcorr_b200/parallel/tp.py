"""Tensor-parallel ViT engine (Megatron split, one process per GPU, peer-memory collectives).

Weights: qkv and fc1 / w1||w2 are split by output (heads / hidden units), proj and fc2 / w3 by
input, so each rank computes its heads' attention and its slice of the MLP for every token and
produces a partial product of proj and of fc2. The residual stream, the per-layer increment
cache and the correction plan are replicated; the K/V cache is split by head (no K/V traffic).

Per layer (approximate pass):
    LN1 -> qkv (local heads) -> CLS score (local heads) -> attention (local heads)
        -> proj partial -> barrier -> all-reduce + residual/LayerScale epilogue -> barrier
        -> LN2 -> fc1 slice -> fc2 partial -> barrier -> all-reduce + epilogue -> barrier
The all-reduce is csrc/comm.cu `tp_allreduce_epi`: each rank reduces its own row block from every
peer's partial over NVLink and writes the finished rows into every replica, so the block's
residual add, LayerScale and increment bookkeeping ride on the collective. The correction pass
is the same on the packed selected rows; the final epilogue scatters them into every replica.
Reference: none (the reference is single-GPU); semantics are those of models/engine.py.
"""
from __future__ import annotations

from dataclasses import replace
from typing import Dict, Optional

import torch

from ..common.protocol import LAYERMEAN_SERVER_PSCORES
from ..models.dinov3.vit import ViTConfig
from ..models.engine import BF16, EngineWeights, LayerW, Session, ViTEngine, random_weights
from ..models.weights import SWIGLU_BLOCK, pack_swiglu, unpack_swiglu
from ..ops import kernels as K
from .comm import TPComm


def shard_layer(cfg: ViTConfig, lw: LayerW, rank: int, world: int) -> LayerW:
    D, Hd = cfg.embed_dim, cfg.ffn_hidden
    if cfg.num_heads % world or Hd % world:
        raise ValueError(f"heads ({cfg.num_heads}) and hidden ({Hd}) must divide the TP degree {world}")
    d = D // world
    sl = slice(rank * d, (rank + 1) * d)
    qkv = lw.qkv_w.view(3, D, D)[:, sl].reshape(3 * d, D).contiguous()
    qkv_b = lw.qkv_b.view(3, D)[:, sl].reshape(3 * d).contiguous() if lw.qkv_b is not None else None
    h = Hd // world
    hs = slice(rank * h, (rank + 1) * h)
    if cfg.is_swiglu:
        if h % SWIGLU_BLOCK:
            raise ValueError(f"SwiGLU hidden slice {h} must be a multiple of {SWIGLU_BLOCK}")
        w1, w2 = unpack_swiglu(lw.fc1_w)
        b1 = b2 = None
        if lw.fc1_b is not None:
            bb = lw.fc1_b.view(-1, 2, SWIGLU_BLOCK)
            b1, b2 = bb[:, 0].reshape(-1), bb[:, 1].reshape(-1)
        fc1_w, fc1_b = pack_swiglu(w1[hs].contiguous(), w2[hs].contiguous(),
                                   b1[hs].contiguous() if b1 is not None else None,
                                   b2[hs].contiguous() if b2 is not None else None)
    else:
        fc1_w = lw.fc1_w[hs].contiguous()
        fc1_b = lw.fc1_b[hs].contiguous() if lw.fc1_b is not None else None
    return replace(lw, qkv_w=qkv, qkv_b=qkv_b, proj_w=lw.proj_w[:, sl].contiguous(), fc1_w=fc1_w, fc1_b=fc1_b,
                   fc2_w=lw.fc2_w[:, hs].contiguous())


def shard_weights(w: EngineWeights, rank: int, world: int) -> EngineWeights:
    return replace(w, layers=[shard_layer(w.cfg, lw, rank, world) for lw in w.layers])


class ViTEngineTP(ViTEngine):
    """ViTEngine whose layers run split over `comm.world` GPUs. Construct from full weights
    (`from_full`) or generate random shards directly (`random`)."""

    def __init__(self, weights: EngineWeights, comm: TPComm, device=None, precision="bf16"):
        super().__init__(weights, device, precision)
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.local_heads = self.cfg.num_heads // self.world
        self.local_dim = self.cfg.embed_dim // self.world

    @classmethod
    def from_full(cls, full: EngineWeights, comm: TPComm, precision="bf16") -> "ViTEngineTP":
        return cls(shard_weights(full, comm.rank, comm.world), comm, comm.device, precision)

    @classmethod
    def random_tp(cls, cfg: ViTConfig, comm: TPComm, seed: int = 0, precision="bf16") -> "ViTEngineTP":
        full = random_weights(cfg, comm.device, seed)  # identical on every rank (same seed)
        w = shard_weights(full, comm.rank, comm.world)
        del full
        torch.cuda.empty_cache()
        return cls(w, comm, comm.device, precision)

    # -------------------------------------------------------------- sessions
    def new_session(self, B: int, H: int, W: int) -> Session:
        c, comm = self.cfg, self.comm
        sess = super().new_session(B, H, W)
        M, D, L = B * sess.N, c.embed_dim, c.depth
        d, hd = self.local_dim, c.ffn_hidden // self.world
        dev = self.device
        # replicated state that peers write into
        x = comm.empty((M, D), BF16)
        bos = comm.empty((L, M, D), BF16)
        x_att = comm.empty((B * (c.n_prefix + sess.P), D), BF16)
        part = comm.empty((M, D), BF16)
        ps_local = comm.empty((B, sess.N), torch.float32)
        sess.extra.update({"sym_x": x, "sym_bos": bos, "sym_x_att": x_att, "sym_part": part, "sym_ps": ps_local})
        sess.x, sess.bos, sess.x_att = x.local, bos.local, x_att.local
        # head-split buffers
        sess.q = torch.empty(M, d, device=dev, dtype=BF16)
        sess.o = torch.empty(M, d, device=dev, dtype=BF16)
        sess.kc = torch.empty(L, M, d, device=dev, dtype=BF16)
        sess.vc = torch.empty(L, M, d, device=dev, dtype=BF16)
        sess.h = torch.empty(M, hd, device=dev, dtype=BF16)
        sess.ps_scratch = torch.empty(B, self.local_heads, sess.N, device=dev, dtype=torch.float32)
        return sess

    # -------------------------------------------------------------- helpers
    def _reduce(self, sess: Session, M: int, **kw) -> None:
        comm = self.comm
        comm.barrier()
        comm.allreduce_epilogue(sess.extra["sym_part"], M=M, N=self.cfg.embed_dim, **kw)
        comm.barrier()

    # -------------------------------------------------------------- approximate pass
    def approx_layer(self, sess: Session, l: int, x: torch.Tensor, x_out: torch.Tensor, server_pscore: str) -> None:
        c, lw = self.cfg, self.w.layers[l]
        B, N, Dh = sess.B, sess.N, c.head_dim
        M = B * N
        sym = sess.extra
        part = sym["sym_part"].local
        a, sa = self._norm(sess, x, lw.norm1_w, lw.norm1_b, sess.xn)
        w, ws = self._w(lw, "qkv")
        K.qkv_gemm(a, w, lw.qkv_b, sess.q, sess.kc[l], sess.vc[l], head_dim=Dh, seq_len=N,
                   rope=sess.rope, n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        score = server_pscore not in ("none", "disabled")
        self._attention_with_score(sess, l, self.local_heads, score, sym["sym_ps"].local)
        a, sa = self._act(sess, sess.o)
        w, ws = self._w(lw, "proj")
        K.gemm(a, w, part, a_scale=sa, b_scale=ws)
        bos = sym["sym_bos"]
        off = l * M * c.embed_dim
        self._reduce(sess, M, out=sym["sym_x"], aux=bos, aux_offset=off, aux_mode=K.AUX_SET, bias=lw.proj_b,
                     gamma=lw.ls1, resid=x)
        if score:  # every rank's local-head mean is ready (barrier above): average them
            self.comm.mean_f32(sym["sym_ps"], sess.pscore[l])
        a, sa = self._norm(sess, x, lw.norm2_w, lw.norm2_b, sess.xn)
        self._mlp(lw, a, sess.h, sa)
        a, sa = self._act(sess, sess.h)
        w, ws = self._w(lw, "fc2")
        K.gemm(a, w, part, a_scale=sa, b_scale=ws)
        self._reduce(sess, M, out=sym["sym_x"], aux=bos, aux_offset=off, aux_mode=K.AUX_ADD, bias=lw.fc2_b,
                     gamma=lw.ls2, resid=x)

    def approx(self, sess: Session, start: int, end: int, server_pscore: str = "cls_attn_prob") -> torch.Tensor:
        if start == 0:
            sess.x.copy_(sess.x_in)
        self._set_pass(sess, "approx")
        for l in range(start, end):
            self.approx_layer(sess, l, sess.x, sess.x, server_pscore)
        sess.approx_done = max(sess.approx_done, end)
        return sess.x

    # -------------------------------------------------------------- correction pass
    def correct_layer(self, sess: Session, l: int, x: torch.Tensor, upd: torch.Tensor, rows: torch.Tensor) -> None:
        c, lw = self.cfg, self.w.layers[l]
        B, N, Dh = sess.B, sess.N, c.head_dim
        T = upd.shape[1]
        MT = B * T
        sym = sess.extra
        part = sym["sym_part"].local[:MT]
        x_act, x_att = sess.x_act[:MT], sess.x_att[:MT]
        xn, q, o, h = sess.xn[:MT], sess.q[:MT], sess.o[:MT], sess.h[:MT]
        a, sa = self._norm(sess, x, lw.norm1_w, lw.norm1_b, xn, rows=rows, copy_out=x_act)
        K.add_(x, sess.bos[l])
        w, ws = self._w(lw, "qkv")
        K.qkv_gemm(a, w, lw.qkv_b, q, sess.kc[l], sess.vc[l], head_dim=Dh, tok_idx=upd.view(-1),
                   kv_rows=rows, rope=sess.rope, n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        K.attention(q, sess.kc[l], sess.vc[l], o, B=B, Tq=T, Tk=N, H=self.local_heads, Dh=Dh)
        a, sa = self._act(sess, o)
        w, ws = self._w(lw, "proj")
        K.gemm(a, w, part, a_scale=sa, b_scale=ws)
        self._reduce(sess, MT, out=sym["sym_x_att"], bias=lw.proj_b, gamma=lw.ls1, resid=x_act)
        a, sa = self._norm(sess, x_att, lw.norm2_w, lw.norm2_b, xn)
        self._mlp(lw, a, h, sa)
        a, sa = self._act(sess, h)
        w, ws = self._w(lw, "fc2")
        K.gemm(a, w, part, a_scale=sa, b_scale=ws)
        self._reduce(sess, MT, out=sym["sym_x"], out_rows=rows, aux=sym["sym_bos"],
                     aux_offset=l * B * N * c.embed_dim, aux_mode=K.AUX_OUT_MINUS, bias=lw.fc2_b, gamma=lw.ls2,
                     resid=x_att, resid2=x_act)
