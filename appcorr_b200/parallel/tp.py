"""Tensor-parallel ViT engine, sequence-parallel layout (one process per GPU, collectives fused
into the kernels that produce and consume them, over NVLink / NVSwitch peer memory).

Weights: qkv and fc1 / w1||w2 are split by output (heads / hidden units), proj and fc2 / w3 by
input. The residual stream and the per-layer increment cache are split by ROWS: rank r owns token
rows [r*R, (r+1)*R), R = ceil(M / T). The K/V cache is split by head (no K/V traffic).

Per layer (approximate pass):
    [gather buffer xg holds LN1(x) of every row, e4m3 + row scales (or bf16)]
    qkv GEMM (local heads) -> CLS score + attention (local heads) -> proj GEMM (partial product)
    -> barrier -> owner row kernel: sum of the T partials (the reduce-scatter: peer loads of
    each rank's partial rows, or with APPCORR_TP_RS=push local loads of rows that the GEMM
    epilogue already stored into the owner's slots over NVLink) + bias, LayerScale, residual,
    increment := delta, then LN2 of the finished row quantised and stored into every rank's xg
    (fused all-gather) -> barrier -> w1||w2 GEMM (local hidden) -> fc2 GEMM (partial)
    -> barrier -> owner row kernel (reduce-scatter, residual, increment += delta, LN1 of
    the next layer + all-gather) -> barrier
Bytes per layer and rank: (T-1)/T * M * D * (2 + 2) for the two reduce-scatters (bf16 partials)
plus (T-1)/T * M * D * (1 + 1) for the two all-gathers (e4m3 rows), against 8 * (T-1)/T * M * D
for two bf16 all-reduces of a replicated stream.
The correction pass is the same on the packed selected rows: the owner of a selected token runs
its LN (gather), the partial rows of the packed GEMM outputs are routed to the owners of their
tokens, and the increments are updated on the owners.
Reference: none (the reference is single-GPU); semantics are those of models/engine.py.
"""
from __future__ import annotations

import os
from dataclasses import replace
from typing import Dict, Optional

import torch

from ..models.dinov3.vit import ViTConfig
from ..models.engine import BF16, EngineWeights, LayerW, Session, ViTEngine, _score_kind, random_weights
from ..models.weights import SWIGLU_BLOCK, pack_swiglu, unpack_swiglu
from ..ops import kernels as K
from ..utils.tracing import PhaseTimer
from .comm import SymTensor, TPComm


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
    (`from_full`) or generate random shards directly (`random_tp`)."""

    def __init__(self, weights: EngineWeights, comm: TPComm, device=None, precision="bf16"):
        super().__init__(weights, device, precision)
        if self.cfg.padded_head_dim:
            raise ValueError("tensor parallelism does not support padded attention heads")
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.local_heads = self.cfg.num_heads // self.world
        self.local_dim = self.cfg.embed_dim // self.world
        self.timer = PhaseTimer.from_env()
        # micro-batches per session: each runs on its own stream with its own barriers, so one
        # micro-batch's collectives overlap the other's GEMMs
        self.microbatch = max(1, int(os.environ.get("APPCORR_TP_MICROBATCH", "2")))
        self._streams = []
        # reduce-scatter of the row-parallel GEMMs: "pull" (owner loads peers' partials in the row
        # kernel) or "push" (GEMM epilogue stores partial rows into the owner's slots)
        # "ce": contiguous row blocks (approximate pass) travel by copy-engine peer copies into the
        # owners' slots, packed correction rows are pulled
        # "pushk": the GEMM writes locally, then a row kernel pushes every row owned by a peer
        # into the owner's slot with coalesced peer stores; owners reduce from local memory
        self.ag_push = os.environ.get("APPCORR_TP_AG", "push") == "push"
        self.rs_mode = os.environ.get("APPCORR_TP_RS", "pull")
        if self.rs_mode not in ("pull", "push", "ce", "pushk"):
            raise ValueError("APPCORR_TP_RS must be 'pull', 'push', 'pushk' or 'ce'")

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
        k = self.microbatch
        if k > 1 and B % k == 0 and self.world > 1:
            return self._new_split_session(B, H, W, k)
        return self._new_sub_session(B, H, W)

    def _new_split_session(self, B: int, H: int, W: int, k: int) -> Session:
        """A session of B images served as k micro-batches of B/k images (sub-sessions)."""
        c, comm = self.cfg, self.comm
        Bh = B // k
        D = c.embed_dim
        subs = []
        feat = comm.empty((B * ((H // c.patch_size) * (W // c.patch_size)), D), BF16)
        for i in range(k):
            subs.append(self._new_sub_session(Bh, H, W))
        s0 = subs[0]
        N, P = s0.N, s0.P
        M = B * N
        dev = self.device
        parent = Session(
            B=B, img_hw=(H, W), grid_hw=s0.grid_hw, N=N, P=P,
            x_in=torch.empty(M, D, device=dev, dtype=BF16), x=s0.x, x_tmp=s0.x_tmp, xn=s0.xn, q=s0.q, o=s0.o,
            h=s0.h, kc=s0.kc, vc=s0.vc, bos=s0.bos, pscore=torch.zeros(c.depth, B, N, device=dev),
            ps_scratch=s0.ps_scratch, cols=torch.zeros(B * P, self.w.patch_w.shape[1], device=dev, dtype=BF16),
            patch_rows=(torch.arange(B, device=dev)[:, None] * N + c.n_prefix
                        + torch.arange(P, device=dev)[None, :]).reshape(-1).to(torch.int32).contiguous(),
            rope=s0.rope, upd=s0.upd, rows=s0.rows, x_act=s0.x_act, x_att=s0.x_att, plan_stats=s0.plan_stats,
            stat_acc=s0.stat_acc)
        Mh = Bh * N
        for i, sub in enumerate(subs):
            sub.x_in = parent.x_in[i * Mh:(i + 1) * Mh]
            sub.pscore = parent.pscore[:, i * Bh:(i + 1) * Bh]
            off = i * Bh * P
            sub.extra["sym_feat"] = SymTensor(feat.local[off:off + Bh * P], feat.view_ptrs(off * D))
        parent.extra["subs"] = subs
        parent.extra["feat"] = feat
        return parent

    def _new_sub_session(self, B: int, H: int, W: int) -> Session:
        c, comm = self.cfg, self.comm
        sess = super().new_session(B, H, W)
        M, D, L = B * sess.N, c.embed_dim, c.depth
        d, hd = self.local_dim, c.ffn_hidden // self.world
        dev = self.device
        R = (M + self.world - 1) // self.world
        # symmetric buffers that peers store into
        xg = comm.empty((M, D), BF16)                       # gathered LN rows (bf16, or e4m3 in its first M*D bytes)
        xg8 = SymTensor(xg.local.view(torch.uint8).view(-1)[: M * D].view(M, D).view(torch.float8_e4m3fn), xg.ptrs)
        # NVFP4 gather: packed e2m1 rows in the first M*D/2 bytes, blocked block scales alongside
        xg4 = SymTensor(xg.local.view(torch.uint8).view(-1)[: M * D // 2].view(M, D // 2), xg.ptrs)
        if "nvfp4" in self.precision.values():
            sess.extra["sym_xg_sf"] = comm.empty((K.nvfp4_sf_bytes(M, D),), torch.uint8)
        sess.extra.update({
            "R": R, "chan": comm.channel(), "sym_xg": xg, "sym_xg8": xg8, "sym_xg4": xg4,
            "sym_xg_scale": comm.empty((M,), torch.float32),
            "sym_part": (comm.empty((self.world, M, D), BF16) if self.rs_mode in ("push", "pushk")
                         else comm.empty((M, D), BF16)),
            "sym_slot": comm.empty((self.world, M, D), BF16) if self.rs_mode == "ce" else None,
            "sym_ps": comm.empty((B, sess.N), torch.float32),
            "sym_feat": comm.empty((B * sess.P, D), BF16)})
        # head-split buffers
        sess.q = torch.empty(M, d, device=dev, dtype=BF16)
        sess.o = torch.empty(M, d, device=dev, dtype=BF16)
        sess.kc = torch.empty(L, M, d, device=dev, dtype=BF16)
        sess.vc = torch.empty(L, M, d, device=dev, dtype=BF16)
        sess.h = torch.empty(M, hd, device=dev, dtype=BF16)
        sess.ps_scratch = torch.empty(B, self.local_heads, sess.N, device=dev, dtype=torch.float32)
        return sess

    # -------------------------------------------------------------- helpers
    def _gathered(self, sess: Session, n: int):
        """The all-gathered GEMM operand rows [:n] (and their e4m3 scales)."""
        e = sess.extra
        if self._fp4:
            return e["sym_xg4"].local[:n], (e["sym_xg_scale"].local[:n], e["sym_xg_sf"].local)
        if self._fp8:
            return e["sym_xg8"].local[:n], e["sym_xg_scale"].local[:n]
        return e["sym_xg"].local[:n], None

    def _ag(self, sess: Session) -> Dict:
        e = sess.extra
        push = self.ag_push  # contiguous rows: local gather stores + one bulk peer push
        if self._fp4:
            return {"ag": e["sym_xg4"], "ag_scale": e["sym_xg_scale"], "ag_sf": e["sym_xg_sf"], "ag_push": push}
        if self._fp8:
            return {"ag": e["sym_xg8"], "ag_scale": e["sym_xg_scale"], "ag_push": push}
        return {"ag": e["sym_xg"], "ag_push": push}

    def _row_gemm(self, sess: Session, a, w, rows_out, a_scale, b_scale, n: int) -> None:
        """Row-parallel GEMM producing this rank's partial product of n (packed) rows."""
        e = sess.extra
        if self.rs_mode == "push":  # partial rows stored into their owners' slots by the epilogue
            K.gemm(a, w, None, out_rows=rows_out, a_scale=a_scale, b_scale=b_scale,
                   rs=(e["sym_part"].ptrs, e["R"], self.rank, n, self.cfg.embed_dim))
        elif self.rs_mode == "pushk":  # local GEMM into my slot, then a push of the peers' rows
            D = self.cfg.embed_dim
            part = e["sym_part"]
            mine = part.local.view(-1)[self.rank * n * D:(self.rank + 1) * n * D].view(n, D)
            K.gemm(a, w, mine, a_scale=a_scale, b_scale=b_scale)
            self.comm.push_rows(part.view_ptrs(self.rank * n * D)[self.rank], part.view_ptrs(self.rank * n * D),
                                rows_out, n, D, e["R"])
        else:
            K.gemm(a, w, e["sym_part"].local[:n], a_scale=a_scale, b_scale=b_scale)

    def _ce_scatter(self, sess: Session, n: int) -> None:
        """Copy-engine reduce-scatter of a contiguous partial product: row block p (owned by rank
        p) goes to slot [my rank] of rank p with one peer cudaMemcpyAsync per peer."""
        e = sess.extra
        views = e.get("slot_views")
        if views is None:
            from ..ops.native import lib

            slot = e["sym_slot"]
            views = e["slot_views"] = [lib().tensor_from_ptr(p, [self.world * n, self.cfg.embed_dim], BF16,
                                                             self.device.index) for p in slot.ptrs]
        R, part = e["R"], e["sym_part"].local
        for p in range(self.world):
            if p == self.rank:
                continue
            lo, hi = p * R, min((p + 1) * R, n)
            if hi > lo:
                views[p][self.rank * n + lo:self.rank * n + hi].copy_(part[lo:hi], non_blocking=True)

    def _src(self, sess: Session, n: int, contiguous: bool = False) -> tuple:
        """Where the owner finds row i of every rank's partial product (pointers, row offsets)."""
        e = sess.extra
        part = e["sym_part"]
        if self.rs_mode in ("push", "pushk"):
            return [part.ptrs[self.rank]] * self.world, [s * n for s in range(self.world)]
        if self.rs_mode == "ce" and contiguous:
            ptrs = [e["sym_slot"].ptrs[self.rank]] * self.world
            ptrs[self.rank] = part.ptrs[self.rank]
            return ptrs, [s * n if s != self.rank else 0 for s in range(self.world)]
        return part.ptrs, [0] * self.world

    # -------------------------------------------------------------- approximate pass
    def approx_layer(self, sess: Session, l: int, x: torch.Tensor, x_out: torch.Tensor, server_pscore: str) -> None:
        c, lw, comm = self.cfg, self.w.layers[l], self.comm
        B, N, Dh, D = sess.B, sess.N, c.head_dim, c.embed_dim
        M = B * N
        e = sess.extra
        R = e["R"]
        tm = self.timer
        a, sa = self._gathered(sess, M)
        w, ws = self._w(lw, "qkv")
        with tm("a.qkv"):
            K.qkv_gemm(a, w, lw.qkv_b, sess.q, sess.kc[l], sess.vc[l], head_dim=Dh, seq_len=N,
                       rope=sess.rope, n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        score = _score_kind(server_pscore) != "none"
        with tm("a.attn"):
            self._attention_with_score(sess, l, self.local_heads, server_pscore, e["sym_ps"].local)
        with tm("a.quant"):
            a, sa = self._act(sess, sess.o, "proj")
        w, ws = self._w(lw, "proj")
        with tm("a.proj"):
            self._row_gemm(sess, a, w, None, sa, ws, M)
        if self.rs_mode == "ce":
            with tm("a.rs_copy"):
                self._ce_scatter(sess, M)
        with tm("a.barrier"):
            comm.barrier(e["chan"])
        if score:  # every rank's local-head mean is ready (barrier above): average them
            comm.mean_f32(e["sym_ps"], sess.pscore[l])
        with tm("a.row_ln_ag"):
            comm.sp_row(M, D, R, src=self._src(sess, M, contiguous=True), bias=lw.proj_b, gamma=lw.ls1, resid=x, out=x,
                        aux=sess.bos[l], aux_mode=K.AUX_SET, ln_w=lw.norm2_w, ln_b=lw.norm2_b, eps=c.norm_eps,
                        **self._ag(sess))
        with tm("a.barrier"):
            comm.barrier(e["chan"])
        a, sa = self._gathered(sess, M)
        with tm("a.w12"):
            self._mlp(lw, a, sess.h, sa)
        with tm("a.quant"):
            a, sa = self._act(sess, sess.h)
        w, ws = self._w(lw, "fc2")
        with tm("a.fc2"):
            self._row_gemm(sess, a, w, None, sa, ws, M)
        if self.rs_mode == "ce":
            with tm("a.rs_copy"):
                self._ce_scatter(sess, M)
        with tm("a.barrier"):
            comm.barrier(e["chan"])
        nxt = self.w.layers[l + 1] if l + 1 < sess.extra.get("approx_end", c.depth) else None
        with tm("a.row_ln_ag"):
            comm.sp_row(M, D, R, src=self._src(sess, M, contiguous=True), bias=lw.fc2_b, gamma=lw.ls2, resid=x, out=x,
                        aux=sess.bos[l], aux_mode=K.AUX_ADD,
                        ln_w=nxt.norm1_w if nxt is not None else None, ln_b=nxt.norm1_b if nxt is not None else None,
                        eps=c.norm_eps, **self._ag(sess))
        if nxt is not None:
            with tm("a.barrier"):
                comm.barrier(e["chan"])

    def _fork(self, k: int):
        cur = torch.cuda.current_stream(self.device)
        while len(self._streams) < k:
            self._streams.append(torch.cuda.Stream(self.device))
        for st in self._streams[:k]:
            st.wait_stream(cur)
        return self._streams[:k]

    def _join(self, streams) -> None:
        cur = torch.cuda.current_stream(self.device)
        for st in streams:
            cur.wait_stream(st)

    def _approx_begin(self, sess: Session, start: int, end: int) -> None:
        c = self.cfg
        if start == 0:
            sess.x.copy_(sess.x_in)
            sess.extra.pop("layermean", None)
            sess.extra.pop("random_score", None)
        self._set_pass(sess, "approx")
        sess.extra["approx_end"] = end
        if start < end:
            lw = self.w.layers[start]
            self.comm.sp_row(sess.B * sess.N, c.embed_dim, sess.extra["R"], x=sess.x, ln_w=lw.norm1_w,
                             ln_b=lw.norm1_b, eps=c.norm_eps, **self._ag(sess))
            self.comm.barrier(sess.extra["chan"])

    def approx(self, sess: Session, start: int, end: int, server_pscore: str = "cls_attn_prob") -> torch.Tensor:
        subs = sess.extra.get("subs")
        if subs is None:
            self._approx_begin(sess, start, end)
            for l in range(start, end):
                self.approx_layer(sess, l, sess.x, sess.x, server_pscore)
        else:  # micro-batches interleaved layer by layer on their own streams
            if start == 0:
                sess.extra.pop("layermean", None)
                sess.extra.pop("random_score", None)
            streams = self._fork(len(subs))
            for sub, st in zip(subs, streams):
                with torch.cuda.stream(st):
                    self._approx_begin(sub, start, end)
            for l in range(start, end):
                for sub, st in zip(subs, streams):
                    with torch.cuda.stream(st):
                        self.approx_layer(sub, l, sub.x, sub.x, server_pscore)
            self._join(streams)
            for sub in subs:
                sub.approx_done = max(sub.approx_done, end)
        sess.approx_done = max(sess.approx_done, end)
        return sess.x

    def correct(self, sess: Session, start: int, end: int, pre: torch.Tensor, cand: torch.Tensor, opts: Dict,
                mobile: Optional[torch.Tensor] = None, valid: Optional[torch.Tensor] = None) -> torch.Tensor:
        if opts.get("token_prune_enabled"):
            # the prune scores read every token row of the running features, which are split by
            # rows across the ranks here
            raise NotImplementedError("token_prune_enabled is supported by the one-GPU engine only")
        subs = sess.extra.get("subs")
        if subs is None:
            return super().correct(sess, start, end, pre, cand, opts, mobile=mobile, valid=valid)
        Bh = sess.B // len(subs)

        def part(t, i):
            return None if t is None else t[i * Bh:(i + 1) * Bh]

        streams = self._fork(len(subs))
        states = []
        for i, (sub, st) in enumerate(zip(subs, streams)):
            with torch.cuda.stream(st):
                states.append(self._correct_begin(sub, start, part(cand, i), opts, part(pre, i)))
        for l in range(start, end):
            for i, (sub, st) in enumerate(zip(subs, streams)):
                with torch.cuda.stream(st):
                    self._correct_step(sub, l, states[i], part(pre, i), part(cand, i), opts, part(mobile, i),
                                       part(valid, i))
        self._join(streams)
        return sess.x

    # -------------------------------------------------------------- correction pass
    def correct_layer(self, sess: Session, l: int, x: torch.Tensor, upd: torch.Tensor, rows: torch.Tensor) -> None:
        c, lw, comm = self.cfg, self.w.layers[l], self.comm
        B, N, Dh, D = sess.B, sess.N, c.head_dim, c.embed_dim
        T = upd.shape[1]
        MT = B * T
        e = sess.extra
        R = e["R"]
        x_act, x_att = sess.x_act[:MT], sess.x_att[:MT]
        q, o, h = sess.q[:MT], sess.o[:MT], sess.h[:MT]
        # LN1 of the kept rows on their owners (raw rows kept as x_act), gathered everywhere
        comm.sp_row(MT, D, R, tok=rows, x=x, copy_out=x_act, ln_w=lw.norm1_w, ln_b=lw.norm1_b, eps=c.norm_eps,
                    **self._ag(sess))
        lo, hi = self.rank * R, min((self.rank + 1) * R, B * N)
        K.add_(x[lo:hi], sess.bos[l][lo:hi])
        comm.barrier(e["chan"])
        a, sa = self._gathered(sess, MT)
        w, ws = self._w(lw, "qkv")
        K.qkv_gemm(a, w, lw.qkv_b, q, sess.kc[l], sess.vc[l], head_dim=Dh, tok_idx=upd.view(-1),
                   kv_rows=rows, rope=sess.rope, n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        K.attention(q, sess.kc[l], sess.vc[l], o, B=B, Tq=T, Tk=N, H=self.local_heads, Dh=Dh)
        a, sa = self._act(sess, o, "proj")
        w, ws = self._w(lw, "proj")
        self._row_gemm(sess, a, w, rows, sa, ws, MT)
        comm.barrier(e["chan"])
        comm.sp_row(MT, D, R, tok=rows, src=self._src(sess, MT), bias=lw.proj_b, gamma=lw.ls1, resid=x_act,
                    resid_tok=False, out=x_att, out_tok=False, ln_w=lw.norm2_w, ln_b=lw.norm2_b, eps=c.norm_eps,
                    **self._ag(sess))
        comm.barrier(e["chan"])
        a, sa = self._gathered(sess, MT)
        self._mlp(lw, a, h, sa)
        a, sa = self._act(sess, h)
        w, ws = self._w(lw, "fc2")
        self._row_gemm(sess, a, w, rows, sa, ws, MT)
        comm.barrier(e["chan"])
        # x[row] = x_att + ls2 * mlp; increment[row] = (x_att - x_act) + ls2 * mlp  (owners)
        comm.sp_row(MT, D, R, tok=rows, src=self._src(sess, MT), bias=lw.fc2_b, gamma=lw.ls2, resid=x_att,
                    resid_tok=False, out=x, out_tok=True, aux=sess.bos[l], aux_mode=K.AUX_OUT_MINUS, resid2=x_act)

    # -------------------------------------------------------------- outputs
    def normed_tokens(self, sess: Session) -> torch.Tensor:
        """Final LayerNorm of every token on its owner, gathered to every rank [B*N, D]."""
        c = self.cfg
        subs = sess.extra.get("subs")
        if subs is not None:
            buf = sess.extra.get("sym_normed")
            if buf is None:
                buf = sess.extra["sym_normed"] = self.comm.empty((sess.B * sess.N, c.embed_dim), BF16)
                Mh = sess.B // len(subs) * sess.N
                for i, sub in enumerate(subs):
                    sub.extra["sym_normed"] = SymTensor(buf.local[i * Mh:(i + 1) * Mh],
                                                        buf.view_ptrs(i * Mh * c.embed_dim))
            for sub in subs:
                self.normed_tokens(sub)
            return buf.local
        buf = sess.extra.get("sym_normed")
        if buf is None:
            buf = sess.extra["sym_normed"] = self.comm.empty((sess.B * sess.N, c.embed_dim), BF16)
        self.comm.sp_row(sess.B * sess.N, c.embed_dim, sess.extra["R"], x=sess.x, ln_w=self.w.norm_w,
                         ln_b=self.w.norm_b, eps=c.norm_eps, ag=buf)
        self.comm.barrier(sess.extra["chan"])
        return buf.local

    def patch_features(self, sess: Session, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Final LayerNorm of the patch tokens on their owners, gathered to every rank [B*P, D]."""
        c = self.cfg
        subs = sess.extra.get("subs")
        if subs is not None:
            for sub in subs:
                self.patch_features(sub)
            feat = sess.extra["feat"].local
            if out is not None:
                out.copy_(feat)
                return out
            return feat
        feat = sess.extra["sym_feat"]
        self.comm.sp_row(sess.B * sess.P, c.embed_dim, sess.extra["R"], tok=sess.patch_rows, x=sess.x,
                         ln_w=self.w.norm_w, ln_b=self.w.norm_b, eps=c.norm_eps, ag=feat)
        self.comm.barrier(sess.extra["chan"])
        if out is not None:
            out.copy_(feat.local)
            return out
        return feat.local
