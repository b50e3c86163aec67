"""Tensor-parallel LLM of the Qwen2.5-VL-shaped model, sequence-parallel layout.

Same layout and collectives as parallel/tp.py (ViT): query and key/value heads and the SwiGLU
hidden units are split across ranks (q/k/v and gate/up by output, o and down by input), the
residual stream and the increment cache are split by token rows, and each row-parallel GEMM's
partial product is reduced by the row's owner in the csrc/tp_sp.cu row kernel, which also applies
the residual, the increment bookkeeping and the next RMSNorm, and all-gathers the normalised row
(e4m3 + scale, or bf16) into every rank's GEMM operand. The paged K/V cache holds each rank's own
key/value heads. The vision tower runs replicated on every rank (its output rows are spliced into
every rank's input). Reference: none (the reference is single-GPU); semantics are those of
models/qwen_engine.py.
"""
from __future__ import annotations

import torch

from ..models.qwen25vl import Qwen25VL
from ..models.qwen_engine import BF16, LlmW, QwenSession, QwenVLEngine
from ..models.weights import SWIGLU_BLOCK, pack_swiglu, unpack_swiglu
from ..ops import kernels as K
from .comm import SymTensor, TPComm


def shard_llm_layer(w: LlmW, heads: int, kv_heads: int, dh: int, rank: int, world: int) -> LlmW:
    hq, hk = heads // world, kv_heads // world
    qd, kd = heads * dh, kv_heads * dh
    qs = slice(rank * hq * dh, (rank + 1) * hq * dh)
    ks = slice(rank * hk * dh, (rank + 1) * hk * dh)
    qkv_w = torch.cat([w.qkv_w[:qd][qs], w.qkv_w[qd:qd + kd][ks], w.qkv_w[qd + kd:][ks]]).contiguous()
    qkv_b = torch.cat([w.qkv_b[:qd][qs], w.qkv_b[qd:qd + kd][ks], w.qkv_b[qd + kd:][ks]]).contiguous()
    w1, w2 = unpack_swiglu(w.w12)
    f = w1.shape[0] // world
    fs = slice(rank * f, (rank + 1) * f)
    w12, _ = pack_swiglu(w1[fs].contiguous(), w2[fs].contiguous(), None, None)
    return LlmW(w.norm1, qkv_w, qkv_b, w.o_w[:, qs].contiguous(), w.norm2, w12, w.w3[:, fs].contiguous())


class QwenVLEngineTP(QwenVLEngine):
    def __init__(self, model: Qwen25VL, comm: TPComm, precision: str = "bf16"):
        super().__init__(model, comm.device, "bf16")
        c = self.cfg
        T, r = comm.world, comm.rank
        if c.heads % T or c.kv_heads % T or c.ffn % (T * SWIGLU_BLOCK):
            raise ValueError(f"heads {c.heads}, kv heads {c.kv_heads} and FFN {c.ffn} must split over {T} ranks")
        self.comm, self.world, self.rank = comm, T, r
        self.llm = [shard_llm_layer(w, c.heads, c.kv_heads, c.head_dim, r, T) for w in self.llm]
        self.nh, self.nkv, self.nffn = c.heads // T, c.kv_heads // T, c.ffn // T
        self.fp8 = precision == "fp8"
        if self.fp8:
            self.q8 = [{n: K.quantize_weight_e4m3(getattr(w, n)) for n in ("qkv_w", "o_w", "w12", "w3")}
                       for w in self.llm]
        torch.cuda.empty_cache()

    # ------------------------------------------------------------------ sessions
    def new_session(self, H: int, W: int, n_before: int, n_after: int) -> QwenSession:
        sess = super().new_session(H, W, n_before, n_after)
        c, comm = self.cfg, self.comm
        N, D = sess.N, c.hidden
        t = sess.tensors
        xg = comm.empty((N, D), BF16)
        t.update({
            "R": (N + self.world - 1) // self.world, "chan": comm.channel(), "sym_xg": xg,
            "sym_xg8": SymTensor(xg.local.view(torch.uint8).view(-1)[: N * D].view(N, D).view(torch.float8_e4m3fn),
                                 xg.ptrs),
            "sym_xg_scale": comm.empty((N,), torch.float32), "sym_part": comm.empty((N, D), BF16),
            "sym_last": comm.empty((1, D), BF16),
            "last_row": torch.full((1,), N - 1, device=self.device, dtype=torch.int32)})
        return sess

    # ------------------------------------------------------------------ helpers
    def _gathered(self, t, n: int):
        if self.fp8:
            return t["sym_xg8"].local[:n], t["sym_xg_scale"].local[:n]
        return t["sym_xg"].local[:n], None

    def _ag(self, t):
        if self.fp8:
            return {"ag": t["sym_xg8"], "ag_scale": t["sym_xg_scale"]}
        return {"ag": t["sym_xg"]}

    def _src(self, t):
        return t["sym_part"].ptrs, [0] * self.world

    def _bar(self, t):
        self.comm.barrier(t["chan"])

    # ------------------------------------------------------------------ LLM
    def approx(self, sess: QwenSession) -> torch.Tensor:
        c, t, comm = self.cfg, sess.tensors, self.comm
        N, D, R = sess.N, c.hidden, t["R"]
        x = t["x"]
        x.copy_(t["x_in"])
        comm.sp_row(N, D, R, x=x, ln_w=self.llm[0].norm1, eps=c.rms_eps, rms=True, **self._ag(t))
        self._bar(t)
        part = t["sym_part"].local
        for l, w in enumerate(self.llm):
            a, sa = self._gathered(t, N)
            wq, sw = self._wt(l, "qkv_w")
            K.qkv_gemm(a, wq, w.qkv_b, t["q"], t["kc"][l], t["vc"][l], head_dim=c.head_dim, seq_len=N,
                       kv_rows=t["phys"], rope=(t["sin"], t["cos"]), n_prefix=0, kv_dim=self.nkv * c.head_dim,
                       a_scale=sa, b_scale=sw)
            K.attention(t["q"], t["kc"][l], t["vc"][l], t["o"], B=1, Tq=N, Tk=N, H=self.nh, Dh=c.head_dim,
                        Hkv=self.nkv, causal=True, block_table=t["block_table"])
            a, sa = self._act(t, t["o"])
            wq, sw = self._wt(l, "o_w")
            K.gemm(a, wq, part, a_scale=sa, b_scale=sw)
            self._bar(t)
            comm.sp_row(N, D, R, src=self._src(t), resid=x, out=x, aux=t["bos"][l], aux_mode=K.AUX_SET,
                        ln_w=w.norm2, eps=c.rms_eps, rms=True, **self._ag(t))
            self._bar(t)
            a, sa = self._gathered(t, N)
            wq, sw = self._wt(l, "w12")
            K.gemm(a, wq, t["h"], epi=K.EPI_SWIGLU, a_scale=sa, b_scale=sw)
            a, sa = self._act(t, t["h"])
            wq, sw = self._wt(l, "w3")
            K.gemm(a, wq, part, a_scale=sa, b_scale=sw)
            self._bar(t)
            nxt = self.llm[l + 1].norm1 if l + 1 < len(self.llm) else None
            comm.sp_row(N, D, R, src=self._src(t), resid=x, out=x, aux=t["bos"][l], aux_mode=K.AUX_ADD,
                        ln_w=nxt, eps=c.rms_eps, rms=True, **self._ag(t))
            if nxt is not None:
                self._bar(t)
        t["emb_prev"].copy_(t["x_in"][sess.n_before:sess.n_before + sess.n_img])
        sess.approx_done = True
        return x

    def correct(self, sess: QwenSession, keep_ratio: float, units=None) -> torch.Tensor:
        c, t, comm = self.cfg, sess.tensors, self.comm
        N, D, R = sess.N, c.hidden, t["R"]
        upd, rows = self.plan(sess, keep_ratio, units)
        T = upd.shape[1]
        kv_sel = t["phys"].index_select(0, rows)
        x = t["x"]
        x.copy_(t["x_in"])
        q, o, h = t["q"][:T], t["o"][:T], t["h"][:T]
        x_act, x_att = t["x_act"][:T], t["x_att"][:T]
        part = t["sym_part"].local[:T]
        lo, hi = self.rank * R, min((self.rank + 1) * R, N)
        for l, w in enumerate(self.llm):
            comm.sp_row(T, D, R, tok=rows, x=x, copy_out=x_act, ln_w=w.norm1, eps=c.rms_eps, rms=True,
                        **self._ag(t))
            K.add_(x[lo:hi], t["bos"][l][lo:hi])
            self._bar(t)
            a, sa = self._gathered(t, T)
            wq, sw = self._wt(l, "qkv_w")
            K.qkv_gemm(a, wq, w.qkv_b, q, t["kc"][l], t["vc"][l], head_dim=c.head_dim, tok_idx=upd.view(-1),
                       kv_rows=kv_sel, rope=(t["sin"], t["cos"]), n_prefix=0, kv_dim=self.nkv * c.head_dim,
                       a_scale=sa, b_scale=sw)
            K.attention(q, t["kc"][l], t["vc"][l], o, B=1, Tq=T, Tk=N, H=self.nh, Dh=c.head_dim, Hkv=self.nkv,
                        causal=True, q_pos=upd.view(-1), block_table=t["block_table"])
            a, sa = self._act(t, o)
            wq, sw = self._wt(l, "o_w")
            K.gemm(a, wq, part, a_scale=sa, b_scale=sw)
            self._bar(t)
            comm.sp_row(T, D, R, tok=rows, src=self._src(t), resid=x_act, resid_tok=False, out=x_att,
                        out_tok=False, ln_w=w.norm2, eps=c.rms_eps, rms=True, **self._ag(t))
            self._bar(t)
            a, sa = self._gathered(t, T)
            wq, sw = self._wt(l, "w12")
            K.gemm(a, wq, h, epi=K.EPI_SWIGLU, a_scale=sa, b_scale=sw)
            a, sa = self._act(t, h)
            wq, sw = self._wt(l, "w3")
            K.gemm(a, wq, part, a_scale=sa, b_scale=sw)
            self._bar(t)
            comm.sp_row(T, D, R, tok=rows, src=self._src(t), resid=x_att, resid_tok=False, out=x, out_tok=True)
        t["emb_prev"].copy_(t["x_in"][sess.n_before:sess.n_before + sess.n_img])
        return x

    def first_token(self, sess: QwenSession) -> torch.Tensor:
        c, t = self.cfg, sess.tensors
        last = t["sym_last"]
        self.comm.sp_row(1, c.hidden, t["R"], tok=t["last_row"], x=t["x"], ln_w=self.norm, eps=c.rms_eps, rms=True,
                         ag=last)
        self._bar(t)
        lm = t["logits"]
        K.gemm(last.local, self.lm_head, lm, epi=K.EPI_F32)
        return lm[0, : c.vocab].argmax()
