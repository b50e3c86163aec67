"""sm_100a engine for the Qwen2.5-VL-shaped model (models/qwen25vl.py): vision tower, LLM prefill
in approximate / correct mode with a paged K/V cache, and the first-token head.

Kernel path (no PyTorch compute op on the per-layer path):
    vision   im2col (window-major patch order) -> patch GEMM -> per block
             RMSNorm -> qkv GEMM [bias, 2-D RoPE, split] -> windowed / full attention
             -> proj GEMM [+ residual] -> RMSNorm -> gate|up GEMM [SwiGLU] -> down GEMM [+ residual]
             -> RMSNorm -> merge fc1 GEMM [GELU] -> fc2 GEMM scattered into the LLM input rows
    LLM approx   RMSNorm -> qkv GEMM [bias, M-RoPE, K/V into their cache pages]
             -> causal grouped-query attention over the paged cache -> o GEMM [+ residual,
             increment := attn] -> RMSNorm -> SwiGLU GEMM -> down GEMM [+ residual, increment += mlp]
    LLM correct  RMSNorm of the kept rows (gather) -> x += increment -> qkv GEMM on kept rows
             [K/V rewritten in place in the cache] -> attention of the packed queries with each
             query's own causal frontier -> o GEMM [x_act + attn] -> RMSNorm -> SwiGLU -> down GEMM
             [scattered into x]
    vision correct  (after an approximate tower pass that kept every block's K / V)
             patch drift ||cols_new - cols_old||^2 per patch -> summed per 2x2 merge unit -> top-k
             units -> their 4 patches only: patch GEMM -> per block RMSNorm -> qkv GEMM [K / V of
             the corrected tokens rewritten in the block's cache] -> attention of the packed
             corrected queries over the cache, each within its own window (per-query key ranges)
             or over all tokens -> proj / SwiGLU / down GEMMs -> merger on the corrected units,
             scattered into their LLM input rows
The LLM then corrects the prompt text plus exactly the image rows of the corrected units.

Head dims that are not 64 / 128 (the tower's 80) run zero-padded to the next supported size:
rotate-half pairs (d, d + Dh/2) are kept by placing the two halves at [0, Dh/2) and
[Dp/2, Dp/2 + Dh/2); the padded q / k / v columns are zero, so scores and outputs are unchanged.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from ..ops import kernels as K
from .qwen25vl import (CLIP_MEAN, CLIP_STD, Qwen25VL, Qwen25VLConfig, merge_unit_raster, mrope_positions,
                       mrope_tables, vision_rope, window_order)
from .weights import SWIGLU_BLOCK, pack_swiglu

BF16 = torch.bfloat16
PAGE = 128  # rows per K/V cache page


def _pad_to(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def _padded_head(dh: int) -> int:
    if dh > 128:
        raise ValueError("head_dim > 128 is not supported")
    return 64 if dh <= 64 else 128


def _pad_head_rows(w: torch.Tensor, heads: int, dh: int, dp: int) -> torch.Tensor:
    """[heads*dh, ...] -> [heads*dp, ...] with the rotate-half halves at [0, dh/2) and [dp/2, dp/2+dh/2)."""
    tail = w.shape[1:]
    v = w.reshape(heads, dh, *tail)
    out = w.new_zeros(heads, dp, *tail)
    h2, p2 = dh // 2, dp // 2
    out[:, :h2] = v[:, :h2]
    out[:, p2:p2 + h2] = v[:, h2:]
    return out.reshape(heads * dp, *tail)


def _pad_table(t: torch.Tensor, dh: int, dp: int, fill: float) -> torch.Tensor:
    out = torch.full((t.shape[0], dp), fill, dtype=t.dtype)
    h2, p2 = dh // 2, dp // 2
    out[:, :h2] = t[:, :h2]
    out[:, p2:p2 + h2] = t[:, h2:]
    return out


@dataclass
class VisW:
    norm1: torch.Tensor
    qkv_w: torch.Tensor
    qkv_b: torch.Tensor
    proj_w: torch.Tensor
    proj_b: torch.Tensor
    norm2: torch.Tensor
    w12: torch.Tensor
    b12: torch.Tensor
    w3: torch.Tensor
    b3: torch.Tensor


@dataclass
class LlmW:
    norm1: torch.Tensor
    qkv_w: torch.Tensor
    qkv_b: torch.Tensor
    o_w: torch.Tensor
    norm2: torch.Tensor
    w12: torch.Tensor
    w3: torch.Tensor


@dataclass
class QwenSession:
    img_hw: Tuple[int, int]
    n_before: int
    n_after: int
    n_img: int
    N: int
    T: int                                   # vision tokens
    tensors: Dict[str, torch.Tensor] = field(default_factory=dict)
    approx_done: bool = False


class QwenVLEngine:
    """precision "fp8": the LLM's four GEMMs per layer run on e4m3 operands (per-row activation /
    per-channel weight scales, RMSNorm emitting e4m3 rows directly); the vision tower stays bf16."""

    def __init__(self, model: Qwen25VL, device, precision: str = "bf16"):
        if precision not in ("bf16", "fp8"):
            raise ValueError(f"precision must be bf16 or fp8, got {precision!r}")
        self.fp8 = precision == "fp8"
        self.cfg = c = model.cfg
        self.device = dev = torch.device(device)
        bf = lambda t: t.detach().to(device=dev, dtype=BF16).contiguous()  # noqa: E731
        # ---------------- vision
        self.vdp = _padded_head(c.vis_head_dim)
        self.vffn = _pad_to(c.vis_ffn, SWIGLU_BLOCK)
        self.kpatch = _pad_to(3 * c.patch ** 2, 16)
        pw = model.visual.patch_embed.weight.detach().float()
        self.patch_w = bf(torch.nn.functional.pad(pw, (0, self.kpatch - pw.shape[1])))
        self.vis: List[VisW] = []
        H, dh, dp = c.vis_heads, c.vis_head_dim, self.vdp
        for blk in model.visual.blocks:
            qkv_w = blk.qkv.weight.detach().float().view(3, H * dh, -1)
            qkv_b = blk.qkv.bias.detach().float().view(3, H * dh)
            qkv_w = torch.cat([_pad_head_rows(qkv_w[i], H, dh, dp) for i in range(3)])
            qkv_b = torch.cat([_pad_head_rows(qkv_b[i], H, dh, dp) for i in range(3)])
            proj_w = _pad_head_rows(blk.proj.weight.detach().float().T, H, dh, dp).T
            g, u, d = blk.mlp.gate_proj, blk.mlp.up_proj, blk.mlp.down_proj
            pad = self.vffn - c.vis_ffn
            w1 = torch.nn.functional.pad(g.weight.detach().float(), (0, 0, 0, pad))
            w2 = torch.nn.functional.pad(u.weight.detach().float(), (0, 0, 0, pad))
            b1 = torch.nn.functional.pad(g.bias.detach().float(), (0, pad))
            b2 = torch.nn.functional.pad(u.bias.detach().float(), (0, pad))
            w12, b12 = pack_swiglu(w1, w2, b1, b2)
            w3 = torch.nn.functional.pad(d.weight.detach().float(), (0, pad))
            self.vis.append(VisW(bf(blk.norm1.weight), bf(qkv_w), bf(qkv_b), bf(proj_w), bf(blk.proj.bias),
                                 bf(blk.norm2.weight), bf(w12), bf(b12), bf(w3), bf(d.bias)))
        mg = model.visual.merger
        self.merge_norm = bf(mg.ln_q.weight)
        self.merge_w1, self.merge_b1 = bf(mg.fc1.weight), bf(mg.fc1.bias)
        self.merge_w2, self.merge_b2 = bf(mg.fc2.weight), bf(mg.fc2.bias)
        self.vis_ones = torch.ones(c.vis_hidden, device=dev, dtype=BF16)
        # ---------------- LLM
        if c.head_dim not in (64, 128):
            raise ValueError("LLM head_dim must be 64 or 128")
        self.embed = bf(model.embed_tokens.weight)
        self.llm: List[LlmW] = []
        for ly in model.layers:
            qkv_w = torch.cat([ly.q_proj.weight, ly.k_proj.weight, ly.v_proj.weight]).detach()
            qkv_b = torch.cat([ly.q_proj.bias, ly.k_proj.bias, ly.v_proj.bias]).detach()
            w12, _ = pack_swiglu(ly.mlp.gate_proj.weight.detach(), ly.mlp.up_proj.weight.detach(), None, None)
            self.llm.append(LlmW(bf(ly.input_layernorm.weight), bf(qkv_w), bf(qkv_b), bf(ly.o_proj.weight),
                                 bf(ly.post_attention_layernorm.weight), bf(w12), bf(ly.mlp.down_proj.weight)))
        self.q8 = None
        if self.fp8:
            self.q8 = [{n: K.quantize_weight_e4m3(getattr(w, n)) for n in ("qkv_w", "o_w", "w12", "w3")}
                       for w in self.llm]
        self.nh, self.nkv, self.nffn = c.heads, c.kv_heads, c.ffn  # heads / hidden held by this process
        self.norm = bf(model.norm.weight)
        lm = model.lm_head.weight.detach()
        self.lm_head = bf(torch.nn.functional.pad(lm, (0, 0, 0, _pad_to(c.vocab, 32) - c.vocab)))
        self.ones = torch.ones(c.hidden, device=dev, dtype=BF16)

    # ------------------------------------------------------------------ sessions
    def new_session(self, H: int, W: int, n_before: int, n_after: int) -> QwenSession:
        c, dev = self.cfg, self.device
        gh, gw = H // c.patch, W // c.patch
        if gh % c.window or gw % c.window:
            raise ValueError(f"image {H}x{W} must tile into {c.window * c.patch}-pixel windows")
        T = gh * gw
        n_img = T // c.merge ** 2
        N = n_before + n_img + n_after
        e = lambda *s, dtype=BF16: torch.empty(*s, device=dev, dtype=dtype)  # noqa: E731
        sess = QwenSession((H, W), n_before, n_after, n_img, N, T)
        t = sess.tensors
        order = window_order(gh, gw, c.window, c.merge)
        t["order"] = order.to(device=dev, dtype=torch.int32)
        s, co = vision_rope(c, gh, gw, order)
        t["vsin"] = _pad_table(s, c.vis_head_dim, self.vdp, 0.0).to(dev).contiguous()
        t["vcos"] = _pad_table(co, c.vis_head_dim, self.vdp, 1.0).to(dev).contiguous()
        t["nwin"] = torch.tensor((gh // c.window) * (gw // c.window))
        t["cols"] = torch.zeros(T, self.kpatch, device=dev, dtype=BF16)
        dv = c.vis_hidden
        hp = c.vis_heads * self.vdp
        t["vx"], t["vxn"] = e(T, dv), e(T, dv)
        t["vq"], t["vo"] = e(T, hp), e(T, hp)
        # every block's keys / values of the approximate pass (the corrected tokens overwrite theirs)
        t["vkc"], t["vvc"] = e(c.vis_depth, T, hp), e(c.vis_depth, T, hp)
        t["cols_new"] = torch.zeros(T, self.kpatch, device=dev, dtype=BF16)
        t["vdrift"] = torch.zeros(T, device=dev, dtype=torch.float32)
        t["vrows"] = torch.zeros(T, device=dev, dtype=torch.int32)
        t["vh"] = e(T, self.vffn)
        t["m1"] = e(n_img, dv * c.merge ** 2)
        # merged unit u (tower order) -> its LLM input row
        t["img_rows"] = (n_before + merge_unit_raster(c, gh, gw)).to(device=dev, dtype=torch.int32)
        pos = mrope_positions(n_before, gh // c.merge, gw // c.merge, n_after)
        s, co = mrope_tables(c, pos)
        t["sin"], t["cos"] = s.to(dev).contiguous(), co.to(dev).contiguous()
        D, L, kvd = c.hidden, c.depth, self.nkv * c.head_dim
        t["x_in"], t["x"], t["xn"] = e(N, D), e(N, D), e(N, D)
        t["q"], t["o"] = e(N, self.nh * c.head_dim), e(N, self.nh * c.head_dim)
        t["h"] = e(N, self.nffn)
        t["x_act"], t["x_att"] = e(N, D), e(N, D)
        t["bos"] = e(L, N, D)
        t["emb_prev"] = e(n_img, D)
        # paged K/V pool: pages handed out in reverse so logical and physical order differ
        npages = (N + PAGE - 1) // PAGE
        table = torch.arange(npages - 1, -1, -1, dtype=torch.int32)
        t["block_table"] = table[None].to(dev).contiguous()
        phys = (table.long()[torch.arange(N) // PAGE] * PAGE + torch.arange(N) % PAGE).to(torch.int32)
        t["phys"] = phys.to(dev)
        t["kc"] = torch.zeros(L, npages * PAGE, kvd, device=dev, dtype=BF16)
        t["vc"] = torch.zeros(L, npages * PAGE, kvd, device=dev, dtype=BF16)
        t["score"] = torch.zeros(1, N, device=dev)
        t["pre"] = torch.cat([torch.arange(n_before), torch.arange(n_before + n_img, N)]).to(
            device=dev, dtype=torch.int32)[None].contiguous()
        t["cand"] = torch.arange(n_before, n_before + n_img, device=dev, dtype=torch.int32)[None].contiguous()
        t["upd"] = torch.zeros(1, N, device=dev, dtype=torch.int32)
        t["rows"] = torch.zeros(N, device=dev, dtype=torch.int32)
        t["plan_stats"] = torch.zeros(1, 2, device=dev)
        t["logits"] = e(1, _pad_to(c.vocab, 32), dtype=torch.float32)
        if self.fp8:
            t["a8"] = torch.empty(N, max(D, self.nffn), device=dev, dtype=torch.float8_e4m3fn)
            t["a8s"] = torch.empty(N, device=dev, dtype=torch.float32)
        return sess

    # ------------------------------------------------------------------ LLM operand helpers
    def _norm(self, t, x, w, out, **kw):
        """RMSNorm feeding a GEMM -> (operand, row scales or None)."""
        if not self.fp8:
            K.rmsnorm(x, w, self.cfg.rms_eps, out, **kw)
            return out, None
        n = out.shape[0]
        q8, sc = t["a8"][:n, :out.shape[1]], t["a8s"][:n]
        K.layernorm(x, w, None, self.cfg.rms_eps, q8, scale8=sc, rms=True, **kw)
        return q8, sc

    def _act(self, t, a):
        if not self.fp8:
            return a, None
        n, k = a.shape
        q8, sc = t["a8"][:n, :k], t["a8s"][:n]
        K.quant_rows_e4m3(a, q8, sc)
        return q8, sc

    def _wt(self, l: int, name: str):
        if self.fp8:
            return self.q8[l][name]
        return getattr(self.llm[l], name), None

    # ------------------------------------------------------------------ vision tower
    def vision(self, sess: QwenSession, img: torch.Tensor) -> None:
        """uint8 [1, H, W, 3] canvas -> image embeddings written into x_in's image rows."""
        c, t = self.cfg, sess.tensors
        T, dp = sess.T, self.vdp
        K.patch_im2col(img, c.patch, t["cols"], mean=CLIP_MEAN, std=CLIP_STD, perm=t["order"])
        x, xn = t["vx"], t["vxn"]
        K.gemm(t["cols"], self.patch_w, x)
        nwin = int(t["nwin"])
        eps = 1e-6
        for i, w in enumerate(self.vis):
            K.rmsnorm(x, w.norm1, eps, xn)
            K.qkv_gemm(xn, w.qkv_w, w.qkv_b, t["vq"], t["vkc"][i], t["vvc"][i], head_dim=dp, seq_len=T,
                       rope=(t["vsin"], t["vcos"]), n_prefix=0)
            B = 1 if i in c.full_attn_layers else nwin
            K.attention(t["vq"], t["vkc"][i], t["vvc"][i], t["vo"], B=B, Tq=T // B, Tk=T // B, H=c.vis_heads,
                        Dh=dp, scale=c.vis_head_dim ** -0.5)
            K.gemm(t["vo"], w.proj_w, x, epi=K.EPI_RESID, bias=w.proj_b, gamma=self.vis_ones, resid=x)
            K.rmsnorm(x, w.norm2, eps, xn)
            K.gemm(xn, w.w12, t["vh"], epi=K.EPI_SWIGLU, bias=w.b12)
            K.gemm(t["vh"], w.w3, x, epi=K.EPI_RESID, bias=w.b3, gamma=self.vis_ones, resid=x)
        K.rmsnorm(x, self.merge_norm, eps, xn)
        K.gemm(xn.view(sess.n_img, -1), self.merge_w1, t["m1"], epi=K.EPI_GELU, bias=self.merge_b1)
        K.gemm(t["m1"], self.merge_w2, t["x_in"], bias=self.merge_b2, out_rows=t["img_rows"])

    def vision_correct(self, sess: QwenSession, img: torch.Tensor, keep_ratio: float) -> torch.Tensor:
        """Partial tower correction on the new canvas (after `vision` ran on the approximate one):
        the keep_ratio share of merge units whose pixels moved most is recomputed through every
        block against the cached keys / values of the rest; their merged embeddings replace
        their LLM input rows. -> the corrected units (int32, tower order, ascending)."""
        c, t = self.cfg, sess.tensors
        T, dp, g = sess.T, self.vdp, c.merge ** 2
        K.patch_im2col(img, c.patch, t["cols_new"], mean=CLIP_MEAN, std=CLIP_STD, perm=t["order"])
        K.row_sqdist(t["cols_new"], t["cols"], t["vdrift"])
        k = min(max(int(sess.n_img * keep_ratio), 1), sess.n_img)
        units = torch.topk(t["vdrift"].view(sess.n_img, g).sum(1), k, sorted=False).indices.sort().values
        units = units.to(torch.int32)
        n = k * g
        rows = t["vrows"][:n]
        torch.add(units[:, None] * g, torch.arange(g, device=self.device, dtype=torch.int32)[None],
                  out=rows.view(k, g))
        cols = torch.empty(n, self.kpatch, device=self.device, dtype=BF16)
        K.gather_rows(t["cols_new"], rows, cols)
        K.scatter_rows(cols, rows, t["cols"])        # these patches are now current in the tower
        x, xn = t["vx"][:n], t["vxn"][:n]
        q, o, h = t["vq"][:n], t["vo"][:n], t["vh"][:n]
        K.gemm(cols, self.patch_w, x)
        w_tok = c.window ** 2                         # tokens per attention window (tower order)
        lo_w = (rows // w_tok) * w_tok
        hi_w = lo_w + (w_tok - 1)
        lo_f = torch.zeros_like(rows)
        hi_f = torch.full_like(rows, T - 1)
        eps = 1e-6
        for i, w in enumerate(self.vis):
            K.rmsnorm(x, w.norm1, eps, xn)
            K.qkv_gemm(xn, w.qkv_w, w.qkv_b, q, t["vkc"][i], t["vvc"][i], head_dim=dp, tok_idx=rows,
                       kv_rows=rows, rope=(t["vsin"], t["vcos"]), n_prefix=0)
            full = i in c.full_attn_layers
            K.attention(q, t["vkc"][i], t["vvc"][i], o, B=1, Tq=n, Tk=T, H=c.vis_heads, Dh=dp,
                        scale=c.vis_head_dim ** -0.5, causal=True, q_pos=hi_f if full else hi_w,
                        q_lo=lo_f if full else lo_w)
            K.gemm(o, w.proj_w, x, epi=K.EPI_RESID, bias=w.proj_b, gamma=self.vis_ones, resid=x)
            K.rmsnorm(x, w.norm2, eps, xn)
            K.gemm(xn, w.w12, h, epi=K.EPI_SWIGLU, bias=w.b12)
            K.gemm(h, w.w3, x, epi=K.EPI_RESID, bias=w.b3, gamma=self.vis_ones, resid=x)
        K.rmsnorm(x, self.merge_norm, eps, xn)
        m1 = t["m1"][:k]
        K.gemm(xn.view(k, -1), self.merge_w1, m1, epi=K.EPI_GELU, bias=self.merge_b1)
        out_rows = t["img_rows"].index_select(0, units)
        K.gemm(m1, self.merge_w2, t["x_in"], bias=self.merge_b2, out_rows=out_rows)
        return units

    def embed_text(self, sess: QwenSession, ids: torch.Tensor) -> None:
        """int32 token ids of the text rows ([n_before + n_after], prompt order) -> x_in rows."""
        t = sess.tensors
        rows = t["pre"].view(-1)
        emb = torch.empty(rows.numel(), self.cfg.hidden, device=self.device, dtype=BF16)
        K.gather_rows(self.embed, ids.to(torch.int32), emb)
        K.scatter_rows(emb, rows, t["x_in"])

    # ------------------------------------------------------------------ LLM
    def approx(self, sess: QwenSession) -> torch.Tensor:
        c, t = self.cfg, sess.tensors
        N = sess.N
        x, xn = t["x"], t["xn"]
        x.copy_(t["x_in"])
        for l, w in enumerate(self.llm):
            a, sa = self._norm(t, x, w.norm1, xn)
            wq, sw = self._wt(l, "qkv_w")
            K.qkv_gemm(a, wq, w.qkv_b, t["q"], t["kc"][l], t["vc"][l], head_dim=c.head_dim, seq_len=N,
                       kv_rows=t["phys"], rope=(t["sin"], t["cos"]), n_prefix=0,
                       kv_dim=c.kv_heads * c.head_dim, a_scale=sa, b_scale=sw)
            K.attention(t["q"], t["kc"][l], t["vc"][l], t["o"], B=1, Tq=N, Tk=N, H=c.heads, Dh=c.head_dim,
                        Hkv=c.kv_heads, causal=True, block_table=t["block_table"])
            a, sa = self._act(t, t["o"])
            wq, sw = self._wt(l, "o_w")
            K.gemm(a, wq, x, epi=K.EPI_RESID, gamma=self.ones, resid=x, aux=t["bos"][l],
                   aux_mode=K.AUX_SET, a_scale=sa, b_scale=sw)
            a, sa = self._norm(t, x, w.norm2, xn)
            wq, sw = self._wt(l, "w12")
            K.gemm(a, wq, t["h"], epi=K.EPI_SWIGLU, a_scale=sa, b_scale=sw)
            a, sa = self._act(t, t["h"])
            wq, sw = self._wt(l, "w3")
            K.gemm(a, wq, x, epi=K.EPI_RESID, gamma=self.ones, resid=x, aux=t["bos"][l],
                   aux_mode=K.AUX_ADD, a_scale=sa, b_scale=sw)
        t["emb_prev"].copy_(t["x_in"][sess.n_before:sess.n_before + sess.n_img])
        sess.approx_done = True
        return x

    def plan(self, sess: QwenSession, keep_ratio: float,
             units: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Text rows plus image rows (ascending positions): the rows of the corrected merge units
        `units` (tower order) when given, else the top-k image rows by embedding change."""
        t = sess.tensors
        img = slice(sess.n_before, sess.n_before + sess.n_img)
        if units is not None:
            sc = t["score"].view(-1)
            sc.zero_()
            sc.index_fill_(0, t["img_rows"].index_select(0, units).long(), 1.0)
            k = units.numel()
        else:
            K.row_sqdist(t["x_in"][img], t["emb_prev"], t["score"].view(-1)[img])
            k = min(max(int(sess.n_img * keep_ratio), 0), sess.n_img)
        npre = t["pre"].shape[1]
        T = npre + k
        upd = t["upd"].view(-1)[:T].view(1, T)
        rows = t["rows"][:T]
        K.correction_plan(t["score"], t["pre"], t["cand"], k, upd, rows, stats=t["plan_stats"])
        return upd, rows

    def correct(self, sess: QwenSession, keep_ratio: float, units: Optional[torch.Tensor] = None) -> torch.Tensor:
        c, t = self.cfg, sess.tensors
        N = sess.N
        upd, rows = self.plan(sess, keep_ratio, units)
        T = upd.shape[1]
        kv_sel = t["phys"].index_select(0, rows)
        x = t["x"]
        x.copy_(t["x_in"])
        xn, q, o, h = t["xn"][:T], t["q"][:T], t["o"][:T], t["h"][:T]
        x_act, x_att = t["x_act"][:T], t["x_att"][:T]
        for l, w in enumerate(self.llm):
            a, sa = self._norm(t, x, w.norm1, xn, rows=rows, copy_out=x_act)
            K.add_(x, t["bos"][l])
            wq, sw = self._wt(l, "qkv_w")
            K.qkv_gemm(a, wq, w.qkv_b, q, t["kc"][l], t["vc"][l], head_dim=c.head_dim, tok_idx=upd.view(-1),
                       kv_rows=kv_sel, rope=(t["sin"], t["cos"]), n_prefix=0, kv_dim=c.kv_heads * c.head_dim,
                       a_scale=sa, b_scale=sw)
            K.attention(q, t["kc"][l], t["vc"][l], o, B=1, Tq=T, Tk=N, H=c.heads, Dh=c.head_dim, Hkv=c.kv_heads,
                        causal=True, q_pos=upd.view(-1), block_table=t["block_table"])
            a, sa = self._act(t, o)
            wq, sw = self._wt(l, "o_w")
            K.gemm(a, wq, x_att, epi=K.EPI_RESID, gamma=self.ones, resid=x_act, a_scale=sa, b_scale=sw)
            a, sa = self._norm(t, x_att, w.norm2, xn)
            wq, sw = self._wt(l, "w12")
            K.gemm(a, wq, h, epi=K.EPI_SWIGLU, a_scale=sa, b_scale=sw)
            a, sa = self._act(t, h)
            wq, sw = self._wt(l, "w3")
            K.gemm(a, wq, x, epi=K.EPI_RESID, gamma=self.ones, resid=x_att, out_rows=rows, a_scale=sa, b_scale=sw)
        t["emb_prev"].copy_(t["x_in"][sess.n_before:sess.n_before + sess.n_img])
        return x

    def first_token(self, sess: QwenSession) -> torch.Tensor:
        """Greedy next token after the prompt: argmax of the LM head on the last row (device int64)."""
        c, t = self.cfg, sess.tensors
        last = torch.full((1,), sess.N - 1, device=self.device, dtype=torch.int32)
        xn = t["xn"][:1]
        K.rmsnorm(t["x"], self.norm, c.rms_eps, xn, rows=last)
        lm = t["logits"]
        K.gemm(xn, self.lm_head, lm, epi=K.EPI_F32)
        return lm[0, : c.vocab].argmax()
