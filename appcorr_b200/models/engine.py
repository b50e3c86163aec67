"""sm_100a execution engine for the DINOv3 ViT approximate / correct passes.

The engine owns kernel-layout copies of the backbone weights and a per-session workspace, and
drives the hand-written kernels of `appcorr_b200._C` directly; no PyTorch compute op runs on
its hot path. One layer of the approximate pass (reference block.py:312-349) is

    LN1 -> qkv GEMM [+bias, RoPE, split into q / K-cache / V-cache] -> CLS pscore
        -> attention -> proj GEMM [x + ls1*(.), increment := ls1*(.)]
        -> LN2 -> fc1/w12 GEMM [GELU | SwiGLU] -> fc2/w3 GEMM [x + ls2*(.), increment += ls2*(.)]

and one layer of the correction pass (block.py:943-1191) is

    plan (score + top-k, on device) -> gather + LN1 of the kept rows -> x += increment (all rows)
        -> qkv GEMM on kept rows [RoPE, K/V rows scattered into the cache]
        -> attention (packed queries vs. the whole cache) -> proj GEMM [x_act + ls1*(.)]
        -> LN2 -> fc1/w12 GEMM -> fc2/w3 GEMM [scatter x_attn + ls2*(.) into x;
                                               increment := (x_attn - x_act) + ls2*(.)]

Everything is statically shaped for a given (batch, resolution, keep ratio), so a pass can be
captured into a CUDA graph (see `capture`).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ..common.protocol import LAYERMEAN_SERVER_PSCORES
from ..ops import kernels as K
from .dinov3.layers import linear_bias
from .dinov3.vit import DinoVisionTransformer, ViTConfig
from .weights import SWIGLU_BLOCK, pack_swiglu, repack_swiglu

BF16 = torch.bfloat16


@dataclass
class LayerW:
    norm1_w: torch.Tensor
    norm1_b: torch.Tensor
    qkv_w: torch.Tensor
    qkv_b: Optional[torch.Tensor]
    proj_w: torch.Tensor
    proj_b: Optional[torch.Tensor]
    ls1: torch.Tensor
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor
    fc1_w: torch.Tensor           # fc1 [hidden, D] or packed w1||w2 [2*hidden, D]
    fc1_b: Optional[torch.Tensor]
    fc2_w: torch.Tensor           # fc2 / w3 [D, hidden]
    fc2_b: Optional[torch.Tensor]
    ls2: torch.Tensor
    # e4m3 copies (w8 [N, K], per-output-channel fp32 scale [N]) for the fp8 GEMM path
    q8: Optional[Dict[str, Tuple[torch.Tensor, torch.Tensor]]] = None
    # NVFP4 copies (w4 [N, K/2], (channel scale [N], block scales)) of qkv / fc1 / fc2, and the
    # fc1 bias matching the NVFP4 fc1 packing ("fc1_b")
    q4: Optional[Dict[str, object]] = None


@dataclass
class EngineWeights:
    cfg: ViTConfig
    patch_w: torch.Tensor         # [D, 3*p*p]
    patch_b: torch.Tensor         # [D]
    prefix: torch.Tensor          # [1 + n_storage, D]
    periods: torch.Tensor         # RoPE periods (fp32)
    layers: List[LayerW]
    norm_w: torch.Tensor
    norm_b: torch.Tensor
    cls_norm_w: Optional[torch.Tensor] = None
    cls_norm_b: Optional[torch.Tensor] = None
    # learned absolute position embedding [n_prefix + P, D] (periods is then None: no RoPE) and
    # a LayerNorm applied to the tokens before the first block (CLIP-style towers)
    pos_embed: Optional[torch.Tensor] = None
    pre_norm_w: Optional[torch.Tensor] = None
    pre_norm_b: Optional[torch.Tensor] = None
    pixel_mean: Tuple[float, float, float] = K.IMAGENET_MEAN
    pixel_std: Tuple[float, float, float] = K.IMAGENET_STD


def _bf(t: Optional[torch.Tensor], device) -> Optional[torch.Tensor]:
    if t is None:
        return None
    return t.detach().to(device=device, dtype=BF16).contiguous()


def weights_from_module(model: DinoVisionTransformer, device) -> EngineWeights:
    """Kernel-layout copy of a (CPU or GPU) DINOv3 module's parameters."""
    cfg = model.cfg
    layers = []
    for blk in model.blocks:
        mlp = blk.mlp
        if cfg.is_swiglu:
            w, b = pack_swiglu(mlp.w1.weight.detach(), mlp.w2.weight.detach(),
                               None if mlp.w1.bias is None else mlp.w1.bias.detach(),
                               None if mlp.w2.bias is None else mlp.w2.bias.detach())
            fc1_w, fc1_b, fc2 = w, b, mlp.w3
        else:
            fc1_w, fc1_b, fc2 = mlp.fc1.weight.detach(), mlp.fc1.bias, mlp.fc2
        layers.append(LayerW(
            norm1_w=_bf(blk.norm1.weight, device), norm1_b=_bf(blk.norm1.bias, device),
            qkv_w=_bf(blk.attn.qkv.weight, device), qkv_b=_bf(linear_bias(blk.attn.qkv), device),
            proj_w=_bf(blk.attn.proj.weight, device), proj_b=_bf(blk.attn.proj.bias, device),
            ls1=_bf(blk.ls1.gamma, device), norm2_w=_bf(blk.norm2.weight, device),
            norm2_b=_bf(blk.norm2.bias, device), fc1_w=_bf(fc1_w, device), fc1_b=_bf(fc1_b, device),
            fc2_w=_bf(fc2.weight, device), fc2_b=_bf(fc2.bias, device), ls2=_bf(blk.ls2.gamma, device)))
    pw = model.patch_embed.proj.weight.detach()
    return EngineWeights(
        cfg=cfg,
        patch_w=_bf(pw.reshape(pw.shape[0], -1), device),
        patch_b=_bf(model.patch_embed.proj.bias, device),
        prefix=_bf(model.prefix_tokens(), device),
        periods=model.rope_embed.periods.detach().to(device=device, dtype=torch.float32),
        layers=layers,
        norm_w=_bf(model.norm.weight, device), norm_b=_bf(model.norm.bias, device),
        cls_norm_w=_bf(model.cls_norm.weight, device) if model.cls_norm is not None else None,
        cls_norm_b=_bf(model.cls_norm.bias, device) if model.cls_norm is not None else None,
    )


def random_weights(cfg: ViTConfig, device, seed: int = 0, std: float = 0.02) -> EngineWeights:
    """Random-init weights generated directly on the device in kernel layout (synthetic runs).

    Same distribution family as the reference init (trunc-normal std 0.02 Linears, zero biases,
    LayerScale 1e-5, unit LayerNorm); built layer by layer so a 7B model never exists twice.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    D, Hd = cfg.embed_dim, cfg.ffn_hidden

    def lin(o, i):
        return (torch.randn(o, i, device=device, generator=g) * std).clamp_(-2 * std, 2 * std).to(BF16)

    def zeros(n):
        return torch.zeros(n, device=device, dtype=BF16)

    def ones(n):
        return torch.ones(n, device=device, dtype=BF16)

    ls = cfg.layerscale_init or 1.0
    layers = []
    for _ in range(cfg.depth):
        fc1 = 2 * Hd if cfg.is_swiglu else Hd
        layers.append(LayerW(
            norm1_w=ones(D), norm1_b=zeros(D), qkv_w=lin(3 * D, D), qkv_b=zeros(3 * D) if cfg.qkv_bias else None,
            proj_w=lin(D, D), proj_b=zeros(D) if cfg.proj_bias else None, ls1=torch.full((D,), ls, device=device, dtype=BF16),
            norm2_w=ones(D), norm2_b=zeros(D), fc1_w=lin(fc1, D), fc1_b=zeros(fc1) if cfg.ffn_bias else None,
            fc2_w=lin(D, Hd), fc2_b=zeros(D) if cfg.ffn_bias else None, ls2=torch.full((D,), ls, device=device, dtype=BF16)))
    p = cfg.patch_size
    bound = 1.0 / math.sqrt(3 * p * p)
    n = cfg.head_dim // 4
    periods = cfg.pos_embed_rope_base ** (2 * torch.arange(n, device=device, dtype=torch.float32) / (cfg.head_dim // 2))
    return EngineWeights(
        cfg=cfg,
        patch_w=((torch.rand(D, 3 * p * p, device=device, generator=g) * 2 - 1) * bound).to(BF16),
        patch_b=((torch.rand(D, device=device, generator=g) * 2 - 1) * bound).to(BF16),
        prefix=(torch.randn(cfg.n_prefix, D, device=device, generator=g) * 0.02).to(BF16),
        periods=periods, layers=layers, norm_w=ones(D), norm_b=zeros(D),
        cls_norm_w=ones(D) if cfg.untie_cls_and_patch_norms else None,
        cls_norm_b=zeros(D) if cfg.untie_cls_and_patch_norms else None)


def rope_tables(cfg: ViTConfig, periods: torch.Tensor, H: int, W: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """fp32 (sin, cos) [H*W, head_dim], same construction as RopePositionEmbedding.forward."""
    dev = periods.device
    if cfg.pos_embed_rope_normalize_coords == "max":
        dh = dw = max(H, W)
    elif cfg.pos_embed_rope_normalize_coords == "min":
        dh = dw = min(H, W)
    else:
        dh, dw = H, W
    ch = torch.arange(0.5, H, device=dev, dtype=torch.float32) / dh
    cw = torch.arange(0.5, W, device=dev, dtype=torch.float32) / dw
    coords = torch.stack(torch.meshgrid(ch, cw, indexing="ij"), dim=-1).flatten(0, 1) * 2.0 - 1.0
    ang = (2 * math.pi * coords[:, :, None] / periods.float()[None, None, :]).flatten(1, 2).tile(2)
    return torch.sin(ang).contiguous(), torch.cos(ang).contiguous()


_MISSING = object()


@dataclass
class Session:
    """Per-request device state: activations, per-layer caches and correction scratch."""

    B: int
    img_hw: Tuple[int, int]
    grid_hw: Tuple[int, int]
    N: int
    P: int
    x_in: torch.Tensor            # fresh tokens from the current canvas [B*N, D]
    x: torch.Tensor               # running features [B*N, D]
    x_tmp: torch.Tensor           # approx ping-pong partner
    xn: torch.Tensor              # LayerNorm output [B*N, D]
    q: torch.Tensor               # [B*N, D]
    o: torch.Tensor               # attention output [B*N, D]
    h: torch.Tensor               # MLP hidden [B*N, hidden]
    kc: torch.Tensor              # [L, B*N, D] K after RoPE
    vc: torch.Tensor              # [L, B*N, D]
    bos: torch.Tensor             # [L, B*N, D] per-layer increment
    pscore: torch.Tensor          # [L, B, N] fp32 server score
    ps_scratch: torch.Tensor      # [B, H, N] fp32
    cols: torch.Tensor            # im2col [B*P, 3*p*p]
    patch_rows: torch.Tensor      # int32 token rows of the patch tokens [B*P]
    rope: Tuple[torch.Tensor, torch.Tensor]
    # correction scratch (sized for keeping every candidate)
    upd: torch.Tensor
    rows: torch.Tensor
    x_act: torch.Tensor
    x_att: torch.Tensor
    plan_stats: torch.Tensor      # [B, 2] fp32
    stat_acc: torch.Tensor        # [5] fp32 accumulated plan statistics
    approx_done: int = 0
    extra: Dict[str, torch.Tensor] = field(default_factory=dict)


def _score_kind(server_pscore: str) -> str:
    """Family of a server_pscore name: "cls", "patch", "pseudo" or "none" (no attention-derived
    score: none / disabled, and random, which is drawn at correction time)."""
    k = str(server_pscore)
    if k in ("none", "disabled", "random"):
        return "none"
    if k in ("cls_attn_prob", "cls_attn_prob_layermean"):
        return "cls"
    if k in ("patch_attn_prob", "patch_attn_prob_layermean", "patch_attn_prune"):
        return "patch"
    if k in ("patch_pseudo_attn_prob", "patch_pseudo_attn_prob_layermean", "pseudo_patch_attn_prob",
             "pseudo_patch_attn_prob_layermean"):
        return "pseudo"
    raise ValueError(f"unknown server_pscore {server_pscore!r}")


PRECISIONS = ("bf16", "fp8", "nvfp4", "auto")
# "auto": e4m3 operands for a pass whose GEMMs have at least this many rows, bf16 below
# (reference dinov3_precision.py:479-488, config fp8_auto_min_rows)
AUTO_MIN_ROWS = 3072
_Q8_NAMES = ("qkv", "proj", "fc1", "fc2")
# nvfp4 precision: these GEMMs take NVFP4 operands; attn.proj stays e4m3 (the reference's
# FastFP4 path keeps proj in FP8 by default, offload/server/model/fp4_fast_linear.py)
_Q4_NAMES = ("qkv", "fc1", "fc2")


def quantize_layer_e4m3(lw: LayerW) -> None:
    """Attach per-output-channel e4m3 copies of the four GEMM weights of a layer."""
    lw.q8 = {n: K.quantize_weight_e4m3(getattr(lw, n + "_w")) for n in _Q8_NAMES}


def quantize_layer_nvfp4(lw: LayerW, swiglu: bool) -> None:
    """Attach NVFP4 copies of qkv / fc1 / fc2. A packed SwiGLU fc1 keeps blocks of half the NVFP4
    tile width of fc1 (ops.kernels.fp4_tile): 128 rows for the default 256-wide tiles, whose
    accumulator the early-release epilogue frees before its stores (ViT-7B step 87.1 ms against
    87.9 ms with 128-wide tiles); fc2 keeps 128-wide tiles (its residual epilogue measured slower
    at 256)."""
    q4: Dict[str, object] = {"fc1_b": lw.fc1_b}
    for n in _Q4_NAMES:
        w = getattr(lw, n + "_w")
        if w.shape[1] % 256:
            raise ValueError(f"nvfp4 precision needs GEMM K % 256 == 0 ({n}: K = {w.shape[1]})")
        if n == "fc1" and swiglu and K.fp4_tile("fc1") != 2 * SWIGLU_BLOCK:
            w, q4["fc1_b"] = repack_swiglu(w, lw.fc1_b, SWIGLU_BLOCK, K.fp4_tile("fc1") // 2)
        q4[n] = K.quantize_weight_nvfp4(w)
    lw.q4 = q4


class ViTEngine:
    """precision: "bf16" everywhere, "fp8" (e4m3 activations with per-row scales x e4m3 weights
    with per-channel scales on the tcgen05 kind::f8f6f4 GEMM, fp32 accumulation, bf16 residual
    stream), or a dict {"approx": ..., "correct": ...} to choose per pass (reference
    dinov3_precision.py keeps separate approx / correct precisions)."""

    def __init__(self, weights: EngineWeights, device=None, precision="bf16"):
        self.w = weights
        self.cfg = weights.cfg
        self.device = torch.device(device) if device is not None else weights.patch_w.device
        # attention head width the kernels run at (padded heads: zero rows in qkv, zero columns in
        # proj) and the softmax scale of the true head dim
        self.Dh = self.cfg.padded_head_dim or self.cfg.head_dim
        self.A = self.cfg.num_heads * self.Dh
        self.attn_scale = self.cfg.head_dim ** -0.5
        if self.Dh not in (64, 128):
            raise ValueError("the sm_100a engine supports head_dim 64 or 128 (or padded to one of them)")
        kp = (3 * self.cfg.patch_size ** 2 + 15) // 16 * 16  # patch rows padded to 16 elements
        if self.w.patch_w.shape[1] != kp:
            self.w.patch_w = torch.nn.functional.pad(self.w.patch_w, (0, kp - self.w.patch_w.shape[1])).contiguous()
        if isinstance(precision, str):
            precision = {"approx": precision, "correct": precision}
        for v in precision.values():
            if v not in PRECISIONS:
                raise ValueError(f"engine precision must be one of {PRECISIONS}, got {v!r}")
        self.precision = dict(precision)
        self.auto_min_rows = AUTO_MIN_ROWS
        low = {("fp8" if v == "auto" else v) for v in self.precision.values()} - {"bf16"}
        for lw in self.w.layers:
            if low and lw.q8 is None:
                quantize_layer_e4m3(lw)
            if "nvfp4" in low and lw.q4 is None:
                quantize_layer_nvfp4(lw, self.cfg.is_swiglu)
        self._fp8 = False  # precision of the pass being run: e4m3 or NVFP4 operands
        self._fp4 = False  # NVFP4 for the _Q4_NAMES GEMMs
        self.taps: Tuple[int, ...] = ()  # layers whose output is kept for dense heads

    @classmethod
    def from_module(cls, model: DinoVisionTransformer, device, precision="bf16") -> "ViTEngine":
        return cls(weights_from_module(model, device), device, precision)

    @classmethod
    def random(cls, cfg: ViTConfig, device, seed: int = 0, precision="bf16") -> "ViTEngine":
        return cls(random_weights(cfg, device, seed), device, precision)

    # -------------------------------------------------------------- precision helpers
    def _norm(self, sess: Session, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, out: torch.Tensor,
              rows: Optional[torch.Tensor] = None, copy_out: Optional[torch.Tensor] = None):
        """LayerNorm feeding a GEMM: returns (operand, row scale or None)."""
        if not self._fp8:
            K.layernorm(x, w, b, self.cfg.norm_eps, out, rows=rows, copy_out=copy_out)
            return out, None
        n, k = out.shape
        e = sess.extra
        if self._fp4:  # every LayerNorm feeds an NVFP4 GEMM (qkv or fc1)
            q4, s, sf = e["a4"][:n, : k // 2], e["a4_scale"][:n], e["a4_sf"]
            K.layernorm(x, w, b, self.cfg.norm_eps, q4, rows=rows, copy_out=copy_out, scale8=s, sf=sf)
            return q4, (s, sf)
        q8, s = e["a8"][:n, :k], e["a8_scale"][:n]
        K.layernorm(x, w, b, self.cfg.norm_eps, q8, rows=rows, copy_out=copy_out, scale8=s)
        return q8, s

    def _act(self, sess: Session, t: torch.Tensor, name: str = "fc2"):
        """bf16 activation feeding GEMM `name`: returns (operand, row scale(s) or None)."""
        if not self._fp8:
            return t, None
        n, k = t.shape
        e = sess.extra
        if self._fp4 and name in _Q4_NAMES:
            q4, s, sf = e["a4"][:n, : k // 2], e["a4_scale"][:n], e["a4_sf"]
            K.quant_rows_nvfp4(t, q4, sf, s)
            return q4, (s, sf)
        q8, s = e["a8"][:n, :k], e["a8_scale"][:n]
        K.quant_rows_e4m3(t, q8, s)
        return q8, s

    def _w(self, lw: LayerW, name: str):
        if self._fp4 and name in _Q4_NAMES:
            return lw.q4[name]
        if self._fp8:
            return lw.q8[name]
        return getattr(lw, name + "_w"), None

    def _fc1_bias(self, lw: LayerW):
        return lw.q4["fc1_b"] if self._fp4 else lw.fc1_b

    def _ensure_fp8_scratch(self, sess: Session) -> None:
        e = sess.extra
        M = sess.x.shape[0]
        width = max(self.cfg.embed_dim, sess.h.shape[1])
        if "a8" not in e:
            e["a8"] = torch.empty(M, width, device=self.device, dtype=torch.float8_e4m3fn)
            e["a8_scale"] = torch.empty(M, device=self.device, dtype=torch.float32)
        if self._fp4 and "a4" not in e:
            e["a4"] = torch.empty(M, width // 2, device=self.device, dtype=torch.uint8)
            e["a4_scale"] = torch.empty(M, device=self.device, dtype=torch.float32)
            e["a4_sf"] = torch.zeros(K.nvfp4_sf_bytes(M, width), device=self.device, dtype=torch.uint8)

    def effective_precision(self, which: str, rows: int) -> str:
        """Operand precision of a pass whose GEMMs have `rows` rows ("auto" resolves by rows)."""
        p = self.precision[which]
        if p == "auto":
            return "fp8" if rows >= self.auto_min_rows else "bf16"
        return p

    def _set_pass(self, sess: Session, which: str, rows: Optional[int] = None) -> None:
        p = self.effective_precision(which, sess.x.shape[0] if rows is None else rows)
        sess.extra["pass_precision"] = (which, p)
        self._fp4 = p == "nvfp4"
        self._fp8 = p in ("fp8", "nvfp4")
        if self._fp8:
            self._ensure_fp8_scratch(sess)

    # -------------------------------------------------------------- sessions
    def new_session(self, B: int, H: int, W: int) -> Session:
        c, dev = self.cfg, self.device
        p = c.patch_size
        gh, gw = H // p, W // p
        P = gh * gw
        N = P + c.n_prefix
        D, L, Hd = c.embed_dim, c.depth, c.ffn_hidden
        M = B * N

        def e(*shape, dtype=BF16):
            return torch.empty(*shape, device=dev, dtype=dtype)

        patch_rows = (torch.arange(B, device=dev)[:, None] * N + c.n_prefix + torch.arange(P, device=dev)[None, :])
        T = c.n_prefix + P
        order = None
        if c.window_size > 0:
            if c.n_prefix or gh % c.window_size or gw % c.window_size:
                raise ValueError("windowed towers need no prefix tokens and a grid that tiles into windows")
            from .qwen25vl import window_order

            order = window_order(gh, gw, c.window_size, 1).to(device=dev, dtype=torch.int32)
        sess = Session(
            B=B, img_hw=(H, W), grid_hw=(gh, gw), N=N, P=P,
            x_in=e(M, D), x=e(M, D), x_tmp=e(M, D), xn=e(M, D), q=e(M, self.A), o=e(M, self.A), h=e(M, Hd),
            kc=e(L, M, self.A), vc=e(L, M, self.A), bos=e(L, M, D), pscore=torch.zeros(L, B, N, device=dev),
            ps_scratch=e(B, c.num_heads, N, dtype=torch.float32),
            cols=torch.zeros(B * P, self.w.patch_w.shape[1], device=dev, dtype=BF16),
            patch_rows=patch_rows.reshape(-1).to(torch.int32).contiguous(),
            rope=self._rope_global(gh, gw, order),
            upd=torch.zeros(B, T, device=dev, dtype=torch.int32), rows=torch.zeros(B * T, device=dev, dtype=torch.int32),
            x_act=e(B * T, D), x_att=e(B * T, D), plan_stats=torch.zeros(B, 2, device=dev),
            stat_acc=torch.zeros(5, device=dev))
        if order is not None:
            ws = c.window_size
            sess.extra["order"] = order.contiguous()
            sess.extra["n_windows"] = (gh // ws) * (gw // ws)
            if self.w.periods is not None:
                sw, cw = rope_tables(c, self.w.periods, ws, ws)
                reps = (gh // ws) * (gw // ws)
                sess.extra["rope_win"] = (sw.repeat(reps, 1).contiguous(), cw.repeat(reps, 1).contiguous())
        return sess

    def _rope_global(self, gh: int, gw: int, order: Optional[torch.Tensor]):
        if self.w.periods is None:
            return None
        s, c = rope_tables(self.cfg, self.w.periods, gh, gw)
        if order is not None:  # tables follow the token order
            s, c = s[order.long()].contiguous(), c[order.long()].contiguous()
        return s, c

    def _windowed(self, l: int) -> bool:
        return self.cfg.window_size > 0 and l not in self.cfg.global_layers

    def _rope(self, sess: Session, l: int):
        if self._windowed(l) or (self.cfg.window_size > 0 and self.cfg.window_rope_everywhere):
            return sess.extra.get("rope_win", sess.rope)
        return sess.rope

    # -------------------------------------------------------------- tokens
    # -------------------------------------------------------------- CUDA-graph replay of passes
    # Whole approximate / correction passes are launch-bound on the host when run eagerly (about
    # 850 launches per ViT-7B request). A session's buffers are static, so a pass whose inputs all
    # live in them is captured once and replayed: the first call of a key runs eagerly (it creates
    # the lazily allocated buffers), the second is captured and replayed, later calls replay.
    # The Python-side effects of the captured call (session attributes, `extra` entries set or
    # removed, the engine's pass-precision flags, the launch counter) are recorded and re-applied
    # on every replay. APPCORR_ENGINE_GRAPHS=0 turns this off.
    graphs_enabled = os.environ.get("APPCORR_ENGINE_GRAPHS", "1") != "0"
    _GRAPH_ENGINE_ATTRS = ("_fp4", "_fp8")

    def run_graphed(self, sess: Session, key, fn):
        """fn() with every launch on the current stream and every input in `sess`'s buffers (or in
        tensors that stay alive and unchanged while `key` is in use, such as cached index maps).
        The caller puts whatever fn depends on into `key`."""
        if (not self.graphs_enabled or self.device.type != "cuda" or
                torch.cuda.is_current_stream_capturing()):
            return fn()
        cache = sess.__dict__.setdefault("_graphs", {})
        ent = cache.get(key)
        if ent is None or ent == "eager":
            if ent is None:
                cache[key] = "warm"
            return fn()
        if ent == "warm":
            snap = self._py_state(sess)
            n0 = K.LAUNCHES[0]
            g = torch.cuda.CUDAGraph()
            try:
                # thread-local: the server's decoder and reaper threads keep using the GPU
                # (their own streams, host reads) while the launcher thread captures
                with torch.cuda.graph(g, capture_error_mode="thread_local"):
                    out = fn()
            except RuntimeError:  # something in fn cannot be captured: this key stays eager
                cache[key] = "eager"
                K.LAUNCHES[0] = n0
                self._py_apply(([(o, a, e, [k for k in o.extra if k not in e]) for o, a, e in snap[0]], snap[1]))
                torch.cuda.synchronize()
                return fn()
            delta = self._py_delta(snap), K.LAUNCHES[0] - n0
            cache[key] = (g, out, delta)
            g.replay()
            return out
        g, out, (delta, launches) = ent
        self._py_apply(delta)
        K.LAUNCHES[0] += launches
        g.replay()
        return out

    def _py_state(self, sess: Session):
        objs = [sess] + list(sess.extra.get("subs") or [])
        return ([(o, {k: v for k, v in vars(o).items() if k not in ("extra", "_graphs")}, dict(o.extra)) for o in objs],
                {a: getattr(self, a, None) for a in self._GRAPH_ENGINE_ATTRS})

    def _py_delta(self, snap):
        objs, eng0 = snap
        out = []
        for o, attrs0, extra0 in objs:
            attrs = {k: v for k, v in vars(o).items() if k not in ("extra", "_graphs") and attrs0.get(k, _MISSING) is not v}
            ext = {k: v for k, v in o.extra.items() if extra0.get(k, _MISSING) is not v}
            gone = [k for k in extra0 if k not in o.extra]
            out.append((o, attrs, ext, gone))
        return out, {a: getattr(self, a, None) for a in self._GRAPH_ENGINE_ATTRS}

    def _py_apply(self, delta) -> None:
        objs, eng = delta
        for o, attrs, ext, gone in objs:
            for k, v in attrs.items():
                setattr(o, k, v)
            for k in gone:
                o.extra.pop(k, None)
            o.extra.update(ext)
        for a, v in eng.items():
            setattr(self, a, v)

    def prepare_tokens(self, sess: Session, img: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """uint8 [B, H, W, 3] image -> tokens [B*N, D] (CLS + storage + patch embeddings)."""
        c = self.cfg
        out = sess.x_in if out is None else out
        K.patch_im2col(img, c.patch_size, sess.cols, mean=self.w.pixel_mean, std=self.w.pixel_std,
                       perm=sess.extra.get("order"))
        K.gemm(sess.cols, self.w.patch_w, out, bias=self.w.patch_b, out_rows=sess.patch_rows)
        K.set_prefix(out, self.w.prefix, sess.B, sess.N)
        if self.w.pos_embed is not None:
            rep = sess.extra.get("pos_rep")
            if rep is None:
                if self.w.pos_embed.shape[0] != sess.N:
                    raise ValueError(f"learned position embedding has {self.w.pos_embed.shape[0]} rows, "
                                     f"the image has {sess.N} tokens")
                rep = sess.extra["pos_rep"] = self.w.pos_embed.repeat(sess.B, 1).contiguous()
            K.add_(out, rep)
        if self.w.pre_norm_w is not None:  # row-wise in place: each row is read before it is written
            K.layernorm(out, self.w.pre_norm_w, self.w.pre_norm_b, c.norm_eps, out)
        return out

    # -------------------------------------------------------------- approximate pass
    def _mlp(self, lw: LayerW, xin: torch.Tensor, hbuf: torch.Tensor, a_scale=None) -> torch.Tensor:
        w, ws = self._w(lw, "fc1")
        epi = K.EPI_SWIGLU if self.cfg.is_swiglu else K.EPI_GELU
        K.gemm(xin, w, hbuf, epi=epi, bias=self._fc1_bias(lw), a_scale=a_scale, b_scale=ws,
               bn=K.fp4_tile("fc1") if self._fp4 else None)
        return hbuf

    def approx_layer(self, sess: Session, l: int, x: torch.Tensor, x_out: torch.Tensor, server_pscore: str) -> None:
        c, lw = self.cfg, self.w.layers[l]
        B, N, H, Dh = sess.B, sess.N, c.num_heads, self.Dh
        a, sa = self._norm(sess, x, lw.norm1_w, lw.norm1_b, sess.xn)
        w, ws = self._w(lw, "qkv")
        K.qkv_gemm(a, w, lw.qkv_b, sess.q, sess.kc[l], sess.vc[l], head_dim=Dh, seq_len=N,
                   rope=self._rope(sess, l), n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        if self._windowed(l):  # windows are contiguous token runs: a batched attention over windows
            nw = sess.extra["n_windows"]
            K.attention(sess.q, sess.kc[l], sess.vc[l], sess.o, B=B * nw, Tq=N // nw, Tk=N // nw, H=H, Dh=Dh,
                        scale=self.attn_scale)
        else:
            self._attention_with_score(sess, l, H, server_pscore, sess.pscore[l])
        # x_out = x + ls1 * proj(o); bos[l] = ls1 * proj(o)
        a, sa = self._act(sess, sess.o, "proj")
        w, ws = self._w(lw, "proj")
        K.gemm(a, w, x_out, epi=K.EPI_RESID, bias=lw.proj_b, gamma=lw.ls1, resid=x,
               aux=sess.bos[l], aux_mode=K.AUX_SET, a_scale=sa, b_scale=ws)
        a, sa = self._norm(sess, x_out, lw.norm2_w, lw.norm2_b, sess.xn)
        self._mlp(lw, a, sess.h, sa)
        # x_out += ls2 * mlp (in place: each output element reads only its own residual); bos[l] += same
        a, sa = self._act(sess, sess.h)
        w, ws = self._w(lw, "fc2")
        K.gemm(a, w, x_out, epi=K.EPI_RESID, bias=lw.fc2_b, gamma=lw.ls2, resid=x_out,
               aux=sess.bos[l], aux_mode=K.AUX_ADD, a_scale=sa, b_scale=ws, bn=K.fp4_tile("fc2") if self._fp4 else None)

    def _attention_with_score(self, sess: Session, l: int, H: int, kind: str, score_out: torch.Tensor) -> None:
        """Full attention of layer l over H (local) heads, plus the server patch score `kind`
        averaged over those heads into score_out [B, N] (reference attention.py:241-274):
          cls_attn_prob*    the CLS softmax row, written by the same attention pass
          patch_attn_prob*  column means of the probabilities: the attention pass also writes the
                            row LSE, then one tcgen05 Q K^T pass sums exp(s - lse) per key
          patch_pseudo*     softmax row of one pseudo query per (image, head)
          none / disabled / random: no score from the attention (random draws at correction)."""
        B, N, Dh, sc = sess.B, sess.N, self.Dh, self.attn_scale
        kind = _score_kind(kind)
        if kind == "cls" and self.cfg.n_prefix == 0:
            kind = "none"  # no CLS token to score with
        if kind == "cls":
            fused = K.ATTENTION_IMPL[0].startswith("tcgen05")
            if not fused:
                K.cls_attn_pscore(sess.q, sess.kc[l], B=B, N=N, H=H, Dh=Dh, scratch=sess.ps_scratch, out=score_out,
                                  scale=sc)
            K.attention(sess.q, sess.kc[l], sess.vc[l], sess.o, B=B, Tq=N, Tk=N, H=H, Dh=Dh, scale=sc,
                        cls_probs=sess.ps_scratch if fused else None)
            if fused:
                K.head_mean(sess.ps_scratch, B, H, N, score_out)
            return
        if kind == "patch":
            lse = sess.extra.get("lse")
            if lse is None:
                lse = sess.extra["lse"] = torch.empty(B, H, N, device=self.device, dtype=torch.float32)
            K.attention(sess.q, sess.kc[l], sess.vc[l], sess.o, B=B, Tq=N, Tk=N, H=H, Dh=Dh, lse=lse,
                        scale=sc)
            K.attn_colsum_pscore(sess.q, sess.kc[l], lse, B=B, N=N, H=H, Dh=Dh, probs=sess.ps_scratch, out=score_out,
                                 scale=sc)
            return
        if kind == "pseudo":
            pq = sess.extra.get("pseudo_q")
            if pq is None:
                pq = sess.extra["pseudo_q"] = torch.empty(B, H * Dh, device=self.device, dtype=BF16)
            K.pseudo_query(sess.q, B=B, N=N, npre=self.cfg.n_prefix, H=H, Dh=Dh, out=pq)
            K.query_attn_pscore(pq, sess.kc[l], B=B, N=N, H=H, Dh=Dh, scratch=sess.ps_scratch, out=score_out,
                                scale=sc)
        K.attention(sess.q, sess.kc[l], sess.vc[l], sess.o, B=B, Tq=N, Tk=N, H=H, Dh=Dh, scale=sc)

    def approx(self, sess: Session, start: int, end: int, server_pscore: str = "cls_attn_prob") -> torch.Tensor:
        """Approximate pass over layers [start, end) on the running features."""
        if start == 0:
            sess.x.copy_(sess.x_in)
            sess.extra.pop("layermean", None)  # a new request's approximate pass
            sess.extra.pop("random_score", None)
        self._set_pass(sess, "approx")
        for l in range(start, end):
            self.approx_layer(sess, l, sess.x, sess.x, server_pscore)
            self._tap(sess, l)
        sess.approx_done = max(sess.approx_done, end)
        return sess.x

    def _tap(self, sess: Session, l: int) -> None:
        """Keep the running features after layer l when l is a tap layer (dense heads read them)."""
        if l in self.taps:
            t = sess.extra.get(f"tap{l}")
            if t is None:
                t = sess.extra[f"tap{l}"] = torch.empty_like(sess.x)
            t.copy_(sess.x)

    def tap_features(self, sess: Session, l: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Final-norm patch tokens of tap layer l -> [B*P, D] (DINOv3 intermediate layers, norm=True)."""
        c = self.cfg
        if out is None:
            out = torch.empty(sess.B * sess.P, c.embed_dim, device=self.device, dtype=BF16)
        K.layernorm(sess.extra[f"tap{l}"], self.w.norm_w, self.w.norm_b, c.norm_eps, out, rows=sess.patch_rows)
        return out

    # -------------------------------------------------------------- correction pass
    def plan(self, sess: Session, l: int, pre: torch.Tensor, cand: torch.Tensor, k: int, opts: Dict,
             mobile: Optional[torch.Tensor] = None, valid: Optional[torch.Tensor] = None,
             server: Optional[torch.Tensor] = None, thres: Optional[float] = None,
             dynamic: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
        """Packed plan of layer l (block.py:360-560). Top-k: the k best candidates. Threshold
        (`thres`): candidates scoring >= thres, at most k of them (the cap), padded with the last
        kept one. dynamic: threshold without a cap; the plan is built at the full width, then one
        host read of the largest kept count sizes it (the reference's builder syncs likewise)."""
        B = sess.B
        T = pre.shape[1] + k
        upd = sess.upd.view(-1)[: B * T].view(B, T)
        rows = sess.rows[: B * T]
        if server is None:
            server = sess.pscore[l]
        sess.extra["plan_id"] = sess.extra.get("plan_id", 0) + 1
        counts = None
        if dynamic:
            counts = sess.extra.get("plan_counts")
            if counts is None:
                counts = sess.extra["plan_counts"] = torch.zeros(B, device=self.device, dtype=torch.int32)
        K.correction_plan(server, pre, cand, k, upd, rows, mobile=mobile, ws=float(opts.get("server_pscore_weight", 1.0)),
                          wm=float(opts.get("mobile_pscore_weight", 0.0)), fusion=opts.get("pscore_fusion", "add"),
                          valid=valid, stats=sess.plan_stats, thres=thres, counts=counts)
        if dynamic:
            kmax = min(int(counts.max().item()), k)
            T2 = pre.shape[1] + kmax
            u2 = sess.extra.get("upd_dyn")
            if u2 is None or u2.numel() < sess.upd.numel():
                u2 = sess.extra["upd_dyn"] = torch.empty_like(sess.upd)
                sess.extra["rows_dyn"] = torch.empty_like(sess.rows)
            upd2 = u2.view(-1)[: B * T2].view(B, T2)
            upd2.copy_(upd[:, :T2])
            rows2 = sess.extra["rows_dyn"][: B * T2]
            rows2.view(B, T2).copy_(rows.view(B, T)[:, :T2])
            return upd2, rows2
        return upd, rows

    def _window_bounds(self, sess: Session, upd: torch.Tensor):
        """Per packed query: first and last key of its window (cached per plan)."""
        key = upd.data_ptr(), upd.shape[1], sess.extra.get("plan_id", 0)
        wb = sess.extra.get("win_bounds")
        if wb is None or wb[0] != key:
            tw = self.cfg.window_size ** 2
            lo = (upd.view(-1) // tw * tw).to(torch.int32).contiguous()
            wb = sess.extra["win_bounds"] = (key, lo, (lo + tw - 1).contiguous())
        return wb[1], wb[2]

    def correct_layer(self, sess: Session, l: int, x: torch.Tensor, upd: torch.Tensor, rows: torch.Tensor) -> None:
        c, lw = self.cfg, self.w.layers[l]
        B, N, H, Dh = sess.B, sess.N, c.num_heads, self.Dh
        T = upd.shape[1]
        MT = B * T
        x_act, x_att = sess.x_act[:MT], sess.x_att[:MT]
        xn = sess.xn[:MT]
        q, o, h = sess.q[:MT], sess.o[:MT], sess.h[:MT]
        a, sa = self._norm(sess, x, lw.norm1_w, lw.norm1_b, xn, rows=rows, copy_out=x_act)
        K.add_(x, sess.bos[l])
        w, ws = self._w(lw, "qkv")
        K.qkv_gemm(a, w, lw.qkv_b, q, sess.kc[l], sess.vc[l], head_dim=Dh, tok_idx=upd.view(-1),
                   kv_rows=rows, rope=self._rope(sess, l), n_prefix=c.n_prefix, a_scale=sa, b_scale=ws)
        if self._windowed(l):  # each kept query attends its own window's keys
            lo, hi = self._window_bounds(sess, upd)
            K.attention(q, sess.kc[l], sess.vc[l], o, B=B, Tq=T, Tk=N, H=H, Dh=Dh, causal=True, q_pos=hi, q_lo=lo,
                        scale=self.attn_scale)
        else:
            K.attention(q, sess.kc[l], sess.vc[l], o, B=B, Tq=T, Tk=N, H=H, Dh=Dh, scale=self.attn_scale)
        a, sa = self._act(sess, o, "proj")
        w, ws = self._w(lw, "proj")
        K.gemm(a, w, x_att, epi=K.EPI_RESID, bias=lw.proj_b, gamma=lw.ls1, resid=x_act, a_scale=sa, b_scale=ws)
        a, sa = self._norm(sess, x_att, lw.norm2_w, lw.norm2_b, xn)
        self._mlp(lw, a, h, sa)
        # x[rows] = x_att + ls2 * mlp; bos[l][rows] = (x_att - x_act) + ls2 * mlp
        a, sa = self._act(sess, h)
        w, ws = self._w(lw, "fc2")
        K.gemm(a, w, x, epi=K.EPI_RESID, bias=lw.fc2_b, gamma=lw.ls2, resid=x_att, out_rows=rows,
               aux=sess.bos[l], aux_mode=K.AUX_OUT_MINUS, resid2=x_act, a_scale=sa, b_scale=ws,
               bn=K.fp4_tile("fc2") if self._fp4 else None)

    def correct(self, sess: Session, start: int, end: int, pre: torch.Tensor, cand: torch.Tensor, opts: Dict,
                mobile: Optional[torch.Tensor] = None, valid: Optional[torch.Tensor] = None,
                server: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Correction pass over layers [start, end) starting from the fresh tokens `sess.x_in`.

        pre: int32 [B, n_prefix] prefix token indices; cand: int32 [B, P_g] candidate patch tokens
        (the residual group that just arrived). Keeps k = int(P_g * token_keep_ratio) per image.
        """
        st = self._correct_begin(sess, start, cand, opts, pre)
        if server is not None:  # caller-provided per-token score [B, N], one plan for every layer
            st["shared"] = server
        for l in range(start, end):
            self._correct_step(sess, l, st, pre, cand, opts, mobile, valid)
        return sess.x

    def _correct_begin(self, sess: Session, start: int, cand: torch.Tensor, opts: Dict,
                       pre: Optional[torch.Tensor] = None) -> Dict:
        P_g = cand.shape[1]
        ratio = float(opts.get("token_keep_ratio", 0.2))
        thres = opts.get("token_keep_thres")
        cap = int(opts.get("token_keep_cap", 0) or 0)
        kind = str(opts.get("server_pscore", "cls_attn_prob"))
        if start == 0:
            if opts.get("token_prune_enabled") and pre is not None:
                # prune state of this correction segment from the drift between the running
                # features and the fresh tokens (vision_transformer.py:453-489); like the
                # reference, the correction itself does not consume it
                dind = torch.cat([pre, cand], dim=1).to(torch.int32).contiguous()
                sess.extra["prune_state"] = K.token_prune(
                    sess.x, sess.x_in, sess.N, dind, pre.shape[1], float(opts.get("token_prune_threshold", 0.0)),
                    int(opts.get("token_prune_min_keep", 1)))
            sess.x.copy_(sess.x_in)
        k_rows = P_g if thres is not None and cap <= 0 else (min(cap, P_g) if thres is not None else
                                                             min(int(P_g * ratio), P_g))
        self._set_pass(sess, "correct", rows=sess.B * (self.cfg.n_prefix + k_rows))
        shared = None
        _score_kind(kind)  # unknown names raise
        if kind == "random":  # one random score per request, shared by every layer
            shared = sess.extra.get("random_score")
            if shared is None:
                # a generator of the engine's own, consumed in the same order on every
                # tensor-parallel rank, so all ranks draw the same scores
                if getattr(self, "_rand_gen", None) is None:
                    self._rand_gen = torch.Generator(device=self.device)
                    self._rand_gen.manual_seed(0)
                shared = sess.extra["random_score"] = torch.rand(sess.B, sess.N, device=self.device,
                                                                 generator=self._rand_gen)
        elif kind in LAYERMEAN_SERVER_PSCORES:
            shared = sess.extra.get("layermean")
            if shared is None:  # mean over the approximate pass's layers, computed once per request
                shared = sess.pscore[: max(sess.approx_done, 1)].mean(0)
                sess.extra["layermean"] = shared
        if thres is not None:  # threshold selection: width = the cap, or dynamic (one host read)
            k = min(cap, P_g) if cap > 0 else P_g
            return {"k": k, "shared": shared, "upd": None, "rows": None, "thres": float(thres),
                    "dynamic": cap <= 0}
        return {"k": min(int(P_g * ratio), P_g), "shared": shared, "upd": None, "rows": None, "thres": None,
                "dynamic": False}

    def _correct_step(self, sess: Session, l: int, st: Dict, pre, cand, opts, mobile, valid) -> None:
        if st["upd"] is None or st["shared"] is None:
            st["upd"], st["rows"] = self.plan(sess, l, pre, cand, st["k"], opts, mobile=mobile, valid=valid,
                                              server=st["shared"], thres=st.get("thres"),
                                              dynamic=st.get("dynamic", False))
        self.correct_layer(sess, l, sess.x, st["upd"], st["rows"])
        self._tap(sess, l)

    # -------------------------------------------------------------- outputs
    def normed_tokens(self, sess: Session) -> torch.Tensor:
        """Final LayerNorm of every token (CLS, storage and patch) -> [B*N, D]."""
        c = self.cfg
        buf = sess.extra.get("normed")
        if buf is None:
            buf = sess.extra["normed"] = torch.empty_like(sess.x)
        K.layernorm(sess.x, self.w.norm_w, self.w.norm_b, c.norm_eps, buf)
        return buf

    def patch_features(self, sess: Session, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Final LayerNorm of the patch tokens -> [B*P, D]."""
        c = self.cfg
        if out is None:
            out = sess.extra.get("patch_feat")
            if out is None:
                out = torch.empty(sess.B * sess.P, c.embed_dim, device=self.device, dtype=BF16)
                sess.extra["patch_feat"] = out
        K.layernorm(sess.x, self.w.norm_w, self.w.norm_b, c.norm_eps, out, rows=sess.patch_rows)
        return out
