"""Qwen2.5-VL-shaped vision-language model: fp32 reference modules and the sm_100a engine.

Reference: appcorr/models/qwen25vl/llm/decoder_layer.py (approx :207-215, correct :217-245,
attention approx :97-116 and correct :118-186 with the KV-cache rewrite at :157-159) and
offload/server/model/qwen25vl_executor.py:33-339 (splice of the image embeddings :139-146,
correction round :174-250, first-token head :252-286).

Model
    vision tower: 14x14 patches (the two temporal copies of a still image folded into one
    588-wide patch embedding), `vis_depth` pre-RMSNorm blocks (2-D RoPE, SwiGLU MLP), windowed
    attention over 8x8-patch windows except at `full_attn_layers`, then a 2x2 patch merger
    (RMSNorm -> Linear -> GELU -> Linear) to the LLM width.
    LLM: `depth` pre-RMSNorm decoder layers, grouped-query causal attention with M-RoPE (the
    rotary frequencies split into temporal / height / width sections), SwiGLU MLP, final RMSNorm
    and an LM head.

Approximate / correct semantics (LLM, as in the reference decoder layer)
    approx(x):  a = attn(norm1(x)) [K/V cached], m = mlp(norm2(x + a)); inc := a + m; x + a + m
    correct(x, rows): x_out = x + inc for every row; the rows in `rows` are recomputed from x with
        their K/V rewritten in the cache and a causal mask per query position; inc is unchanged.

Token order inside the vision tower is window-major (all 64 patches of an 8x8 window are
contiguous, and inside a window every 2x2 merge unit is contiguous), so windowed attention is
a batched attention over windows and the merger is a free reshape. Positions (RoPE) follow the
patch's (row, col), so the order does not change the math.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn

CLIP_MEAN = (0.48145466, 0.4578275, 0.40821073)
CLIP_STD = (0.26862954, 0.26130258, 0.27577711)


@dataclass
class Qwen25VLConfig:
    # LLM
    hidden: int = 3584
    depth: int = 28
    heads: int = 28
    kv_heads: int = 4
    head_dim: int = 128
    ffn: int = 18944
    vocab: int = 152064
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    mrope_section: Tuple[int, int, int] = (16, 24, 24)
    # vision tower
    vis_hidden: int = 1280
    vis_depth: int = 32
    vis_heads: int = 16
    vis_head_dim: int = 80
    vis_ffn: int = 3420
    patch: int = 14
    merge: int = 2
    window: int = 8                       # patches per window side (112 px)
    full_attn_layers: Tuple[int, ...] = (7, 15, 23, 31)
    vis_rope_theta: float = 10000.0

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads


PRESETS: Dict[str, Qwen25VLConfig] = {
    "qwen25vl7b": Qwen25VLConfig(),
    "tiny": Qwen25VLConfig(hidden=256, depth=2, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                           vis_hidden=128, vis_depth=2, vis_heads=2, vis_head_dim=40, vis_ffn=200,
                           full_attn_layers=(1,)),
}


# ----------------------------------------------------------------------------- positions
def window_order(gh: int, gw: int, window: int, merge: int) -> torch.Tensor:
    """Row-major patch index of every vision token, in the tower's window-major order."""
    assert gh % window == 0 and gw % window == 0 and window % merge == 0
    idx = torch.arange(gh * gw).view(gh // window, window // merge, merge, gw // window, window // merge, merge)
    # (wy, my, dy, wx, mx, dx) -> (wy, wx, my, mx, dy, dx)
    return idx.permute(0, 3, 1, 4, 2, 5).reshape(-1)


def vision_rope(cfg: Qwen25VLConfig, gh: int, gw: int, order: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """2-D rotary angles per vision token (tower order): [T, vis_head_dim] sin / cos whose second
    half repeats the first (rotate-half layout). Half the rotary frequencies follow the row,
    half the column."""
    d = cfg.vis_head_dim // 2          # rotary pairs
    inv = 1.0 / (cfg.vis_rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))  # d/2 freqs
    ys, xs = order // gw, order % gw
    ang = torch.cat([ys[:, None].double() * inv[None], xs[:, None].double() * inv[None]], dim=1)  # [T, d]
    ang = torch.cat([ang, ang], dim=1)
    return ang.sin().float(), ang.cos().float()


def mrope_positions(n_before: int, gh_m: int, gw_m: int, n_after: int) -> torch.Tensor:
    """[3, N] (temporal, height, width) positions of [text | image (gh_m x gw_m merged) | text]:
    text advances all three together; image tokens share the temporal index and use their row /
    column offsets; text after the image restarts at max + 1 (the reference get_rope_index rule)."""
    pos = []
    t = torch.arange(n_before)
    pos.append(torch.stack([t, t, t]))
    s = n_before
    yy, xx = torch.meshgrid(torch.arange(gh_m), torch.arange(gw_m), indexing="ij")
    pos.append(torch.stack([torch.full((gh_m * gw_m,), s), s + yy.reshape(-1), s + xx.reshape(-1)]))
    nxt = s + max(gh_m, gw_m)
    t = torch.arange(n_after) + nxt
    pos.append(torch.stack([t, t, t]))
    return torch.cat(pos, dim=1)


def mrope_tables(cfg: Qwen25VLConfig, pos: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """M-RoPE sin / cos [N, head_dim]: frequency i uses the temporal / height / width position of
    its section; the second half repeats the first."""
    half = cfg.head_dim // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, dtype=torch.float64) / cfg.head_dim))  # [half]
    sec = torch.zeros(half, dtype=torch.long)
    a, b, _ = cfg.mrope_section
    sec[a:a + b] = 1
    sec[a + b:] = 2
    p = pos.double()[sec]                      # [half, N]
    ang = (p * inv[:, None]).T                 # [N, half]
    ang = torch.cat([ang, ang], dim=1)
    return ang.sin().float(), ang.cos().float()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


# ----------------------------------------------------------------------------- fp32 modules
class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight


class SwiGLU(nn.Module):
    def __init__(self, d: int, h: int, bias: bool):
        super().__init__()
        self.gate_proj, self.up_proj = nn.Linear(d, h, bias=bias), nn.Linear(d, h, bias=bias)
        self.down_proj = nn.Linear(h, d, bias=bias)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class VisionBlock(nn.Module):
    def __init__(self, cfg: Qwen25VLConfig):
        super().__init__()
        d = cfg.vis_hidden
        self.cfg = cfg
        self.norm1, self.norm2 = RMSNorm(d), RMSNorm(d)
        self.qkv = nn.Linear(d, 3 * cfg.vis_heads * cfg.vis_head_dim)
        self.proj = nn.Linear(cfg.vis_heads * cfg.vis_head_dim, d)
        self.mlp = SwiGLU(d, cfg.vis_ffn, bias=True)

    def _qkv(self, x, sin, cos):
        c = self.cfg
        n = x.shape[0]
        q, k, v = self.qkv(self.norm1(x)).view(n, 3, c.vis_heads, c.vis_head_dim).unbind(1)
        return q * cos[:, None] + rotate_half(q) * sin[:, None], k * cos[:, None] + rotate_half(k) * sin[:, None], v

    def approx(self, x, sin, cos, windows: int, cache: Dict, tag: str):
        """forward(), keeping this block's (rotated) keys and values for later corrections."""
        _, k, v = self._qkv(x, sin, cos)
        cache[f"{tag}_k"], cache[f"{tag}_v"] = k, v
        return self.forward(x, sin, cos, windows)

    def correct(self, xs, rows: torch.Tensor, sin, cos, windows: int, cache: Dict, tag: str):
        """Corrected tokens only: xs [n, d] are the rows `rows` (tower order) on their new
        trajectory; their keys / values replace the cached ones, the other tokens' stay as cached,
        and each corrected token attends within its window (or to every token when windows == 1)."""
        c = self.cfg
        T = cache[f"{tag}_k"].shape[0]
        q, k, v = self._qkv(xs, sin[rows], cos[rows])
        cache[f"{tag}_k"] = cache[f"{tag}_k"].index_copy(0, rows, k)
        cache[f"{tag}_v"] = cache[f"{tag}_v"].index_copy(0, rows, v)
        kk, vv = cache[f"{tag}_k"].transpose(0, 1), cache[f"{tag}_v"].transpose(0, 1)  # [heads, T, dh]
        w = T // windows
        keys = torch.arange(T, device=xs.device)
        mask = (keys[None] // w) == (rows[:, None] // w)                   # [n, T]
        o = F.scaled_dot_product_attention(q.transpose(0, 1), kk, vv, attn_mask=mask[None])
        xs = xs + self.proj(o.transpose(0, 1).reshape(xs.shape[0], -1))
        return xs + self.mlp(self.norm2(xs))

    def forward(self, x, sin, cos, windows: int):
        """x: [T, d] in window-major order; windows: number of equal attention windows (1 = full)."""
        c = self.cfg
        T = x.shape[0]
        q, k, v = self._qkv(x, sin, cos)
        w = T // windows
        q, k, v = (t.view(windows, w, c.vis_heads, c.vis_head_dim).transpose(1, 2) for t in (q, k, v))
        o = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(T, -1)
        x = x + self.proj(o)
        return x + self.mlp(self.norm2(x))


class Merger(nn.Module):
    def __init__(self, cfg: Qwen25VLConfig):
        super().__init__()
        d4 = cfg.vis_hidden * cfg.merge ** 2
        self.ln_q = RMSNorm(cfg.vis_hidden)
        self.fc1, self.fc2 = nn.Linear(d4, d4), nn.Linear(d4, cfg.hidden)

    def forward(self, x):
        x = self.ln_q(x).reshape(-1, self.fc1.in_features)
        return self.fc2(F.gelu(self.fc1(x)))


class VisionTower(nn.Module):
    def __init__(self, cfg: Qwen25VLConfig):
        super().__init__()
        self.cfg = cfg
        self.patch_embed = nn.Linear(3 * cfg.patch ** 2, cfg.vis_hidden, bias=False)
        self.blocks = nn.ModuleList([VisionBlock(cfg) for _ in range(cfg.vis_depth)])
        self.merger = Merger(cfg)

    def _tokens(self, img_u8: torch.Tensor):
        """-> patch rows in tower order, rotary tables, window count."""
        c = self.cfg
        H, W = img_u8.shape[:2]
        gh, gw = H // c.patch, W // c.patch
        x = (img_u8.float() / 255 - torch.tensor(CLIP_MEAN, device=img_u8.device)) / torch.tensor(CLIP_STD, device=img_u8.device)
        cols = x.view(gh, c.patch, gw, c.patch, 3).permute(0, 2, 4, 1, 3).reshape(gh * gw, -1)
        order = window_order(gh, gw, c.window, c.merge).to(img_u8.device)
        sin, cos = (t.to(img_u8.device) for t in vision_rope(c, gh, gw, order.cpu()))
        return cols[order], sin, cos, (gh // c.window) * (gw // c.window), (gh, gw)

    def forward(self, img_u8: torch.Tensor, cache: Optional[Dict] = None) -> torch.Tensor:
        """uint8 [H, W, 3] -> merged image embeddings [(H/28)*(W/28), hidden] in raster order of
        merge units (window-major inside the tower, restored to raster order on output). With a
        `cache`, every block keeps its keys / values for `correct`."""
        c = self.cfg
        cols, sin, cos, nwin, (gh, gw) = self._tokens(img_u8)
        h = self.patch_embed(cols)
        for i, blk in enumerate(self.blocks):
            win = 1 if i in c.full_attn_layers else nwin
            h = blk(h, sin, cos, win) if cache is None else blk.approx(h, sin, cos, win, cache, f"v{i}")
        emb = self.merger(h)
        return emb[merge_raster_index(c, gh, gw).to(emb.device)]

    def correct(self, img_u8: torch.Tensor, units: torch.Tensor, cache: Dict) -> torch.Tensor:
        """Partial tower correction: only the merge units `units` (tower order) are recomputed
        from the new image, through every block, against the cached keys / values of the other
        tokens; -> their merged embeddings [len(units), hidden] (in the order of `units`)."""
        c = self.cfg
        g = c.merge ** 2
        cols, sin, cos, nwin, _ = self._tokens(img_u8)
        rows = (units[:, None] * g + torch.arange(g, device=units.device)[None]).reshape(-1)
        h = self.patch_embed(cols[rows])
        for i, blk in enumerate(self.blocks):
            h = blk.correct(h, rows, sin, cos, 1 if i in c.full_attn_layers else nwin, cache, f"v{i}")
        return self.merger(h)


def merge_unit_raster(cfg: Qwen25VLConfig, gh: int, gw: int) -> torch.Tensor:
    """For each merge unit in the tower's window-major order, its raster index."""
    order = window_order(gh, gw, cfg.window, cfg.merge)
    unit = order[:: cfg.merge ** 2]                      # first patch of every merge unit (tower order)
    ys, xs = (unit // gw) // cfg.merge, (unit % gw) // cfg.merge
    return ys * (gw // cfg.merge) + xs


def merge_raster_index(cfg: Qwen25VLConfig, gh: int, gw: int) -> torch.Tensor:
    """For each merge unit in raster order, its index in the tower's window-major order."""
    raster = merge_unit_raster(cfg, gh, gw)
    inv = torch.empty_like(raster)
    inv[raster] = torch.arange(raster.numel())
    return inv


class DecoderLayer(nn.Module):
    def __init__(self, cfg: Qwen25VLConfig):
        super().__init__()
        self.cfg = cfg
        d = cfg.hidden
        self.input_layernorm, self.post_attention_layernorm = RMSNorm(d, cfg.rms_eps), RMSNorm(d, cfg.rms_eps)
        self.q_proj = nn.Linear(d, cfg.heads * cfg.head_dim)
        self.k_proj = nn.Linear(d, cfg.kv_heads * cfg.head_dim)
        self.v_proj = nn.Linear(d, cfg.kv_heads * cfg.head_dim)
        self.o_proj = nn.Linear(cfg.heads * cfg.head_dim, d, bias=False)
        self.mlp = SwiGLU(d, cfg.ffn, bias=False)

    def _qkv(self, x, sin, cos):
        c = self.cfg
        T = x.shape[0]
        q = self.q_proj(x).view(T, c.heads, c.head_dim)
        k = self.k_proj(x).view(T, c.kv_heads, c.head_dim)
        v = self.v_proj(x).view(T, c.kv_heads, c.head_dim)
        q = q * cos[:, None] + rotate_half(q) * sin[:, None]
        k = k * cos[:, None] + rotate_half(k) * sin[:, None]
        return q, k, v

    def _attend(self, q, k, v, qpos):
        c = self.cfg
        kk = k.repeat_interleave(c.group, dim=1).transpose(0, 1)
        vv = v.repeat_interleave(c.group, dim=1).transpose(0, 1)
        allowed = torch.arange(k.shape[0], device=q.device)[None] <= qpos[:, None]
        o = F.scaled_dot_product_attention(q.transpose(0, 1), kk, vv, attn_mask=allowed[None])
        return self.o_proj(o.transpose(0, 1).reshape(q.shape[0], -1))

    def approx(self, x, sin, cos, cache: Dict, tag: str):
        q, k, v = self._qkv(self.input_layernorm(x), sin, cos)
        cache[f"{tag}_k"], cache[f"{tag}_v"] = k.clone(), v.clone()
        a = self._attend(q, k, v, torch.arange(x.shape[0], device=x.device))
        m = self.mlp(self.post_attention_layernorm(x + a))
        cache[f"{tag}_inc"] = a + m
        return x + a + m

    def correct(self, x, rows: torch.Tensor, sin, cos, cache: Dict, tag: str):
        xa = x[rows]
        q, k, v = self._qkv(self.input_layernorm(xa), sin[rows], cos[rows])
        cache[f"{tag}_k"][rows], cache[f"{tag}_v"][rows] = k, v
        xatt = xa + self._attend(q, cache[f"{tag}_k"], cache[f"{tag}_v"], rows)
        out = x + cache[f"{tag}_inc"]
        out[rows] = xatt + self.mlp(self.post_attention_layernorm(xatt))
        return out


class Qwen25VL(nn.Module):
    """fp32 reference model (vision tower + LLM) used as the numerics oracle of the engine."""

    def __init__(self, cfg: Qwen25VLConfig):
        super().__init__()
        self.cfg = cfg
        self.visual = VisionTower(cfg)
        self.embed_tokens = nn.Embedding(cfg.vocab, cfg.hidden)
        self.layers = nn.ModuleList([DecoderLayer(cfg) for _ in range(cfg.depth)])
        self.norm = RMSNorm(cfg.hidden, cfg.rms_eps)
        self.lm_head = nn.Linear(cfg.hidden, cfg.vocab, bias=False)

    def init_weights(self, seed: int = 0, std: float = 0.02) -> "Qwen25VL":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("weight") and p.dim() == 1:
                    p.copy_(1.0 + 0.05 * torch.randn(p.shape, generator=g))
                elif name.endswith("bias"):
                    p.copy_(0.02 * torch.randn(p.shape, generator=g))
                else:
                    p.copy_(std * torch.randn(p.shape, generator=g))
        return self

    @classmethod
    def random_on(cls, cfg: Qwen25VLConfig, device, seed: int = 0, std: float = 0.02) -> "Qwen25VL":
        """Random-init model built directly on `device` (no host copy; for full-size presets)."""
        with torch.device("meta"):
            m = cls(cfg)
        m = m.to_empty(device=device)
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if name.endswith("weight") and p.dim() == 1:
                    p.normal_(1.0, 0.05, generator=g)
                elif name.endswith("bias"):
                    p.normal_(0.0, 0.02, generator=g)
                else:
                    p.normal_(0.0, std, generator=g)
        return m.eval()

    def embed(self, ids_before: torch.Tensor, img_emb: torch.Tensor, ids_after: torch.Tensor) -> torch.Tensor:
        return torch.cat([self.embed_tokens(ids_before), img_emb, self.embed_tokens(ids_after)], dim=0)
