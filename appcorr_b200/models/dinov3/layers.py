"""DINOv3 ViT building blocks with the approximate / correct partial-token passes.

Module names and parameter shapes match the DINOv3 state dict (reference
appcorr/models/dinov3/layers/{block,attention,ffn_layers,layer_scale,patch_embed,
rope_position_encoding}.py) so checkpoints load with `strict=True`.

The `approx` / `correct` methods here are the plain-PyTorch statement of the AppCorr math. They
run on CPU in fp32 and serve as the correctness oracle for the sm_100a engine
(appcorr_b200/models/engine.py) and as the CPU serving path:

approx (block.py:312-349, attention.py:215-278): a normal block forward that also caches, per
layer, K (after RoPE) and V of every token, the server patch score, and the block's residual
increment `bos = ls1(attn) + ls2(mlp)`.

correct (block.py:943-1191, attention.py:393-534): given the fresh full-resolution tokens `x`,
pick the top tokens among the candidates, recompute only those rows (new q/k/v, overwrite their
K/V in the cache, attend against the whole cache, proj, MLP), and rebuild every other row as
`x + bos` from the approximate pass. The recomputed increment is written back into `bos` so a
later round that replays the layer reproduces it.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ...common.protocol import LAYERMEAN_SERVER_PSCORES, VALID_SERVER_PSCORES


# ------------------------------------------------------------------------------ RoPE
class RopePositionEmbedding(nn.Module):
    """Axial 2-D RoPE tables (sin, cos) of shape [H*W, head_dim] for a token grid.

    Coordinates are patch centres normalised to [-1, 1] per axis ("separate") or by the longer /
    shorter side; angles 2*pi*coord / period with periods base**(2i/(D/2)), i < D/4, laid out as
    [h-angles | w-angles] and tiled twice (rope_position_encoding.py:16-121).
    """

    def __init__(self, embed_dim: int, *, num_heads: int, base: Optional[float] = 100.0,
                 min_period: Optional[float] = None, max_period: Optional[float] = None,
                 normalize_coords: str = "separate", shift_coords=None, jitter_coords=None,
                 rescale_coords=None, dtype: Optional[torch.dtype] = None, device=None):
        super().__init__()
        assert embed_dim % (4 * num_heads) == 0
        both = min_period is not None and max_period is not None
        if (base is None and not both) or (base is not None and both):
            raise ValueError("Either `base` or `min_period`+`max_period` must be provided.")
        self.D_head = embed_dim // num_heads
        self.base, self.min_period, self.max_period = base, min_period, max_period
        self.normalize_coords = normalize_coords
        self.shift_coords, self.jitter_coords, self.rescale_coords = shift_coords, jitter_coords, rescale_coords
        self.dtype = dtype
        self.register_buffer("periods", torch.empty(self.D_head // 4, device=device, dtype=dtype), persistent=True)
        self._init_weights()

    def _init_weights(self) -> None:
        n = self.D_head // 4
        dev, dt = self.periods.device, self.dtype
        if self.base is not None:
            exps = 2 * torch.arange(n, device=dev, dtype=dt) / (self.D_head // 2)
            periods = self.base ** exps
        else:
            ratio = self.max_period / self.min_period
            periods = ratio ** torch.linspace(0, 1, n, device=dev, dtype=dt) / ratio * self.max_period
        self.periods.data = periods

    def forward(self, *, H: int, W: int) -> Tuple[Tensor, Tensor]:
        dd = {"device": self.periods.device, "dtype": self.dtype}
        if self.normalize_coords == "max":
            dh = dw = max(H, W)
        elif self.normalize_coords == "min":
            dh = dw = min(H, W)
        elif self.normalize_coords == "separate":
            dh, dw = H, W
        else:
            raise ValueError(f"Unknown normalize_coords: {self.normalize_coords}")
        ch = torch.arange(0.5, H, **dd) / dh
        cw = torch.arange(0.5, W, **dd) / dw
        coords = torch.stack(torch.meshgrid(ch, cw, indexing="ij"), dim=-1).flatten(0, 1)
        coords = 2.0 * coords - 1.0
        # (training-time shift / jitter / rescale augmentations are not applied at inference)
        angles = 2 * math.pi * coords[:, :, None] / self.periods[None, None, :]
        angles = angles.flatten(1, 2).tile(2)
        return torch.sin(angles), torch.cos(angles)


def rope_rotate_half(x: Tensor) -> Tensor:
    a, b = x.chunk(2, dim=-1)
    return torch.cat([-b, a], dim=-1)


def rope_apply(x: Tensor, sin: Tensor, cos: Tensor) -> Tensor:
    return x * cos + rope_rotate_half(x) * sin


# ------------------------------------------------------------------------------ small layers
class PatchEmbed(nn.Module):
    """Conv2d(k = s = patch) image -> [B, H/p, W/p, D] tokens (patch_embed.py:21-89)."""

    def __init__(self, img_size=224, patch_size=16, in_chans=3, embed_dim=768, flatten_embedding=False):
        super().__init__()
        p = patch_size if isinstance(patch_size, tuple) else (patch_size, patch_size)
        s = img_size if isinstance(img_size, tuple) else (img_size, img_size)
        self.img_size, self.patch_size = s, p
        self.patches_resolution = (s[0] // p[0], s[1] // p[1])
        self.num_patches = self.patches_resolution[0] * self.patches_resolution[1]
        self.in_chans, self.embed_dim = in_chans, embed_dim
        self.flatten_embedding = flatten_embedding
        self.proj = nn.Conv2d(in_chans, embed_dim, kernel_size=p, stride=p)
        self.norm = nn.Identity()

    def forward(self, x: Tensor) -> Tensor:
        x = self.proj(x)
        H, W = x.shape[2], x.shape[3]
        x = self.norm(x.flatten(2).transpose(1, 2))
        if not self.flatten_embedding:
            x = x.reshape(-1, H, W, self.embed_dim)
        return x

    def reset_parameters(self) -> None:
        bound = 1.0 / math.sqrt(self.in_chans * self.patch_size[0] * self.patch_size[1])
        nn.init.uniform_(self.proj.weight, -bound, bound)
        if self.proj.bias is not None:
            nn.init.uniform_(self.proj.bias, -bound, bound)


class LayerScale(nn.Module):
    def __init__(self, dim: int, init_values: float = 1e-5, inplace: bool = False, device=None):
        super().__init__()
        self.inplace = inplace
        self.init_values = init_values
        self.gamma = nn.Parameter(torch.empty(dim, device=device))

    def reset_parameters(self) -> None:
        nn.init.constant_(self.gamma, self.init_values)

    def forward(self, x: Tensor) -> Tensor:
        return x.mul_(self.gamma) if self.inplace else x * self.gamma


class LinearKMaskedBias(nn.Linear):
    """qkv Linear whose bias is multiplied by a per-output mask (the k third is masked)."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        assert self.out_features % 3 == 0
        if self.bias is not None:
            self.register_buffer("bias_mask", torch.full_like(self.bias, math.nan))

    def effective_bias(self) -> Optional[Tensor]:
        if self.bias is None:
            return None
        return self.bias * self.bias_mask.to(self.bias.dtype)

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight, self.effective_bias())


def linear_bias(lin: nn.Linear) -> Optional[Tensor]:
    if isinstance(lin, LinearKMaskedBias):
        return lin.effective_bias()
    return lin.bias


class Mlp(nn.Module):
    def __init__(self, in_features, hidden_features=None, out_features=None, act_layer=nn.GELU, drop=0.0,
                 bias=True, device=None):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        self.fc1 = nn.Linear(in_features, hidden_features, bias=bias, device=device)
        self.act = act_layer()
        self.fc2 = nn.Linear(hidden_features, out_features, bias=bias, device=device)
        self.drop = nn.Dropout(drop)

    def forward(self, x: Tensor) -> Tensor:
        return self.drop(self.fc2(self.drop(self.act(self.fc1(x)))))


class SwiGLUFFN(nn.Module):
    def __init__(self, in_features, hidden_features=None, out_features=None, act_layer=None, drop=0.0,
                 bias=True, align_to=8, device=None):
        super().__init__()
        out_features = out_features or in_features
        hidden_features = hidden_features or in_features
        d = int(hidden_features * 2 / 3)
        hidden = d + (-d % align_to)
        self.w1 = nn.Linear(in_features, hidden, bias=bias, device=device)
        self.w2 = nn.Linear(in_features, hidden, bias=bias, device=device)
        self.w3 = nn.Linear(hidden, out_features, bias=bias, device=device)

    def forward(self, x: Tensor) -> Tensor:
        return self.w3(F.silu(self.w1(x)) * self.w2(x))


# ------------------------------------------------------------------------------ attention
class SelfAttention(nn.Module):
    def __init__(self, dim, num_heads=8, qkv_bias=False, proj_bias=True, attn_drop=0.0, proj_drop=0.0,
                 mask_k_bias=False, use_qk_norm=False, device=None):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.use_qk_norm = use_qk_norm
        self.q_norm = nn.LayerNorm(self.head_dim, eps=1e-5, device=device) if use_qk_norm else None
        self.k_norm = nn.LayerNorm(self.head_dim, eps=1e-5, device=device) if use_qk_norm else None
        lin = LinearKMaskedBias if mask_k_bias else nn.Linear
        self.qkv = lin(dim, dim * 3, bias=qkv_bias, device=device)
        self.attn_drop = nn.Dropout(attn_drop)
        self.proj = nn.Linear(dim, dim, bias=proj_bias, device=device)
        self.proj_drop = nn.Dropout(proj_drop)

    def _split_qkv(self, x: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
        """[..., D] -> q, k, v each [..., H, Dh] (qk-norm applied, no RoPE)."""
        qkv = self.qkv(x)
        q, k, v = qkv.unflatten(-1, (3, self.num_heads, self.head_dim)).unbind(-3)
        if self.q_norm is not None:
            q, k = self.q_norm(q), self.k_norm(k)
        return q, k, v

    @staticmethod
    def _rope_tokens(t: Tensor, rope, tok: Tensor, n_prefix: int) -> Tensor:
        """Apply RoPE to rows of t ([..., H, Dh]) whose token index tok >= n_prefix."""
        if rope is None:
            return t
        sin, cos = rope
        ridx = (tok - n_prefix).clamp_min(0)
        s = sin[ridx].unsqueeze(-2).to(torch.float32)
        c = cos[ridx].unsqueeze(-2).to(torch.float32)
        rotated = rope_apply(t.to(torch.float32), s, c).to(t.dtype)
        mask = (tok >= n_prefix).view(tok.shape + (1, 1))
        return torch.where(mask, rotated, t)

    def forward(self, x: Tensor, rope=None) -> Tensor:
        B, N, _ = x.shape
        q, k, v = self._split_qkv(x)
        if rope is not None:
            tok = torch.arange(N, device=x.device).expand(B, N)
            npre = N - rope[0].shape[0]
            q = self._rope_tokens(q, rope, tok, npre)
            k = self._rope_tokens(k, rope, tok, npre)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        return self.proj(o.transpose(1, 2).reshape(B, N, -1))


def server_pscore_from_qk(q: Tensor, k: Tensor, kind: str, scale: float, n_patch: int) -> Tensor:
    """Server patch score [B, N] from q, k [B, N, H, Dh] of one layer (attention.py:241-274)."""
    qf = q.transpose(1, 2).float()
    kf = k.transpose(1, 2).float()
    N = qf.shape[2]
    if kind in {"patch_attn_prob", "patch_attn_prob_layermean"}:
        p = (qf @ kf.transpose(-1, -2) * scale).softmax(-1)
        return p.mean(1).mean(1)
    if kind in {"patch_pseudo_attn_prob", "patch_pseudo_attn_prob_layermean"}:
        qp = qf[:, :, N - n_patch:]
        qm = qp.mean(2, keepdim=True)
        qm_norm = qm.norm(dim=-1, keepdim=True).clamp_min(torch.finfo(qm.dtype).eps)
        target = qp.norm(dim=-1, keepdim=True).mean(2, keepdim=True)
        qpseudo = qm * (target / qm_norm)
        p = (qpseudo @ kf.transpose(-1, -2) * scale).softmax(-1)
        return p.mean(1).mean(1)
    # cls_attn_prob (+ layermean, random): softmax of the CLS query, averaged over heads
    s = qf[:, :, 0:1] @ kf.transpose(-1, -2) * scale
    return s.softmax(-1).mean(1).squeeze(1)


@dataclass
class PartialTokenPlan:
    """Packed correction plan of one layer: `update_indice[b]` = prefix tokens then kept patches."""

    update_indice: Tensor          # [B, T] token indices
    combined_scores: Tensor        # [B, P]
    kept_mass: Tensor
    full_mass: Tensor
    kept_patches: Tensor
    full_patches: Tensor
    samples: Tensor


def select_keep_mask(scores: Tensor, keep_ratio: float, keep_thres: Optional[float]) -> Tensor:
    B, P = scores.shape
    if P == 0:
        return torch.zeros(B, 0, dtype=torch.bool, device=scores.device)
    if keep_thres is not None:
        return scores >= keep_thres
    k = min(int(P * keep_ratio), P)
    mask = torch.zeros(B, P, dtype=torch.bool, device=scores.device)
    if k <= 0:
        return mask
    if k == P:
        return mask.fill_(True)
    mask.scatter_(1, torch.topk(scores, k, dim=1).indices, True)
    return mask


def build_update_indice(pre: Tensor, cand: Tensor, keep: Tensor, keep_cap: int, thres_mode: bool) -> Tensor:
    """Ascending packed plan. Threshold + cap keeps the first `cap` kept candidates in candidate
    order and pads short rows with their last kept candidate (block.py:495-560); otherwise rows
    are padded up to the longest row with their last kept candidate."""
    B, P = cand.shape
    counts = keep.sum(1)
    order = torch.argsort(keep.to(torch.uint8), dim=1, descending=True, stable=True)
    if thres_mode and keep_cap > 0:
        K = max(0, min(int(keep_cap), P))
    else:
        K = int(counts.max().item()) if B > 0 else 0
    if K == 0:
        return pre.clone()
    pos = torch.arange(K, device=cand.device).unsqueeze(0)
    pos = torch.minimum(pos, (counts - 1).clamp_min(0).unsqueeze(1))
    sel = order.gather(1, pos)
    return torch.cat([pre, cand.gather(1, sel)], dim=1)


class SelfAttentionBlock(nn.Module):
    _VALID_SERVER_PSCORES = VALID_SERVER_PSCORES
    _LAYERMEAN_SERVER_PSCORES = LAYERMEAN_SERVER_PSCORES

    def __init__(self, dim, num_heads, ffn_ratio=4.0, qkv_bias=False, proj_bias=True, ffn_bias=True, drop=0.0,
                 attn_drop=0.0, init_values=None, drop_path=0.0, act_layer=nn.GELU, norm_layer=nn.LayerNorm,
                 attn_class=SelfAttention, ffn_layer=SwiGLUFFN, mask_k_bias=False, use_qk_norm=False, device=None):
        super().__init__()
        self.norm1 = norm_layer(dim)
        self.attn = attn_class(dim, num_heads=num_heads, qkv_bias=qkv_bias, proj_bias=proj_bias,
                               attn_drop=attn_drop, proj_drop=drop, mask_k_bias=mask_k_bias,
                               use_qk_norm=use_qk_norm, device=device)
        self.ls1 = LayerScale(dim, init_values=init_values, device=device) if init_values else nn.Identity()
        self.norm2 = norm_layer(dim)
        self.mlp = ffn_layer(in_features=dim, hidden_features=int(dim * ffn_ratio), act_layer=act_layer,
                             drop=drop, bias=ffn_bias, device=device)
        self.ls2 = LayerScale(dim, init_values=init_values, device=device) if init_values else nn.Identity()

    # -- stock forward
    def forward(self, x: Tensor, rope=None) -> Tensor:
        x = x + self.ls1(self.attn(self.norm1(x), rope=rope))
        return x + self.ls2(self.mlp(self.norm2(x)))

    # -- approximate pass
    def approx(self, x: Tensor, rope, cache: Dict, tag: str, *, server_pscore: str = "cls_attn_prob",
               server_pscore_weight: float = 1.0, **_) -> Tuple[Tensor, Dict]:
        """Stock block forward that also caches K/V, the server score and the increment."""
        B, N, _ = x.shape
        a = self.attn
        q, k, v = a._split_qkv(self.norm1(x))
        if rope is not None:
            npre = N - rope[0].shape[0]
            tok = torch.arange(N, device=x.device).expand(B, N)
            q = a._rope_tokens(q, rope, tok, npre)
            k = a._rope_tokens(k, rope, tok, npre)
            n_patch = rope[0].shape[0]
        else:
            n_patch = N
        for key in [k for k in cache if k.startswith("_plan") or k.startswith("_shared")]:
            cache.pop(key)
        cache[f"{tag}_k"] = k.detach().clone()
        cache[f"{tag}_v"] = v.detach().clone()
        if server_pscore_weight != 0.0 and server_pscore not in {"none", "disabled"}:
            cache[f"{tag}_server_pscore"] = server_pscore_from_qk(q, k, server_pscore, a.scale, n_patch).detach()
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        attn_inc = self.ls1(a.proj(o.transpose(1, 2).reshape(B, N, -1)))
        x_attn = x + attn_inc
        mlp_inc = self.ls2(self.mlp(self.norm2(x_attn)))
        cache[f"{tag}_bos"] = (attn_inc + mlp_inc).detach()
        return x_attn + mlp_inc, cache

    # -- correction pass
    @staticmethod
    def server_scores(cache: Dict, tag: str, kind: str) -> Tensor:
        stack = tag.rstrip("0123456789")
        if kind in LAYERMEAN_SERVER_PSCORES:
            key = f"_shared_{kind}_{stack}"
            if key not in cache:
                names = sorted(k for k in cache if k.endswith("_server_pscore")
                               and k[: -len("_server_pscore")].rstrip("0123456789") == stack)
                if not names:
                    raise KeyError(f"no cached server pscores for stack '{stack}'")
                cache[key] = torch.stack([cache[n] for n in names]).mean(0)
            return cache[key]
        s = cache.get(f"{tag}_server_pscore")
        if s is None:
            raise KeyError(f"Missing cached {tag}_server_pscore; it is produced by approx")
        if kind == "random":
            key = f"_shared_random_{stack}"
            if key not in cache:
                cache[key] = torch.rand_like(s)
            return cache[key]
        return s

    def make_plan(self, cache: Dict, tag: str, dindice: Tensor, n_prefix: int, opts: Dict,
                  mobile_hint: Optional[Tensor] = None, candidate_valid: Optional[Tensor] = None) -> PartialTokenPlan:
        pre, cand = dindice[:, :n_prefix], dindice[:, n_prefix:]
        ws = float(opts.get("server_pscore_weight", 1.0))
        kind = str(opts.get("server_pscore", "cls_attn_prob"))
        if kind not in VALID_SERVER_PSCORES:
            raise ValueError(f"Unknown server_pscore '{kind}'")
        B = dindice.shape[0]
        if ws == 0.0:
            server = torch.zeros(B, cand.shape[1], device=dindice.device)
        else:
            server = self.server_scores(cache, tag, kind).float().gather(1, cand)
        comb = ws * server
        wm = float(opts.get("mobile_pscore_weight", 0.0))
        if mobile_hint is not None and wm != 0.0 and opts.get("mobile_pscore", "none") != "none":
            N = cache[f"{tag}_k"].shape[1]
            hint = mobile_hint.float()
            m = hint.gather(1, cand - n_prefix) if hint.shape[1] == N - n_prefix else hint.gather(1, cand)
            mt = wm * m
            fusion = opts.get("pscore_fusion", "add")
            if fusion == "multiply":
                comb = comb * mt
            elif fusion == "geo_mean":
                comb = torch.sqrt(torch.clamp(comb * mt, min=0.0))
            else:
                comb = comb + mt
        if candidate_valid is not None:
            comb = comb.masked_fill(~candidate_valid, float("-inf"))
        thres = opts.get("token_keep_thres")
        keep = select_keep_mask(comb, float(opts.get("token_keep_ratio", 0.2)), thres)
        upd = build_update_indice(pre, cand, keep, int(opts.get("token_keep_cap", 0) or 0), thres is not None)
        finite = torch.where(torch.isfinite(comb), comb, torch.zeros_like(comb))
        return PartialTokenPlan(
            update_indice=upd,
            combined_scores=comb,
            kept_mass=(finite * keep).sum(),
            full_mass=finite.sum(),
            kept_patches=keep.sum().float(),
            full_patches=torch.tensor(float(keep.numel())),
            samples=torch.tensor(float(B)),
        )

    def correct(self, x: Tensor, dindice: Tensor, rope, cache: Dict, tag: str, *,
                query_plan: Optional[PartialTokenPlan] = None, mobile_pscore_hint: Optional[Tensor] = None,
                candidate_valid_mask: Optional[Tensor] = None, **opts) -> Tuple[Tensor, Dict]:
        B, N, C = x.shape
        n_prefix = int(opts.get("num_pretokens", N - rope[0].shape[0] if rope is not None else 0))
        plan = query_plan
        if plan is None:
            plan = self.make_plan(cache, tag, dindice, n_prefix, opts, mobile_pscore_hint, candidate_valid_mask)
        upd = plan.update_indice                      # [B, T]
        T = upd.shape[1]
        bidx = torch.arange(B, device=x.device).unsqueeze(1).expand(B, T)
        x_act = x[bidx, upd]                          # [B, T, C]
        a = self.attn
        q, k, v = a._split_qkv(self.norm1(x_act))     # [B, T, H, Dh]
        if rope is not None:
            q = a._rope_tokens(q, rope, upd, n_prefix)
            k = a._rope_tokens(k, rope, upd, n_prefix)
        kc, vc = cache[f"{tag}_k"], cache[f"{tag}_v"]
        kc[bidx, upd] = k.to(kc.dtype)
        vc[bidx, upd] = v.to(vc.dtype)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), kc.transpose(1, 2).to(q.dtype),
                                           vc.transpose(1, 2).to(q.dtype))
        x_attn = x_act + self.ls1(a.proj(o.transpose(1, 2).reshape(B, T, C)))
        mlp = self.ls2(self.mlp(self.norm2(x_attn)))
        bos = cache[f"{tag}_bos"]
        out = x + bos.to(x.dtype)
        out[bidx, upd] = x_attn + mlp
        bos[bidx, upd] = ((x_attn - x_act) + mlp).to(bos.dtype)
        cache[f"{tag}_plan"] = plan
        for name, val in (("kept_mass", plan.kept_mass), ("full_mass", plan.full_mass),
                          ("kept_patches", plan.kept_patches), ("full_patches", plan.full_patches),
                          ("samples", plan.samples)):
            cache[f"_stat_{name}"] = cache.get(f"_stat_{name}", 0.0) + val.detach().float().cpu()
        return out, cache
