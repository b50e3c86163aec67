"""Convolutional dense-prediction heads on the sm_100a kernels: a DPT depth head and an RRDB
super-resolution network, each as an fp32 reference module plus a GPU runner.

Convolutions run NHWC: a 1x1 convolution is one GEMM on the pixel rows; a KxK convolution is the
`im2col_nhwc` kernel followed by one GEMM against the weight reshaped to [Cout, ky, kx, Cin]
(K zero-padded to a multiple of 16). Bilinear resampling (and the fusion blocks' skip additions)
is the `resize_nhwc` kernel. ReLU / LeakyReLU between convolutions are PyTorch elementwise ops.

References: the DINOv3 depther's DPT head (reassemble 4 backbone layers, residual conv units,
feature fusion with 2x bilinear upsampling, depth head; the reference's
appcorr/models/dinov3/eval/depth models, executor offload/server/model/dinov3_depther.py) and
Real-ESRGAN's RRDBNet (offload/server/sr/realesrgan.py:102-304: conv_first, residual-in-residual
dense blocks of five 3x3 convolutions with LeakyReLU(0.2) and 0.2 residual scaling, nearest 2x
upsampling convolutions, conv_last). Differences by design in DPT: the reassemble resampling
uses bilinear up / strided 3x3 down instead of transposed convolutions.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from ..ops import kernels as K

BF16 = torch.bfloat16


def _pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def _pad32(n: int) -> int:
    return (n + 31) // 32 * 32


class ConvGPU:
    """nn.Conv2d (dilation 1, groups 1) as im2col + tcgen05 GEMM on NHWC bf16 maps."""

    def __init__(self, conv: nn.Conv2d, device):
        w = conv.weight.detach().float()                         # [Cout, Cin, kh, kw]
        self.cout, self.cin, self.kh, self.kw = w.shape
        self.stride, self.pad = conv.stride[0], conv.padding[0]
        k = self.kh * self.kw * self.cin
        self.kp = _pad16(k)
        wm = w.permute(0, 2, 3, 1).reshape(self.cout, k)         # column (ky*kw + kx)*Cin + c
        wm = F.pad(wm, (0, self.kp - k, 0, _pad32(self.cout) - self.cout))
        self.w = wm.to(device=device, dtype=BF16).contiguous()
        b = conv.bias.detach().float() if conv.bias is not None else torch.zeros(self.cout)
        self.b = F.pad(b, (0, _pad32(self.cout) - self.cout)).to(device=device, dtype=BF16).contiguous()
        self._cols: Dict[Tuple, torch.Tensor] = {}

    def out_hw(self, H: int, W: int) -> Tuple[int, int]:
        return ((H + 2 * self.pad - self.kh) // self.stride + 1, (W + 2 * self.pad - self.kw) // self.stride + 1)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, resid: Optional[torch.Tensor] = None
                 ) -> torch.Tensor:
        """x [B, H, W, Cin] -> [B, Ho, Wo, Cout] (+ resid, same shape as the output)."""
        B, H, W, C = x.shape
        Ho, Wo = self.out_hw(H, W)
        co = _pad32(self.cout)
        if self.kh == 1 and self.kw == 1 and self.stride == 1 and self.pad == 0 and C % 16 == 0:
            a = x.reshape(B * H * W, C)
        else:
            key = (B, H, W)
            a = self._cols.get(key)
            if a is None:
                a = self._cols[key] = torch.zeros(B * Ho * Wo, self.kp, device=x.device, dtype=BF16)
            K.im2col_nhwc(x, self.kh, self.kw, self.stride, self.pad, a)
        res = torch.empty(B * Ho * Wo, co, device=x.device, dtype=BF16)
        if resid is not None and co == self.cout:
            ones = torch.ones(co, device=x.device, dtype=BF16)
            K.gemm(a, self.w, res, epi=K.EPI_RESID, bias=self.b, gamma=ones, resid=resid.reshape(B * Ho * Wo, co))
        else:
            K.gemm(a, self.w, res, bias=self.b)
            if resid is not None:
                res[:, :self.cout] += resid.reshape(B * Ho * Wo, self.cout)
        y = res.view(B, Ho, Wo, co)
        y = y[..., :self.cout] if co != self.cout else y
        if out is not None:
            out.copy_(y)
            return out
        return y.contiguous() if co != self.cout else y


def resize(x: torch.Tensor, Ho: int, Wo: int, align_corners: bool, add: Optional[torch.Tensor] = None) -> torch.Tensor:
    out = torch.empty(x.shape[0], Ho, Wo, x.shape[3], device=x.device, dtype=BF16)
    return K.resize_nhwc(x.contiguous(), out, align_corners, add)


# ----------------------------------------------------------------------------- DPT
class ResidualConvUnit(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.conv1 = nn.Conv2d(c, c, 3, padding=1)
        self.conv2 = nn.Conv2d(c, c, 3, padding=1)

    def forward(self, x):
        return x + self.conv2(F.relu(self.conv1(F.relu(x))))


class FusionBlock(nn.Module):
    def __init__(self, c: int):
        super().__init__()
        self.rcu1, self.rcu2 = ResidualConvUnit(c), ResidualConvUnit(c)
        self.out_conv = nn.Conv2d(c, c, 1)

    def forward(self, x, skip=None):
        if skip is not None:
            x = x + self.rcu1(skip)
        x = self.rcu2(x)
        x = F.interpolate(x, scale_factor=2, mode="bilinear", align_corners=True)
        return self.out_conv(x)


class DPTHead(nn.Module):
    """Depth from 4 backbone layers: reassemble (1x1 projection, resample to strides 4/8/16/32 of
    the patch grid ... here x4, x2, x1, x0.5), 3x3 to `features`, fusion from deep to shallow,
    then conv 3x3 -> 2x up -> conv 3x3 -> ReLU -> conv 1x1 -> ReLU."""

    def __init__(self, in_dim: int, features: int = 256, channels: Sequence[int] = (256, 512, 1024, 1024)):
        super().__init__()
        self.proj = nn.ModuleList([nn.Conv2d(in_dim, c, 1) for c in channels])
        self.down = nn.Conv2d(channels[3], channels[3], 3, stride=2, padding=1)
        self.layer_rn = nn.ModuleList([nn.Conv2d(c, features, 3, padding=1, bias=False) for c in channels])
        self.fusion = nn.ModuleList([FusionBlock(features) for _ in range(4)])
        self.head1 = nn.Conv2d(features, features // 2, 3, padding=1)
        self.head2 = nn.Conv2d(features // 2, 32, 3, padding=1)
        self.head3 = nn.Conv2d(32, 1, 1)

    def init_weights(self, seed: int = 0) -> "DPTHead":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                fan = p[0].numel() if p.dim() > 1 else 1
                p.copy_(torch.randn(p.shape, generator=g) * (0.02 if p.dim() == 1 else fan ** -0.5))
        return self.eval()

    def forward(self, taps: List[torch.Tensor], gh: int, gw: int) -> torch.Tensor:
        """taps: 4 x [B, gh*gw, D] patch tokens -> depth [B, 1, 8*gh, 8*gw] (patch grid x 8)."""
        B = taps[0].shape[0]
        maps = [t.transpose(1, 2).reshape(B, -1, gh, gw) for t in taps]
        x = [self.proj[i](maps[i]) for i in range(4)]
        x[0] = F.interpolate(x[0], size=(4 * gh, 4 * gw), mode="bilinear", align_corners=False)
        x[1] = F.interpolate(x[1], size=(2 * gh, 2 * gw), mode="bilinear", align_corners=False)
        x[3] = self.down(x[3])
        r = [self.layer_rn[i](x[i]) for i in range(4)]
        p = self.fusion[3](r[3])
        p = self.fusion[2](p[..., : r[2].shape[2], : r[2].shape[3]], r[2])
        p = self.fusion[1](p, r[1])
        p = self.fusion[0](p, r[0])
        p = self.head1(p)
        p = F.interpolate(p, scale_factor=2, mode="bilinear", align_corners=True)
        return F.relu(self.head3(F.relu(self.head2(p))))


class DPTHeadGPU:
    def __init__(self, mod: DPTHead, device):
        cv = lambda c: ConvGPU(c, device)  # noqa: E731
        self.proj = [cv(c) for c in mod.proj]
        self.down = cv(mod.down)
        self.rn = [cv(c) for c in mod.layer_rn]
        self.fus = [(cv(f.rcu1.conv1), cv(f.rcu1.conv2), cv(f.rcu2.conv1), cv(f.rcu2.conv2), cv(f.out_conv))
                    for f in mod.fusion]
        self.h1, self.h2, self.h3 = cv(mod.head1), cv(mod.head2), cv(mod.head3)

    @staticmethod
    def _rcu(c1, c2, x):
        return c2(c1(torch.relu(x)).relu_(), resid=x)

    def _fuse(self, i, x, skip=None):
        c1, c2, c3, c4, co = self.fus[i]
        if skip is not None:
            x = self._rcu(c1, c2, skip).add_(x)
        x = self._rcu(c3, c4, x)
        x = resize(x, 2 * x.shape[1], 2 * x.shape[2], True)
        return co(x)

    def forward(self, taps: List[torch.Tensor], B: int, gh: int, gw: int) -> torch.Tensor:
        """taps: 4 x [B*gh*gw, D] bf16 patch tokens -> depth [B, 8*gh, 8*gw] fp32."""
        maps = [t.view(B, gh, gw, -1) for t in taps]
        x = [self.proj[i](maps[i]) for i in range(4)]
        x[0] = resize(x[0], 4 * gh, 4 * gw, False)
        x[1] = resize(x[1], 2 * gh, 2 * gw, False)
        x[3] = self.down(x[3])
        r = [self.rn[i](x[i]) for i in range(4)]
        p = self._fuse(3, r[3])
        p = self._fuse(2, p[:, : r[2].shape[1], : r[2].shape[2]].contiguous(), r[2])
        p = self._fuse(1, p, r[1])
        p = self._fuse(0, p, r[0])
        p = self.h1(p)
        p = resize(p, 2 * p.shape[1], 2 * p.shape[2], True)
        d = self.h3(self.h2(p).relu_()).relu_()
        return d[..., 0].float()


# ----------------------------------------------------------------------------- RRDB super-resolution
class RDB(nn.Module):
    def __init__(self, nf: int = 64, gc: int = 32):
        super().__init__()
        self.convs = nn.ModuleList([nn.Conv2d(nf + i * gc, gc if i < 4 else nf, 3, padding=1) for i in range(5)])

    def forward(self, x):
        feats = [x]
        for i, c in enumerate(self.convs):
            y = c(torch.cat(feats, 1))
            if i < 4:
                feats.append(F.leaky_relu(y, 0.2))
        return x + 0.2 * y


class RRDB(nn.Module):
    def __init__(self, nf: int = 64, gc: int = 32):
        super().__init__()
        self.rdbs = nn.ModuleList([RDB(nf, gc) for _ in range(3)])

    def forward(self, x):
        y = x
        for r in self.rdbs:
            y = r(y)
        return x + 0.2 * y


class RRDBNet(nn.Module):
    """x4 super-resolution network (RGB in [0, 1])."""

    def __init__(self, nf: int = 64, nb: int = 23, gc: int = 32, scale: int = 4):
        super().__init__()
        self.scale = scale
        self.conv_first = nn.Conv2d(3, nf, 3, padding=1)
        self.body = nn.ModuleList([RRDB(nf, gc) for _ in range(nb)])
        self.conv_body = nn.Conv2d(nf, nf, 3, padding=1)
        self.conv_up = nn.ModuleList([nn.Conv2d(nf, nf, 3, padding=1) for _ in range(scale // 2)])
        self.conv_hr = nn.Conv2d(nf, nf, 3, padding=1)
        self.conv_last = nn.Conv2d(nf, 3, 3, padding=1)

    def init_weights(self, seed: int = 0) -> "RRDBNet":
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for p in self.parameters():
                fan = p[0].numel() if p.dim() > 1 else 1
                p.copy_(torch.randn(p.shape, generator=g) * (0.1 * fan ** -0.5 if p.dim() > 1 else 0.0))
        return self.eval()

    def forward(self, x):
        f = self.conv_first(x)
        b = f
        for blk in self.body:
            b = blk(b)
        f = f + self.conv_body(b)
        for c in self.conv_up:
            f = F.leaky_relu(c(F.interpolate(f, scale_factor=2, mode="nearest")), 0.2)
        return self.conv_last(F.leaky_relu(self.conv_hr(f), 0.2))


class RRDBNetGPU:
    """RRDBNet on NHWC bf16 maps; the dense concatenations are channel slices of one buffer per RDB
    (each conv writes its growth channels in place), so no concatenation copies are made."""

    def __init__(self, mod: RRDBNet, device):
        cv = lambda c: ConvGPU(c, device)  # noqa: E731
        self.nf = mod.conv_first.out_channels
        self.gc = mod.body[0].rdbs[0].convs[0].out_channels
        self.first = cv(mod.conv_first)
        self.body = [[[cv(c) for c in r.convs] for r in blk.rdbs] for blk in mod.body]
        self.conv_body, self.conv_hr, self.conv_last = cv(mod.conv_body), cv(mod.conv_hr), cv(mod.conv_last)
        self.up = [cv(c) for c in mod.conv_up]
        self.dev = device

    def forward(self, img_u8: torch.Tensor) -> torch.Tensor:
        """uint8 [B, H, W, 3] -> uint8 [B, sH, sW, 3]."""
        B, H, W, _ = img_u8.shape
        x = torch.zeros(B, H, W, 8, device=self.dev, dtype=BF16)   # RGB padded to 8 channels
        x[..., :3] = img_u8.to(BF16) / 255.0
        f = self._conv_padded_in(self.first, x)
        nf, gc = self.nf, self.gc
        buf = torch.empty(B, H, W, nf + 4 * gc, device=self.dev, dtype=BF16)
        b = f
        for blk in self.body:
            y = b
            for convs in blk:
                buf[..., :nf] = y
                for i, c in enumerate(convs):
                    inp = buf[..., : nf + i * gc].contiguous()
                    o = c(inp)
                    if i < 4:
                        buf[..., nf + i * gc: nf + (i + 1) * gc] = F.leaky_relu(o, 0.2)
                    else:
                        y = y + 0.2 * o
            b = b + 0.2 * y
        f = self.conv_body(b, resid=f)
        for c in self.up:
            up = f.repeat_interleave(2, 1).repeat_interleave(2, 2)
            f = F.leaky_relu(c(up), 0.2)
        out = self.conv_last(F.leaky_relu(self.conv_hr(f), 0.2))
        return (out.float().clamp(0, 1) * 255.0).round().to(torch.uint8)

    def _conv_padded_in(self, conv: ConvGPU, x8: torch.Tensor) -> torch.Tensor:
        """conv_first takes 3 channels; run it on the 8-channel padded input (zero weights)."""
        if not hasattr(conv, "_w8"):
            w = conv.w[:, : conv.kh * conv.kw * conv.cin].float().view(-1, conv.kh, conv.kw, conv.cin)
            w8 = F.pad(w, (0, 8 - conv.cin)).reshape(w.shape[0], -1)
            conv._w8 = F.pad(w8, (0, _pad16(w8.shape[1]) - w8.shape[1])).to(BF16).contiguous()
            conv._kp8 = conv._w8.shape[1]
        B, H, W, _ = x8.shape
        cols = torch.zeros(B * H * W, conv._kp8, device=x8.device, dtype=BF16)
        K.im2col_nhwc(x8, conv.kh, conv.kw, conv.stride, conv.pad, cols)
        out = torch.empty(B * H * W, _pad32(conv.cout), device=x8.device, dtype=BF16)
        K.gemm(cols, conv._w8, out, bias=conv.b)
        return out.view(B, H, W, -1)[..., : conv.cout].contiguous()
