"""Progressive Laplacian transmission: base first, residual crops in groups
(reference offload/policies/transmission/progressive.py:8-732).

Group 0 carries the base level. The residual crops of every finer level are assigned to groups
1..num_groups by `grouping_strategy`:

  grid / block_grid / expansion / sequential   fixed spatial layouts, identical on both ends
                                               (must agree with models/dinov3/vit.py
                                               create_group_index for the server's plan)
  random / geometric                           random draws
  uniform_diff                                 equal compressed bytes per group, from the batch-
                                               mean sorted crop sizes
  energy_asc / energy_desc                     equal residual energy per group
  top_energy / top_energy_threshold            one group of the highest-energy crops (keep_rate)
                                               or of crops above `pscore_threshold`; the rest are
                                               never sent

Each residual patch carries `pscore_hint`: the crop's residual RMS, or its energy when
`mobile_pscore` is residual_energy (the mobile-side score the server may fuse).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np

from ...common.protocol import ExperimentConfig, Patch, normalize_appcorr_kwargs
from .laplacian import LaplacianPyramidPolicy, as_image_list, compress_crops, cut_crops, levels_of, pool

DATA_DEPENDENT = {"uniform_diff", "energy_asc", "energy_desc"}


def crop_rms(crop: np.ndarray) -> float:
    return float(np.sqrt(np.square(crop.astype(np.float32)).mean(dtype=np.float32)))


def crop_energy(crop: np.ndarray) -> float:
    return float(np.square(crop.astype(np.float32)).sum(dtype=np.float32))


def _square_side(num_groups: int, name: str) -> int:
    s = int(num_groups ** 0.5)
    if s * s != num_groups:
        raise ValueError(f"{name} grouping requires a square num_groups, got {num_groups}")
    return s


def assign_groups(strategy: str, items: Sequence[dict], num_groups: int, config: Optional[ExperimentConfig] = None,
                  rng: Optional[np.random.Generator] = None) -> np.ndarray:
    """Group id per residual crop. `items` carry row, col, grid_hw, spatial_idx and (for the
    energy strategies) pscore; group 0 means "not transmitted"."""
    N = len(items)
    rng = rng or np.random.default_rng()
    if strategy == "grid":
        s = _square_side(num_groups, "grid")
        pat = np.arange(1, num_groups + 1).reshape(s, s)
        return np.asarray([pat[it["row"] % s, it["col"] % s] for it in items], dtype=int)
    if strategy == "block_grid":
        s = _square_side(num_groups, "block_grid")
        out = []
        for it in items:
            gh, gw = it["grid_hw"]
            out.append(min(it["row"] * s // max(gh, 1), s - 1) * s + min(it["col"] * s // max(gw, 1), s - 1) + 1)
        return np.asarray(out, dtype=int)
    if strategy == "expansion":
        if num_groups > N:
            raise ValueError(f"expansion grouping needs at least one patch per group, got num_groups={num_groups} "
                             f"for {N} patches")
        keys = []
        for i, it in enumerate(items):
            gh, gw = it["grid_hw"]
            dr, dc = 2 * it["row"] - (gh - 1), 2 * it["col"] - (gw - 1)
            keys.append((dr * dr * max(gw - 1, 1) ** 2 + dc * dc * max(gh - 1, 1) ** 2, i))
        order = sorted(range(N), key=lambda i: keys[i])
        out = np.empty(N, dtype=int)
        for rank, i in enumerate(order):
            out[i] = rank * num_groups // N + 1
        return out
    if strategy == "sequential":
        order = np.asarray([it["spatial_idx"] for it in items], dtype=int)
        return 1 + order * num_groups // max(N, 1)
    if strategy == "top_energy":
        keep = min(max(float((config.transmission_kwargs if config else {}).get("keep_rate", 1.0)), 0.0), 1.0)
        scores = np.asarray([it["pscore"] for it in items], dtype=np.float64)
        out = np.zeros(N, dtype=int)
        n_keep = int(round(keep * N))
        if n_keep > 0:
            out[np.argsort(-scores, kind="stable")[:n_keep]] = 1
        return out
    if strategy == "top_energy_threshold":
        thr = float((config.transmission_kwargs if config else {}).get("pscore_threshold", 0.0))
        return np.where(np.asarray([it["pscore"] for it in items]) >= thr, 1, 0).astype(int)
    if strategy == "crop_cover":
        from .windows import _assign_with_crop_cover

        return _assign_with_crop_cover(strategy, items, num_groups, config, rng)
    if strategy == "random":
        return rng.integers(1, num_groups + 1, size=N)
    if strategy == "geometric":
        g = np.floor(-np.log2(1 - rng.random(N))) + 1
        return np.clip(g, 1, num_groups).astype(int)
    return np.ones(N, dtype=int)


def balanced_rank_groups(values: np.ndarray, num_groups: int, descending: bool = False) -> np.ndarray:
    """values [B, N] per crop -> group ids [B, N] so every group holds ~1/num_groups of the
    batch-mean sorted total (crops ranked per image, boundaries from the mean curve)."""
    B, N = values.shape
    key = -values if descending else values
    order = np.argsort(key, axis=1, kind="stable")
    curve = np.cumsum(np.take_along_axis(values, order, axis=1).mean(0))
    groups = np.ones((B, N), dtype=int)
    if curve[-1] <= 0 or num_groups <= 0:
        return groups
    bounds = np.arange(1, num_groups) * (curve[-1] / num_groups)
    by_rank = np.searchsorted(bounds, curve) + 1
    np.put_along_axis(groups, order, np.broadcast_to(by_rank, (B, N)), axis=1)
    return groups


class ProgressiveLPyramidPolicy(LaplacianPyramidPolicy):
    default_levels = (2, 0)

    def num_groups(self, config: ExperimentConfig, images) -> int:
        return int(config.transmission_kwargs.get("num_groups", 4))

    @staticmethod
    def mobile_pscore(config: ExperimentConfig) -> str:
        return str(normalize_appcorr_kwargs(config.appcorr_kwargs, config.transmission_kwargs).get("mobile_pscore", "none"))

    @staticmethod
    def hint(crop: np.ndarray, kind: str) -> float:
        return crop_energy(crop) if kind == "residual_energy" else crop_rms(crop)

    # ------------------------------------------------------------------ per image work
    def _base(self, b, image, config, hw):
        levels = levels_of(config, self.default_levels)
        ph, pw = config.patch_size
        comp = config.transmission_kwargs.get("compression_level", 1)
        g = self.gaussians(image, max(levels))
        band = self.project(g[levels[0]], levels[0], config, np.uint8, hw)
        ts = tuple(image.shape[:2]) if hw is not None else ()
        patches = [Patch(b, i, d, levels[0], 0, target_shape=ts)
                   for i, d in enumerate(compress_crops(cut_crops(band, ph, pw), np.uint8, comp))]
        return patches, g

    def _residual_crops(self, g, config, hw) -> List[dict]:
        """Every residual crop of every finer level, in level-major row-major order."""
        levels = levels_of(config, self.default_levels)
        ph, pw = config.patch_size
        out = []
        prev = levels[0]
        for lvl in levels[1:]:
            res = self.closed_loop_residual(g, prev, lvl, config, hw)
            gh, gw = res.shape[0] // ph, res.shape[1] // pw
            for i, crop in enumerate(cut_crops(res, ph, pw)):
                r, c = divmod(i, gw)
                out.append({"spatial_idx": i, "res_level": lvl, "grid_hw": (gh, gw), "row": r, "col": c,
                            "crop": crop})
            prev = lvl
        return out

    def _make_patch(self, b, it, group, config, kind, ts) -> Patch:
        import zlib

        comp = config.transmission_kwargs.get("compression_level", 1)
        crop = it["crop"].astype(np.int16, copy=False)
        data = it.get("data") or zlib.compress(np.ascontiguousarray(crop).tobytes(), comp)
        return Patch(b, it["spatial_idx"], data, it["res_level"], int(group), pscore_hint=self.hint(crop, kind),
                     target_shape=ts)

    # ------------------------------------------------------------------ encode
    def encode(self, images, config: ExperimentConfig):
        import zlib

        imgs = as_image_list(images)
        B = len(imgs)
        ng = self.num_groups(config, imgs)
        kind = self.mobile_pscore(config)
        preserve = self.preserve_shape(config)
        hws = [im.shape[:2] if preserve else None for im in imgs]
        tss = [tuple(im.shape[:2]) if preserve else () for im in imgs]
        base = [pool().submit(self._base, b, im, config, hws[b]) for b, im in enumerate(imgs)]
        base = [f.result() for f in base]
        g0 = [p for ps, _ in base for p in ps]
        for p in g0:
            p.batch_group_total = len(g0)
        yield g0
        strategy = config.transmission_kwargs.get("grouping_strategy", "uniform_diff")
        crops = [f.result() for f in [pool().submit(self._residual_crops, g, config, hws[b])
                                      for b, (_, g) in enumerate(base)]]
        comp = config.transmission_kwargs.get("compression_level", 1)
        if strategy in DATA_DEPENDENT:
            if strategy == "uniform_diff":
                for items in crops:
                    for it in items:
                        it["data"] = zlib.compress(np.ascontiguousarray(it["crop"].astype(np.int16)).tobytes(), comp)
                vals = np.asarray([[len(it["data"]) for it in items] for items in crops], dtype=np.float64)
                gid = balanced_rank_groups(vals, ng)
            else:
                vals = np.asarray([[crop_energy(it["crop"]) for it in items] for items in crops])
                gid = balanced_rank_groups(vals, ng, descending=strategy == "energy_desc")
        else:
            if strategy in ("top_energy", "top_energy_threshold"):
                for items in crops:
                    for it in items:
                        it["pscore"] = crop_energy(it["crop"])
            gid = [assign_groups(strategy, items, ng, config) for items in crops]
        groups: Dict[int, List[Patch]] = {}
        for b, items in enumerate(crops):
            for it, g in zip(items, gid[b]):
                if g > 0:
                    groups.setdefault(int(g), []).append(self._make_patch(b, it, g, config, kind, tss[b]))
        for g in sorted(groups):
            ps = groups[g]
            for p in ps:
                p.batch_group_total = len(ps)
            yield ps
