from .basic import FullImageCompressionPolicy, RawTransmissionPolicy, ZlibTransmissionPolicy  # noqa: F401
from .fourier import FourierLaplacianProgressivePolicy, FourierProgressiveTransmissionPolicy  # noqa: F401
from .laplacian import LaplacianPyramidPolicy  # noqa: F401
from .progressive import ProgressiveLPyramidPolicy  # noqa: F401
from .windows import (  # noqa: F401
    ADE20KWindowProgressiveLaplacianPolicy,
    COCOWindowProgressiveLaplacianPolicy,
    FixedModelGridMixin,
    NYUAppCorrProgressiveLaplacianPolicy,
    VGGTLaplacianPolicy,
)


class FourierLaplacianHybridPolicy(FourierLaplacianProgressivePolicy):
    """DCT base + residual groups over the 3x3 detector windows."""

    default_strategy = "block_grid"

    def num_groups(self, config, images) -> int:
        return int(config.transmission_kwargs.get("num_window_groups", config.transmission_kwargs.get("num_groups", 9)))


class FourierADE20KWindowHybridPolicy(FourierLaplacianProgressivePolicy):
    default_strategy = "crop_cover"

    def encode(self, images, config):
        from .windows import slide_crops

        prof = config.get_input_profile_config()
        H, W = config.image_shape[:2]
        n = len(slide_crops(H, W, int(prof.get("server_crop_size", 512)), int(prof.get("server_stride", 341))))
        self._n = n
        for group in super().encode(images, config):
            for p in group:
                p.num_correction_groups = n
            yield group

    def num_groups(self, config, images) -> int:
        return getattr(self, "_n", 1)


class NYUAppCorrRawTransmissionPolicy(RawTransmissionPolicy):
    """Raw NYU transmission (reference nyu_appcorr_progressive.py:87-122): every image resized to
    the fixed model grid (config.image_shape) and sent whole, one patch per image with a
    (h, w, c, target_h, target_w) header."""

    def encode(self, images, config):
        import numpy as np

        from ...common.protocol import Patch
        from .basic import _HDR, _split_item

        h, w = FixedModelGridMixin.model_hw(config)
        items = [images[b] for b in range(images.shape[0])] if isinstance(images, np.ndarray) else list(images)
        out = []
        for b, item in enumerate(items):
            img, meta = _split_item(item)
            if img is None or img.ndim != 3:
                raise RuntimeError(f"expected an HWC image, got {None if img is None else img.shape}")
            ts = tuple(int(v) for v in (meta.get("target_shape") or img.shape[:2]))
            img = FixedModelGridMixin.to_model_grid(img, h, w)
            p = Patch(image_idx=b, spatial_idx=0, data=_HDR.pack(*img.shape, *ts) + img.tobytes())
            p.batch_group_total = len(items)
            p.target_shape = ts
            out.append(p)
        yield out

    def decode(self, patches, config, canvas=None):
        import numpy as np

        from .basic import _HDR

        H, W, C = config.image_shape
        out = np.zeros((config.batch_size, H, W, C), np.uint8) if not isinstance(canvas, np.ndarray) else canvas
        for p in patches:
            if p.spatial_idx != 0 or not p.data:
                continue
            h, w, c, _, _ = _HDR.unpack(p.data[:_HDR.size])
            img = np.frombuffer(p.data[_HDR.size:], np.uint8).reshape(h, w, c)
            out[p.image_idx] = FixedModelGridMixin.to_model_grid(img, H, W)
        return out


class NYUAppCorrLaplacianPolicy(FixedModelGridMixin, LaplacianPyramidPolicy):
    """Single- or multi-level Laplacian NYU transmission on the fixed model grid."""


class NYUAppCorrFourierLaplacianHybridPolicy(FixedModelGridMixin, FourierLaplacianProgressivePolicy):
    """DCT base + Laplacian residual groups on NYU's fixed model grid."""
