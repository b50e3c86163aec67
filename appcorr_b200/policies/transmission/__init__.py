from .basic import FullImageCompressionPolicy, RawTransmissionPolicy, ZlibTransmissionPolicy  # noqa: F401
from .fourier import FourierLaplacianProgressivePolicy, FourierProgressiveTransmissionPolicy  # noqa: F401
from .laplacian import LaplacianPyramidPolicy  # noqa: F401
from .progressive import ProgressiveLPyramidPolicy  # noqa: F401
from .windows import (  # noqa: F401
    ADE20KWindowProgressiveLaplacianPolicy,
    COCOWindowProgressiveLaplacianPolicy,
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
    pass


class NYUAppCorrLaplacianPolicy(LaplacianPyramidPolicy):
    pass


class NYUAppCorrFourierLaplacianHybridPolicy(FourierLaplacianProgressivePolicy):
    pass
