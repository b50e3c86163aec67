"""Small helpers shared by client and server."""
from __future__ import annotations


def calculate_total_patches(config) -> int:
    """Patches per image for the configured transmission policy (ceil division per level)."""
    H, W = config.image_shape[:2]
    ph, pw = config.patch_size
    if config.transmission_policy_name == "Laplacian":
        levels = config.transmission_kwargs.get("pyramid_levels", [2, 1, 0])
        total = 0
        for lvl in levels:
            s = 2 ** lvl
            total += (-(-(H // s) // ph)) * (-(-(W // s) // pw))
        return total
    return (-(-H // ph)) * (-(-W // pw))
