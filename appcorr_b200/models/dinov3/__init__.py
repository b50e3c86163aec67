from .layers import (  # noqa: F401
    LayerScale,
    LinearKMaskedBias,
    Mlp,
    PartialTokenPlan,
    PatchEmbed,
    RopePositionEmbedding,
    SelfAttention,
    SelfAttentionBlock,
    SwiGLUFFN,
    rope_apply,
    server_pscore_from_qk,
)
from .vit import (  # noqa: F401
    PRESETS,
    DinoVisionTransformer,
    ViTConfig,
    build_vit,
    create_group_index,
    dinov3_vit7b16,
    dinov3_vitl16,
    dinov3_vits16,
)
