"""The stock `transformers` SAM 3 detector downstream of this build's tower (as the reference runs
it: features in through `vision_embeds`, everything after the tower untouched), on the CPU with
the fp32 tower of a small SAM 3-shaped preset."""
import numpy as np
import torch

from appcorr_b200.models.qwen25vl import window_order
from appcorr_b200.models.sam3 import SAM3_PRESETS, SAM3Tower, build_stock_head, raster_features, stock_head_forward


def test_raster_features_restores_row_major_order():
    c = SAM3_PRESETS["sam3_tiny"]
    gh = gw = 16
    order = window_order(gh, gw, c.window_size, 1)
    tok = order.float().view(1, -1, 1).repeat(2, 1, 3)  # token i (window-major) carries its raster index
    f = raster_features(tok, c, gh, gw)
    assert torch.equal(f[..., 0], torch.arange(gh * gw).float().view(1, gh, gw).repeat(2, 1, 1))


def test_stock_head_on_tower_features():
    from appcorr_b200.server.model.sam3_executor import stock_results

    torch.manual_seed(0)
    c = SAM3_PRESETS["sam3_tiny"]
    tower = SAM3Tower(c).init_weights(0).eval()
    img = torch.randn(2, 3, c.img_size, c.img_size)
    with torch.no_grad():
        feat = raster_features(tower(img), c, 16, 16)
    head = build_stock_head(c, seed=0)
    out = stock_head_forward(head, feat)
    nq = head.config.detr_decoder_config.num_queries
    assert out.pred_masks.shape[:2] == (2, nq) and out.pred_boxes.shape == (2, nq, 4)
    assert torch.isfinite(out.pred_logits).all()
    boxes = torch.tensor([[[0.3, 0.3, 0.2, 0.2], [0.7, 0.6, 0.3, 0.4]]]).repeat(2, 1, 1)
    out2 = stock_head_forward(head, feat, boxes=boxes)
    again = stock_head_forward(head, feat, boxes=boxes)
    assert torch.equal(out2.pred_logits, again.pred_logits)  # deterministic for the same prompt
    assert not torch.equal(out2.pred_logits, out.pred_logits)  # the box prompt reaches the detector
    res = stock_results(out2)
    assert set(res) == {0, 1}
    assert res[0]["mask"].dtype == np.uint8 and res[0]["mask"].shape == tuple(out2.pred_masks.shape[-2:])
    assert 0.0 <= res[0]["score"] <= 1.0 and len(res[0]["box"]) == 4
