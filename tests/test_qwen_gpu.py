"""Qwen2.5-VL-shaped VLM: the sm_100a engine (vision tower, paged-KV LLM approx / correct, first
token) against the fp32 PyTorch model of the same math (models/qwen25vl.py)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _setup(seed=0):
    from appcorr_b200.models.qwen25vl import PRESETS, Qwen25VL
    from appcorr_b200.models.qwen_engine import QwenVLEngine

    cfg = PRESETS["tiny"]
    m = Qwen25VL(cfg).init_weights(seed).to(DEV).eval()
    eng = QwenVLEngine(m, DEV)
    g = torch.Generator().manual_seed(seed)
    nb, na = 8, 24
    ids = torch.randint(0, cfg.vocab, (nb + na,), generator=g).to(DEV)
    return cfg, m, eng, ids, nb, na


def _oracle_x_in(m, img, ids, nb):
    with torch.no_grad():
        return m.embed(ids[:nb], m.visual(img[0]), ids[nb:])


def test_vision_tower_matches_module():
    cfg, m, eng, ids, nb, na = _setup()
    img = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(224, 224, nb, na)
    eng.vision(sess, img)
    eng.embed_text(sess, ids)
    ref = _oracle_x_in(m, img, ids, nb)
    assert _rel(sess.tensors["x_in"], ref) < 2e-2


def test_llm_approx_correct_and_first_token():
    from appcorr_b200.models.qwen25vl import mrope_positions, mrope_tables

    cfg, m, eng, ids, nb, na = _setup(1)
    img0 = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    img1 = img0.clone()
    img1[:, :112] = torch.randint(0, 256, (1, 112, 224, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(224, 224, nb, na)
    t = sess.tensors
    eng.vision(sess, img0)
    eng.embed_text(sess, ids)
    x = eng.approx(sess)
    pos = mrope_positions(nb, 8, 8, na)
    sin, cos = (v.to(DEV) for v in mrope_tables(cfg, pos))
    cache = {}
    with torch.no_grad():
        xr = _oracle_x_in(m, img0, ids, nb)
        for i, ly in enumerate(m.layers):
            xr = ly.approx(xr, sin, cos, cache, f"l{i}")
    torch.cuda.synchronize()
    assert _rel(x, xr) < 3e-2
    phys = t["phys"].long()
    for i in range(cfg.depth):
        k = t["kc"][i][phys].view(sess.N, cfg.kv_heads, cfg.head_dim)
        assert _rel(k, cache[f"l{i}_k"]) < 2e-2
        assert _rel(t["bos"][i], cache[f"l{i}_inc"]) < 3e-2
    # correction round on the changed canvas: 25% of the image tokens plus all text rows
    eng.vision(sess, img1)
    xc = eng.correct(sess, 0.25).clone()
    rows = t["rows"][: (nb + na) + sess.n_img // 4].long()
    # text rows first (prompt order), then the kept image rows ascending; queries carry their own
    # positions, so the packed order does not matter to the math
    assert rows.numel() == nb + na + 16 and rows.unique().numel() == rows.numel()
    assert set(range(nb)) | set(range(nb + 64, nb + 64 + na)) <= set(rows.tolist())
    with torch.no_grad():
        xr2 = _oracle_x_in(m, img1, ids, nb)
        for i, ly in enumerate(m.layers):
            xr2 = ly.correct(xr2, rows, sin, cos, cache, f"l{i}")
    torch.cuda.synchronize()
    assert _rel(xc, xr2) < 3e-2
    tok = eng.first_token(sess)
    with torch.no_grad():
        logits = m.lm_head(m.norm(xr2[-1:]))
    top2 = logits[0].topk(2).values
    if (top2[0] - top2[1]).item() > 1e-2 * top2[0].abs().item():
        assert int(tok) == int(logits[0].argmax())


def test_full_correction_equals_forward_on_new_image():
    cfg, m, eng, ids, nb, na = _setup(2)
    from appcorr_b200.models.qwen25vl import mrope_positions, mrope_tables

    img0 = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    img1 = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(224, 224, nb, na)
    eng.vision(sess, img0)
    eng.embed_text(sess, ids)
    eng.approx(sess)
    eng.vision(sess, img1)
    xc = eng.correct(sess, 1.0).clone()
    pos = mrope_positions(nb, 8, 8, na)
    sin, cos = (v.to(DEV) for v in mrope_tables(cfg, pos))
    with torch.no_grad():
        xr = _oracle_x_in(m, img1, ids, nb)
        for i, ly in enumerate(m.layers):
            xr = ly.approx(xr, sin, cos, {}, f"l{i}")
    torch.cuda.synchronize()
    assert _rel(xc, xr) < 3e-2


@pytest.mark.parametrize("impl", ["tcgen05", "tcgen05_split"])
def test_attention_gqa_causal_paged(impl):
    """Kernel-level: grouped-query causal attention over a paged pool, packed query subset."""
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(3)
    H, Hkv, Dh, N = 8, 2, 128, 300
    npages = 3
    table = torch.tensor([[2, 0, 1]], device=DEV, dtype=torch.int32)
    kl = torch.randn(N, Hkv * Dh, device=DEV).to(torch.bfloat16)
    vl = torch.randn(N, Hkv * Dh, device=DEV).to(torch.bfloat16)
    kpool = torch.zeros(npages * 128, Hkv * Dh, device=DEV, dtype=torch.bfloat16)
    vpool = torch.zeros_like(kpool)
    phys = (table[0].long()[torch.arange(N, device=DEV) // 128] * 128 + torch.arange(N, device=DEV) % 128)
    kpool[phys], vpool[phys] = kl, vl
    qpos = torch.tensor(sorted(torch.randperm(N)[:77].tolist()), device=DEV, dtype=torch.int32)
    q = torch.randn(qpos.numel(), H * Dh, device=DEV).to(torch.bfloat16)
    o = torch.empty_like(q)
    K.attention(q, kpool, vpool, o, B=1, Tq=qpos.numel(), Tk=N, H=H, Dh=Dh, Hkv=Hkv, causal=True, q_pos=qpos,
                block_table=table, impl=impl)
    qq = q.float().view(-1, H, Dh).transpose(0, 1)
    kk = kl.float().view(N, Hkv, Dh).repeat_interleave(H // Hkv, dim=1).transpose(0, 1)
    vv = vl.float().view(N, Hkv, Dh).repeat_interleave(H // Hkv, dim=1).transpose(0, 1)
    mask = torch.arange(N, device=DEV)[None] <= qpos[:, None].long()
    ref = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask[None])
    ref = ref.transpose(0, 1).reshape(-1, H * Dh)
    assert (o.float() - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 2e-2
    # contiguous causal prefill (q_pos implicit) with multiple query tiles
    q2 = torch.randn(N, H * Dh, device=DEV).to(torch.bfloat16)
    o2 = torch.empty_like(q2)
    K.attention(q2, kpool, vpool, o2, B=1, Tq=N, Tk=N, H=H, Dh=Dh, Hkv=Hkv, causal=True, block_table=table, impl=impl)
    qq = q2.float().view(-1, H, Dh).transpose(0, 1)
    ref2 = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=True).transpose(0, 1).reshape(N, -1)
    assert (o2.float() - ref2).abs().max().item() < 2e-2 * ref2.abs().max().item() + 2e-2


def test_llm_fp8_tracks_fp32():
    """e4m3 LLM GEMMs: approximate and full-correction passes stay close to the fp32 model."""
    from appcorr_b200.models.qwen25vl import PRESETS, Qwen25VL, mrope_positions, mrope_tables
    from appcorr_b200.models.qwen_engine import QwenVLEngine

    cfg = PRESETS["tiny"]
    m = Qwen25VL(cfg).init_weights(4).to(DEV).eval()
    eng = QwenVLEngine(m, DEV, "fp8")
    nb, na = 8, 24
    ids = torch.randint(0, cfg.vocab, (nb + na,), generator=torch.Generator().manual_seed(4)).to(DEV)
    img = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(224, 224, nb, na)
    eng.vision(sess, img)
    eng.embed_text(sess, ids)
    x = eng.approx(sess).clone()
    sin, cos = (v.to(DEV) for v in mrope_tables(cfg, mrope_positions(nb, 8, 8, na)))
    with torch.no_grad():
        xr = _oracle_x_in(m, img, ids, nb)
        for i, ly in enumerate(m.layers):
            xr = ly.approx(xr, sin, cos, {}, f"l{i}")
    assert _rel(x, xr) < 8e-2
    xc = eng.correct(sess, 1.0)
    assert _rel(xc, xr) < 8e-2


def test_partial_vision_correction_matches_oracle():
    """Only the merge units whose pixels moved most are recomputed through the tower (against the
    approximate pass's cached K / V); their LLM input rows change, the others do not; the LLM
    correction then covers the text plus exactly those rows. Both against the fp32 model."""
    from appcorr_b200.models.qwen25vl import merge_unit_raster, mrope_positions, mrope_tables

    cfg, m, eng, ids, nb, na = _setup(4)
    img0 = torch.randint(0, 256, (1, 224, 224, 3), dtype=torch.uint8, device=DEV)
    img1 = img0.clone()
    img1[:, 56:112, 112:224] = torch.randint(0, 256, (1, 56, 112, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(224, 224, nb, na)
    t = sess.tensors
    eng.vision(sess, img0)
    eng.embed_text(sess, ids)
    eng.approx(sess)
    x_in0 = t["x_in"].clone()
    units = eng.vision_correct(sess, img1, 0.125)                      # 8 of 64 units
    raster = merge_unit_raster(cfg, 16, 16).to(DEV)
    changed = set((nb + raster[units.long()]).tolist())
    # the changed pixels cover raster units rows 2..3 x cols 4..7 = 8 units: exactly those are picked
    expect = {nb + r * 8 + c for r in (2, 3) for c in range(4, 8)}
    assert changed == expect
    cache = {}
    with torch.no_grad():
        m.visual(img0[0], cache)
        emb = m.visual.correct(img1[0], units.long(), cache)
    got = t["x_in"][(nb + raster[units.long()]).long()]
    assert _rel(got, emb) < 2e-2
    keep_rows = [i for i in range(sess.N) if i not in changed]
    assert torch.equal(t["x_in"][keep_rows], x_in0[keep_rows])
    xc = eng.correct(sess, 0.125, units=units).clone()
    rows = t["rows"][: nb + na + units.numel()].long()
    assert set(rows.tolist()) == set(range(nb)) | set(range(nb + 64, nb + 64 + na)) | changed
    pos = mrope_positions(nb, 8, 8, na)
    sin, cos = (v.to(DEV) for v in mrope_tables(cfg, pos))
    lcache = {}
    with torch.no_grad():
        xr = _oracle_x_in(m, img0, ids, nb)
        for i, ly in enumerate(m.layers):
            xr = ly.approx(xr, sin, cos, lcache, f"l{i}")
        x_in1 = _oracle_x_in(m, img0, ids, nb)
        x_in1[(nb + raster[units.long()]).long()] = emb
        xr2 = x_in1
        for i, ly in enumerate(m.layers):
            xr2 = ly.correct(xr2, rows, sin, cos, lcache, f"l{i}")
    torch.cuda.synchronize()
    assert _rel(xc, xr2) < 3e-2
