"""The vision encoder + projector on the B200 (tcgen05 contractions, the full-attention tcgen05 kernel, the patch
gather with the bake's pad, the 2D RoPE, the 2x2 unfold, the GELU) through the C ABI, against the CPU oracle
(oracle/vision.c, the restatement of app/crates/ocr-wgpu/src/vision.rs:266-423).

Tolerance: the embeddings (and the residual stream after k layers) within 2e-3 of the largest |value| and a relative
L2 of 1e-3 — the north star's logit bound. Both sides round K and V to f16 (the reference's f16 path); the device
splits every other operand exactly into f16 hi + lo and accumulates in f32, the oracle in f64.
Checked:
- a small encoder (width 256, 4 heads of 64, 2 layers) on images of 1, 10 and 3 x 32-row groups and 1-5 query / key
  tiles: after 0, 1 and 2 layers, and the projector's output;
- the LightOnOCR shape (width 1024, 16 heads, ffn 4096, 24 layers) on a small image, and at config 4's full size
  (1540 x 1100 → 1540 x 1120 baked, 8800 patches): the first layer's output rows against the oracle's row subset
  (every patch's keys and values computed), and the bake fused into the patch gather equals the encode of the
  oracle's baked copy bit for bit;
- the page read end to end at small size: the embeddings left on the device, prefilled between prompt ids (the
  reference's prompt layout, engine.rs:460-474), then greedy ids equal to the oracle text model's on the same rows;
- the attention alone (ocr_op_attention_full) against f64, including scores that force the one-pass softmax to
  rescale (the reference's own check of its f16 vision attention against f64 is f16_paths_match_cpu,
  app/crates/ocr-wgpu/src/text.rs:1186-1240);
- the bake on the device (the Lanczos-3 resize and the pads) byte for byte against the CPU restatement, and a page
  that needs the resize encoded end to end.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def close(got: np.ndarray, want: np.ndarray, tol: float = 2e-3, l2: float = 1e-3) -> None:
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    err = float(np.abs(got - want).max() / np.abs(want).max())
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    assert err <= tol and rel <= l2, f"max err {err:.2e} of max |value|, relative L2 {rel:.2e}"


def small_cfg(ocr, **kw):
    return ocr.VisionConfig(**{**dict(n_layer=2, dim=256, n_head=4, n_ff=1024, proj_dim=256), **kw})


def image(seed: int, h: int, w: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, (h, w, 3), dtype=np.uint8)


@pytest.mark.parametrize("h,w", [(56, 84), (196, 308), (364, 392)])
def test_small_encoder_matches_oracle(ocr, orc, ctx, h, w):
    cfg = small_cfg(ocr)
    v = ocr.Vision.synthetic(ctx, cfg, 41)
    ov = orc.Vision(cfg.as_dict(), 41)
    img = image(h + w, h, w)
    for layers in (0, 1, 2):
        close(v.encode(img, layers=layers), ov.encode(img, layers=layers))
    close(v.encode(img), ov.encode(img))
    v.close()


def test_encode_refuses_unbaked_images(ocr, ctx):
    v = ocr.Vision.synthetic(ctx, small_cfg(ocr, n_layer=1), 3)
    with pytest.raises(ocr.OcrError, match="not baked"):
        v.encode(image(1, 56, 70))  # 70 px: not on the 28 grid
    with pytest.raises(ocr.OcrError, match="not baked"):
        v.encode(image(1, 28, 1568))  # longer than image_size
    with pytest.raises(ocr.OcrError, match="layers"):
        v.encode(image(1, 56, 56), layers=2)
    v.close()


def test_lightonocr_shape_small_image(ocr, orc, ctx):
    cfg = ocr.VisionConfig()
    v = ocr.Vision.synthetic(ctx, cfg, 7)
    ov = orc.Vision(cfg.as_dict(), 7)
    img = image(9, 56, 112)
    close(v.encode(img, layers=1), ov.encode(img, layers=1))
    close(v.encode(img), ov.encode(img))
    v.close()


def test_config4_page_full_size(ocr, orc, ctx, torch_cuda):
    torch = torch_cuda
    cfg = ocr.VisionConfig()
    v = ocr.Vision.synthetic(ctx, cfg, 7)
    ov = orc.Vision(cfg.as_dict(), 7)
    page = image(4, 1100, 1540)
    baked = orc.bake_pad(page)
    assert baked.shape == (1120, 1540, 3)
    # the first layer's output at full size: rows across the grid (corners, the pad rows, the middle)
    rows = [0, 1, 109, 110, 4321, 8690, 8799]
    res = v.encode(baked, layers=1)
    assert res.shape == (8800, 1024)
    close(res[rows], ov.layer1_rows(baked, rows))
    # the whole encoder: the bake inside the patch gather equals the encode of the baked copy, bit for bit
    out_dev = torch.empty((2200, 1024), dtype=torch.float32, device="cuda")
    v.encode_page(page, out=out_dev)
    torch.cuda.synchronize()
    a = out_dev.cpu().numpy()
    b = v.encode(baked)
    assert np.array_equal(a, b)
    assert np.isfinite(a).all() and float(np.abs(a).max()) > 0
    v.close()


def test_page_read_end_to_end_small(ocr, orc, ctx, torch_cuda):
    """Engine::read_text's flow (engine.rs:447-524) at small size: encode → prompt [prefix ids, image rows, suffix
    ids] prefilled from the device rows → greedy decode with the window seeded by image-pad ids + the suffix"""
    torch = torch_cuda
    vcfg = small_cfg(ocr, proj_dim=256)
    v = ocr.Vision.synthetic(ctx, vcfg, 21)
    ov = orc.Vision(vcfg.as_dict(), 21)
    tcfg = dict(n_layer=2, dim=256, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000, eps=1e-6, rope_base=1e6)
    m = ocr.TextModel.synthetic(ctx, ocr.TextConfig(**{**tcfg, "n_ctx_train": 4096}), 5, 0.2, 1.0)
    om = orc.Model(tcfg, seed=5, sigma_w=0.2, sigma_e=1.0)
    page = image(8, 110, 150)  # bakes to 112 x 168: 6 x 4 merged tokens
    n_img = 24
    emb = torch.empty((n_img, 256), dtype=torch.float32, device="cuda")
    v.encode_page(page, out=emb)
    torch.cuda.synchronize()
    emb_h = emb.cpu().numpy()
    close(emb_h, ov.encode(orc.bake_pad(page)))
    prefix, suffix = [11, 12, 13, 14, 15, 16, 17], [21, 22, 23, 24, 25, 26, 27]
    ids = prefix + [-1] * n_img + suffix
    rows = np.zeros((len(ids), 256), np.float32)
    rows[len(prefix):len(prefix) + n_img] = emb_h
    dev_rows = torch.from_numpy(rows).cuda()
    s = m.session(128)
    lg = s.prefill(0, ids=ids, embd=dev_rows)
    os_ = om.session(128)
    lo = os_.prefill(ids, rows, len(ids))
    err = float(np.abs(lg - lo).max() / np.abs(lo).max())
    assert err <= 2e-3
    history = [999] * n_img + suffix  # the image-pad id stands in for 151655 in this 1000-token vocabulary
    preset = ocr.Preset("page", 0.0, 1.0, 1.15, 64, 0.0, 32)
    got = s.decode_gpu(0, preset, history)
    want, _ = os_.decode(lo, 1.15, 64, 0.0, history, 32)
    assert got == want.tolist()
    s.close()
    m.close()
    v.close()


@pytest.mark.parametrize("n_keys,L,step", [(300, 200, 0.0), (1000, 130, 0.0), (300, 200, 6.0), (640, 129, 2.5)])
def test_full_attention_op_matches_f64(ocr, ctx, torch_cuda, n_keys, L, step):
    """ocr_op_attention_full against softmax(q k^T / 8) v in f64 on the same f16 K / V. `step` > 0 raises every
    key tile's scores by step nats over the tile before (dimension 0 of q is 10, of K tile t is step * 8 t / 10), so
    the one-pass softmax's running maximum jumps past its headroom (8 in log2 units, 5.5 nats) and rescales O and
    the row sums at every tile (step 6), or at some tiles (step 2.5)."""
    torch = torch_cuda
    H, D = 2, 64
    rng = np.random.default_rng(n_keys + L)
    q = rng.standard_normal((L, H, D)).astype(np.float32)
    k = rng.standard_normal((H, n_keys, D)).astype(np.float16)
    v = rng.standard_normal((H, n_keys, D)).astype(np.float16)
    if step:
        q[:, :, 0] = 10.0
        k[:, :, 0] = (step * 8.0 / 10.0 * (np.arange(n_keys) // 64)).astype(np.float16)
    n_pad = (n_keys + 63) // 64 * 64
    kt, vt = ocr.attention_tiles(k, v, n_pad)
    dq = torch.from_numpy(q.reshape(L, H * D)).cuda()
    dk = torch.from_numpy(kt.reshape(-1).view(np.int16)).cuda()
    dv = torch.from_numpy(vt.reshape(-1).view(np.int16)).cuda()
    out = torch.zeros((L, H * D), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ocr.op_attention_full(ctx, dq.data_ptr(), H * D, L, H, dk.data_ptr(), dv.data_ptr(), n_pad, n_keys, 0.125,
                          out.data_ptr(), H * D)
    ctx.sync()
    got = out.cpu().numpy().reshape(L, H, D)
    s = np.einsum("lhd,hnd->lhn", q.astype(np.float64), k.astype(np.float64)) * 0.125
    p = np.exp(s - s.max(axis=2, keepdims=True))
    want = np.einsum("lhn,hnd->lhd", p / p.sum(axis=2, keepdims=True), v.astype(np.float64))
    close(got, want.astype(np.float32))


@pytest.mark.parametrize("w0,h0", [(3000, 2000), (1700, 500), (800, 1600), (1540, 1100), (40, 30)])
def test_image_bake_matches_oracle(ocr, orc, ctx, w0, h0):
    """ocr_image_bake (the Lanczos-3 resize of pages longer than 1540 px and the white pads, on the device) equals the
    CPU restatement byte for byte: the same taps (computed on the host in f32) and each sum taken tap by tap"""
    img = np.random.default_rng(w0 * h0).integers(0, 256, (h0, w0, 3), dtype=np.uint8)
    got = ocr.image_bake(ctx, img)
    want = orc.bake(img)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


def test_encode_page_with_resize_matches_oracle(ocr, orc, ctx):
    cfg = small_cfg(ocr, image_size=280)
    v = ocr.Vision.synthetic(ctx, cfg, 17)
    ov = orc.Vision(cfg.as_dict(), 17)
    page = image(12, 300, 400)  # scaled to 280 x 210, padded to 280 x 224: 20 x 16 patches
    got = v.encode_page(page)
    want = ov.encode(orc.bake(page, longest=280))
    close(got, want)
    v.close()
