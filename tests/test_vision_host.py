"""The vision encoder's host pieces without a GPU: the bake's plan (libocrcuda's ocr_bake_plan_for and the oracle's
orc_bake_plan) against a plain-Python restatement of the reference's plan (app/crates/ocr-core/src/imageops.rs:275-316)
and its known cases, the bake's pad, the oracle's 2D RoPE table, pixel LUT and GELU against numpy restatements of
vision.rs:152-175 and gelu.wgsl, the synthetic vision weights' padded patch embedding, and the oracle's layer-1 row
subset (the full-size pin of the device encoder) against its whole-image encode.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

VCFG = dict(n_layer=2, dim=256, n_head=4, n_ff=1024, patch=14, merge=2, image_size=1540, proj_dim=256, eps=1e-5,
            rope_theta=1e4, mean=[0.48145466, 0.4578275, 0.40821073], std=[0.26862954, 0.26130258, 0.27577711])


def plan_py(longest, grid, w0, h0):
    """imageops.rs:275-316, step by step"""
    w, h = float(w0), float(h0)
    if max(w, h) > longest:
        s = longest / max(w, h)
        w, h = max(1.0, float(round_half_away(w * s))), max(1.0, float(round_half_away(h * s)))
    sw, sh = int(w), int(h)
    pads = [0, 0, 0, 0]  # left, top, right, bottom

    def pad(nw, nh):
        nonlocal w, h
        pw, ph = int(nw - w), int(nh - h)
        pads[0] += pw // 2
        pads[2] += pw - pw // 2
        pads[1] += ph // 2
        pads[3] += ph - ph // 2
        w, h = nw, nh

    if min(w, h) < 56.0:
        pad(56.0, h) if w <= h else pad(w, 56.0)
    gw, gh = math.ceil(w / grid) * grid, math.ceil(h / grid) * grid
    if gw != w or gh != h:
        pad(float(gw), float(gh))
    return (sw, sh, pads[0], pads[1], pads[2], pads[3])


def round_half_away(x):  # Rust f64::round
    return math.floor(x + 0.5) if x >= 0 else -math.floor(-x + 0.5)


SIZES = [(1540, 1100), (1540, 1120), (3000, 2000), (2000, 3000), (40, 30), (30, 40), (10, 2000), (1541, 700),
         (1100, 1540), (28, 28), (56, 57), (1, 1), (777, 333), (4000, 4000), (1539, 1541)]


@pytest.mark.parametrize("w0,h0", SIZES)
def test_bake_plan_matches_the_reference_rules(ocr, orc, w0, h0):
    want = plan_py(1540, 28, w0, h0)
    assert orc.bake_plan(1540, 28, w0, h0) == want
    assert ocr.bake_plan(1540, 28, w0, h0) == want
    sw, sh, l, t, r, b = want
    fw, fh = sw + l + r, sh + t + b
    assert fw % 28 == 0 and fh % 28 == 0
    assert (fw if sw <= sh else fh) >= 56  # the short edge (width on a tie) reaches 56
    assert max(sw, sh) <= 1540


def test_bake_plan_known_cases(ocr):
    # config 4's page: 1540 x 1100 is on the size limit; the height pads 20 px, 10 top and 10 bottom → 110 x 80 patches
    assert ocr.bake_plan(1540, 28, 1540, 1100) == (1540, 1100, 0, 10, 0, 10)
    # the pad's odd pixel goes right / bottom (left / top take the smaller half)
    assert ocr.bake_plan(1540, 28, 1540, 1099) == (1540, 1099, 0, 10, 0, 11)


def test_bake_pad_places_the_image_in_white(orc):
    rng = np.random.default_rng(5)
    img = rng.integers(0, 255, (1099, 1540, 3), dtype=np.uint8)
    out = orc.bake_pad(img)
    assert out.shape == (1120, 1540, 3)
    assert (out[:10] == 255).all() and (out[1109:] == 255).all()
    assert np.array_equal(out[10:1109], img)
    with pytest.raises(ValueError):
        orc.bake_pad(np.zeros((2000, 3000, 3), np.uint8))


def test_rope2d_table_and_lut_and_gelu(orc):
    # vision.rs:159-175 in numpy f32, the angle multiplied up step by step
    theta, dh, mp = np.float32(1e4), 64, 110
    tab = orc.rope2d_table(1e4, dh, mp)
    ts = np.power(theta, np.float32(-2.0 / 32), dtype=np.float32)
    for half in range(2):
        fs = np.float32(1.0) if half == 0 else np.power(theta, np.float32(-2.0 / 64), dtype=np.float32)
        for pos in (0, 1, 37, 109):
            t = np.float32(pos)
            for k in range(16):
                a = np.float32(fs * t)
                # (numpy's f32 power and the C library's powf may differ by an ulp, which the step-by-step products
                # carry into the angle: a bound of a few ulps of the angle)
                tol = 2e-7 + 8 * abs(float(a)) * 2.0 ** -24 * (k + 1)
                assert abs(tab[half, pos, k, 0] - math.cos(a)) <= tol and abs(tab[half, pos, k, 1] - math.sin(a)) <= tol
                t = np.float32(t * ts)
    assert (tab[:, 0, :, 0] == 1).all() and (tab[:, 0, :, 1] == 0).all()
    assert tab[0, 1, 0, 0] == np.float32(math.cos(1.0)) and tab[0, 1, 0, 1] == np.float32(math.sin(1.0))
    lut = orc.pixel_lut(VCFG)
    v = np.arange(256, dtype=np.float32)
    for c in range(3):
        want = (v / np.float32(255) - np.float32(VCFG["mean"][c])) / np.float32(VCFG["std"][c])
        assert np.array_equal(lut[c], want.astype(np.float32))
    x = np.linspace(-30, 30, 2001).astype(np.float32)
    g = np.array([orc.lib().orc_gelu_tanh(float(a)) for a in x], np.float32)
    xd = x.astype(np.float64)
    t = np.clip(0.7978845608028654 * xd * (1 + 0.044715 * xd * xd), -15, 15)
    # (1 + tanh) cancels for negative x: the bound is in units of |x|, the f32 evaluation's error there
    assert (np.abs(g - 0.5 * xd * (1 + np.tanh(t))) <= 1e-6 * np.maximum(1.0, np.abs(xd))).all()


def test_padded_patch_embedding_is_zero_past_the_patch(orc):
    rows, cols, valid = 8, 768, 588
    b = np.empty(rows * cols // 32 * 34, np.uint8)
    orc.lib().orc_synth_q8_0_padded(b.ctypes.data, rows, cols, valid, 1234, 0.02)
    w = orc.dequantize_q8_0(b, rows * cols).reshape(rows, cols)
    assert (w[:, valid:] == 0).all() and (w[:, :valid] != 0).mean() > 0.9
    # columns below `valid` hold the generator's values for the flat index r * valid + c
    x = orc.gauss(1234, rows * valid, 0.02).reshape(rows, valid)
    assert np.abs(w[:, :576] - x[:, :576]).max() <= np.abs(x).max() / 127 * 0.51 + 1e-7
    # valid == cols: the plain generator
    b2 = np.empty(4 * 256 // 32 * 34, np.uint8)
    orc.lib().orc_synth_q8_0_padded(b2.ctypes.data, 4, 256, 256, 77, 0.02)
    assert np.array_equal(b2, orc.synth_q8_0(4 * 256, 77, 0.02))


def test_oracle_layer1_rows_equal_its_encode(orc):
    v = orc.Vision(VCFG, 11)
    img = np.random.default_rng(0).integers(0, 256, (84, 112, 3), dtype=np.uint8)
    full = v.encode(img, layers=1)
    rows = [0, 5, 23, 47]
    assert np.array_equal(v.layer1_rows(img, rows), full[rows])
    out = v.encode(img)
    assert out.shape == (12, 256) and np.isfinite(out).all()
    with pytest.raises(ValueError):
        v.encode(img[:, :100])  # 100 px: not on the 28 grid


def resize_np(img: np.ndarray, w: int, h: int) -> np.ndarray:
    """imageops::resize(.., Lanczos3) of the image crate 0.25 in numpy f32: a vertical pass into f32, a horizontal pass
    into bytes; the taps summed one by one in order"""
    f = np.float32

    def lanczos3(x):
        def sinc(t):
            a = f(t * f(np.pi))
            return f(1.0) if t == 0 else f(np.sin(a) / a)
        return f(sinc(x) * sinc(f(x / f(3.0)))) if abs(x) < 3 else f(0.0)

    def taps(n_in, n_out, o):
        ratio = f(f(n_in) / f(n_out))
        sr = max(ratio, f(1.0))
        sup = f(f(3.0) * sr)
        c = f(f(f(o) + f(0.5)) * ratio)
        left = min(max(int(math.floor(f(c - sup))), 0), n_in - 1)
        right = min(max(int(math.ceil(f(c + sup))), left + 1), n_in)
        c = f(c - f(0.5))
        ws = [lanczos3(f(f(f(i) - c) / sr)) for i in range(left, right)]
        s = f(0.0)
        for x in ws:
            s = f(s + x)
        return left, [f(x / s) for x in ws]

    h0, w0 = img.shape[:2]
    tmp = np.zeros((h, w0, 3), np.float32)
    for y in range(h):
        l, ws = taps(h0, h, y)
        t = np.zeros((w0, 3), np.float32)
        for i, wv in enumerate(ws):
            t = (t + img[l + i].astype(np.float32) * wv).astype(np.float32)
        tmp[y] = t
    out = np.zeros((h, w, 3), np.uint8)
    for x in range(w):
        l, ws = taps(w0, w, x)
        t = np.zeros((h, 3), np.float32)
        for i, wv in enumerate(ws):
            t = (t + tmp[:, l + i] * wv).astype(np.float32)
        t = np.clip(t, 0, 255)
        out[:, x] = np.where(t >= 0, np.floor(t + 0.5), -np.floor(-t + 0.5)).astype(np.uint8)
    return out


@pytest.mark.parametrize("src,dst", [((90, 60), (41, 27)), ((37, 80), (20, 43)), ((64, 48), (64, 24))])
def test_oracle_resize_matches_a_numpy_restatement(orc, src, dst):
    # (numpy's sin and the C library's sinf may differ by an ulp in a weight: a byte may move by one)
    img = np.random.default_rng(sum(src)).integers(0, 256, (src[1], src[0], 3), dtype=np.uint8)
    got = orc.resize_lanczos3(img, *dst).astype(int)
    want = resize_np(img, *dst).astype(int)
    assert np.abs(got - want).max() <= 1 and (got != want).mean() < 0.01
    flat = np.full((src[1], src[0], 3), 131, np.uint8)
    assert (orc.resize_lanczos3(flat, *dst) == 131).all()  # the weights sum to one


def test_oracle_bake_scales_then_pads(orc):
    img = np.random.default_rng(3).integers(0, 256, (2000, 3000, 3), dtype=np.uint8)
    out = orc.bake(img)
    sw, sh, l, t, r, b = orc.bake_plan(1540, 28, 3000, 2000)
    assert out.shape == (sh + t + b, sw + l + r, 3) == (1036, 1540, 3)
    assert (out[:t] == 255).all() and (out[t + sh:] == 255).all()
    assert np.array_equal(out[t:t + sh, l:l + sw], orc.resize_lanczos3(img, sw, sh))


def test_vision_c_abi_refuses_bad_arguments_without_a_device(ocr):
    import ctypes as C

    L = ocr.lib()
    p = ocr.BakePlan()
    assert L.ocr_bake_plan_for(1540, 28, 0, 10, C.byref(p)) == 1  # OCR_ERR_ARG: sizes must be positive
    assert L.ocr_bake_plan_for(1540, 28, 10, 10, None) == 1
    assert L.ocr_vision_encode(None, None, 56, 56, -1, None, 0, None, None) == 1
    assert "null" in L.ocr_last_error().decode()
    assert L.ocr_vision_encode_page(None, None, 56, 56, None, 0, None) == 1
    assert L.ocr_vision_config(None, None) == 1
    assert L.ocr_vision_destroy(None) == 0
    assert L.ocr_image_bake(None, None, 10, 10, 1540, 28, None, 0, None, None) == 1
    assert L.ocr_op_attention_full(None, None, 0, 0, 0, None, None, 0, 0, 0.0, None, 0) == 1


def encode_np(orc, cfg: dict, seed: int, sigma: float, img: np.ndarray) -> np.ndarray:
    """An independent numpy restatement of the vision encoder + projector (vision.rs:266-317, 405-423; patchify.wgsl,
    rope2d.wgsl, attention.wgsl with K / V rounded to f16, swiglu.wgsl, unfold2x2.wgsl, gelu.wgsl), in f64 on the
    synthetic weights' dequantised values — a second implementation the C restatement is checked against"""
    d, H, f, p, pd = cfg["dim"], cfg["n_head"], cfg["n_ff"], cfg["patch"], cfg["proj_dim"]
    dh, pp = d // H, 3 * p * p
    pcols = (pp + 255) // 256 * 256

    def mat(kind_stream, rows, cols):
        return orc.dequantize_q8_0(orc.synth_q8_0(rows * cols, orc.substream(seed, kind_stream), sigma),
                                   rows * cols).reshape(rows, cols).astype(np.float64)

    def norm(x, w):
        return x / np.sqrt((x * x).mean(axis=1, keepdims=True) + cfg["eps"]) * w

    h0, w0 = img.shape[:2]
    px, py = w0 // p, h0 // p
    n = px * py
    lut = orc.pixel_lut(cfg).astype(np.float64)
    P = np.zeros((n, pcols))
    for t in range(n):
        ty, tx = divmod(t, px)
        patch = img[ty * p:(ty + 1) * p, tx * p:(tx + 1) * p]  # [ky][kx][c]
        P[t, :pp] = np.stack([lut[c][patch[:, :, c]] for c in range(3)]).reshape(-1)
    wp = np.zeros((d, pcols))
    b = np.empty(d * pcols // 32 * 34, np.uint8)
    orc.lib().orc_synth_q8_0_padded(b.ctypes.data, d, pcols, pp, orc.substream(seed, orc.V_PATCH_STREAM), sigma)
    wp[:] = orc.dequantize_q8_0(b, d * pcols).reshape(d, pcols)
    x = norm(P @ wp.T, orc.fill_norm(orc.substream(seed, orc.V_PRE_LN_STREAM), d))
    cs = orc.rope2d_table(cfg["rope_theta"], dh, max(px, py)).astype(np.float64)
    pos = [np.arange(n) // px, np.arange(n) % px]

    def rope(v):  # [n][H][dh]
        v = v.copy()
        for half in range(2):
            c, s = cs[half, pos[half], :, 0][:, None, :], cs[half, pos[half], :, 1][:, None, :]
            a = v[:, :, half * dh // 2:(half + 1) * dh // 2]
            x0, x1 = a[:, :, 0::2].copy(), a[:, :, 1::2].copy()
            a[:, :, 0::2], a[:, :, 1::2] = x0 * c - x1 * s, x0 * s + x1 * c
        return v

    for l in range(cfg["n_layer"]):
        st = lambda k: orc.V_LAYER_STREAM + l * 16 + k
        hn = norm(x, orc.fill_norm(orc.substream(seed, st(orc.V_LN1)), d))
        q = rope((hn @ mat(st(orc.V_Q), d, d).T).reshape(n, H, dh))
        k = rope((hn @ mat(st(orc.V_K), d, d).T).reshape(n, H, dh)).astype(np.float16).astype(np.float64)
        v = (hn @ mat(st(orc.V_V), d, d).T).reshape(n, H, dh).astype(np.float16).astype(np.float64)
        s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(dh)
        pr = np.exp(s - s.max(axis=2, keepdims=True))
        a = np.einsum("hqk,khd->qhd", pr / pr.sum(axis=2, keepdims=True), v).reshape(n, d)
        x = x + a @ mat(st(orc.V_O), d, d).T
        hn = norm(x, orc.fill_norm(orc.substream(seed, st(orc.V_LN2)), d))
        g, u = hn @ mat(st(orc.V_GATE), f, d).T, hn @ mat(st(orc.V_UP), f, d).T
        x = x + (g / (1 + np.exp(-g)) * u) @ mat(st(orc.V_DOWN), d, f).T
    xn = norm(x, orc.fill_norm(orc.substream(seed, orc.V_INPUT_NORM_STREAM), d))
    grid = xn.reshape(py, px, d)
    z = np.stack([grid[ky::2, kx::2] for ky in range(2) for kx in range(2)], axis=-1)  # [oy][ox][c][ky*2+kx]
    z = z.reshape(-1, 4 * d)
    m1 = (z @ mat(orc.V_MERGER_STREAM, d, 4 * d).T) @ mat(orc.V_MM1_STREAM, pd, d).T
    t = np.clip(0.7978845608028654 * m1 * (1 + 0.044715 * m1 * m1), -15, 15)
    return (0.5 * m1 * (1 + np.tanh(t))) @ mat(orc.V_MM2_STREAM, pd, pd).T


def test_oracle_encoder_matches_a_numpy_restatement(orc):
    cfg = dict(VCFG, n_layer=2)
    img = np.random.default_rng(4).integers(0, 256, (56, 84, 3), dtype=np.uint8)
    got = orc.Vision(cfg, 29).encode(img)
    want = encode_np(orc, cfg, 29, 0.02, img)
    assert got.shape == want.shape == (6, 256)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-5, f"{err:.2e}"  # (3e-7 here: f32 vs f64 roundings)


def test_bake_plan_reference_known_answers(ocr, orc):
    """the reference's own tests of the plan (app/crates/ocr-core/src/imageops.rs:517-530:
    plan_scales_down_and_pads_to_grid, plan_never_upscales)"""
    for bake_plan in (ocr.bake_plan, orc.bake_plan):
        sw, sh, l, t, r, b = bake_plan(1540, 28, 3000, 2000)
        assert (sw, sh) == (1540, 1027) and (sw + l + r, sh + t + b) == (1540, 1036) and (t, b) == (4, 5)
        sw, sh, l, t, r, b = bake_plan(1540, 28, 500, 30)
        assert (sw, sh) == (500, 30) and (sw + l + r, sh + t + b) == (504, 56)


def mmproj_kvs(**over):
    """the clip.* metadata of a LightOnOCR mmproj GGUF (VisionConfig::from_gguf's keys, vision.rs:55-88)"""
    import gguf_writer as W

    kv = {"clip.projector_type": (W.STR, "lightonocr"), "clip.use_silu": (W.BOOL, 1),
          "clip.vision.embedding_length": (W.U32, 1024), "clip.vision.attention.head_count": (W.U32, 16),
          "clip.vision.block_count": (W.U32, 24), "clip.vision.feed_forward_length": (W.U32, 4096),
          "clip.vision.patch_size": (W.U32, 14), "clip.vision.spatial_merge_size": (W.U32, 2),
          "clip.vision.image_size": (W.U32, 1540), "clip.vision.projection_dim": (W.U32, 1024),
          "clip.vision.attention.layer_norm_epsilon": (W.F32, 1e-5),
          "clip.vision.image_mean": (W.ARR, (W.F32, [0.48145466, 0.4578275, 0.40821073])),
          "clip.vision.image_std": (W.ARR, (W.F32, [0.26862954, 0.26130258, 0.27577711]))}
    kv.update(over)
    return [(k, t, v) for k, (t, v) in kv.items() if t is not None]


def test_vision_config_from_gguf(ocr):
    import gguf_writer as W

    c = ocr.Gguf(data=W.write(mmproj_kvs(), [])).vision_config()
    want = ocr.VisionConfig()
    assert (c.n_layer, c.dim, c.n_head, c.n_ff, c.patch, c.merge, c.image_size, c.proj_dim) == \
        (want.n_layer, want.dim, want.n_head, want.n_ff, want.patch, want.merge, want.image_size, want.proj_dim)
    assert c.eps == np.float32(1e-5) and c.rope_theta == 10000.0
    assert np.allclose(c.mean, want.mean) and np.allclose(c.std, want.std)
    # the reference's refusals (vision.rs:57-73), message for message
    for over, match in [({"clip.projector_type": (W.STR, "pixtral")}, "runs lightonocr only"),
                        ({"clip.use_silu": (W.BOOL, 0)}, "would not be SwiGLU"),
                        ({"clip.vision.attention.head_count": (W.U32, 8)}, "written for 64"),
                        ({"clip.vision.image_std": (W.ARR, (W.F32, [0.5, 0.5]))}, "has 2 values"),
                        ({"clip.vision.block_count": (None, None)}, "clip.vision.block_count")]:
        with pytest.raises(ocr.OcrError, match=match):
            ocr.Gguf(data=W.write(mmproj_kvs(**over), [])).vision_config()
