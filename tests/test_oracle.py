"""The oracle pinned against the reference's own known answers (CPU, no GPU).

- sampling.rs tests (app/crates/ocr-decode/src/sampling.rs:297-321): windowed penalty on distinct tokens, frequency
  penalty
- the reference's penalty implementation itself (hf/window_rep_penalty.py apply(), run when the fixture was made):
  tests/golden/penalty_ref.json, bit for bit
- choose_pen_is_exact's sweep (app/crates/ocr-wgpu/src/text.rs:1061-1099): the penalty's product / quotient are IEEE
  f32, subnormals and extremes included (numpy's float32 arithmetic is the independent check)
- the q8_0 quantizer (text.rs:676-691, ggml quantize_row_q8_0_ref) against an independent numpy restatement
- f16 round to nearest even (half 2.7.1) against numpy's float16
- the seeded generators: the numpy spec (ocr_b200.gauss / fill_ids) and the C oracle give identical bits
- the C decoder against an independent numpy restatement of the Qwen3 prefill (7e-7 of the largest logit)
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_windowed_rp_hits_distinct_tokens_in_window_only(orc):
    # sampling.rs:298-304: token 0 is outside the window of 2, token 1 twice inside counts once
    t, l = orc.choose_greedy(np.array([2.0, 2.2, -1.0], np.float32), 1.1, 2, 0.0, [0, 1, 1])
    assert t == 0
    assert abs(l[1] - 2.0) < 1e-6


def test_frequency_penalty_counts_output(orc):
    # sampling.rs:316-321
    t, _ = orc.choose_greedy(np.array([1.0, 1.05], np.float32), 1.0, 2, 0.1, [], {1: 2})
    assert t == 0


def test_argmax_first_maximum_and_nan_rules(orc):
    # ties → the first index; ±0 tie; a NaN never wins; NaN at index 0 → 0; all -inf → 0
    assert orc.choose_greedy(np.array([1, 3, 3, 2], np.float32), 1.0, 1, 0.0, [])[0] == 1
    assert orc.choose_greedy(np.array([-0.0, 0.0], np.float32), 1.0, 1, 0.0, [])[0] == 0
    assert orc.choose_greedy(np.array([1, np.nan, 5, np.nan], np.float32), 1.0, 1, 0.0, [])[0] == 2
    assert orc.choose_greedy(np.array([np.nan, 1, 5], np.float32), 1.0, 1, 0.0, [])[0] == 0
    assert orc.choose_greedy(np.full(7, -np.inf, np.float32), 1.0, 1, 0.0, [])[0] == 0
    # -0.0 takes the division branch (x < 0 is false): stays -0.0
    l = orc.apply_window_penalty(np.array([-0.0, 1.0], np.float32), 1.1, 4, [0])
    assert l.view(np.uint32)[0] == np.float32(-0.0).view(np.uint32)


def _penalty_logits(seed, vocab):
    from tests.golden.make_golden import penalty_logits

    return penalty_logits(seed, vocab)


def test_penalty_matches_reference_fixture(orc):
    fx = json.loads((GOLDEN / "penalty_ref.json").read_text())
    assert len(fx["cases"]) >= 8
    for c in fx["cases"]:
        l = _penalty_logits(c["seed"], c["vocab"])
        hist = c["tail"] + c["out"]
        got = orc.apply_window_penalty(l, c["rp"], c["window"], hist)
        changed = np.nonzero(got.view(np.uint32) != l.view(np.uint32))[0]
        assert changed.tolist() == c["changed"], c
        assert got[changed].view(np.uint32).tolist() == c["values_bits"], c
        t, _ = orc.choose_greedy(l, c["rp"], c["window"], 0.0, hist)
        assert t == c["argmax"]


def test_penalty_is_exact_f32(orc):
    # text.rs:1061-1099: 8192 distinct window tokens over logits of every magnitude
    n = 8192
    s = np.uint64(3)
    bits = []
    with np.errstate(over="ignore"):
        for _ in range(n):
            s = s * np.uint64(6364136223846793005) + np.uint64(1442695040888963407)
            bits.append(int(s >> np.uint64(32)))
    l = np.empty(n, np.float32)
    for i, b in enumerate(bits):
        if i % 3 == 2:
            l[i] = -np.array([0x0D800000 + b % (0x7F000000 - 0x0D800000)], np.uint32).view(np.float32)[0]
        else:
            l[i] = np.array([b % 0x7F800000], np.uint32).view(np.float32)[0]
    l[:6] = np.array([0.0, -0.0, np.inf, np.finfo(np.float32).max, np.uint32(1).view(np.float32),
                      np.finfo(np.float32).tiny], np.float32)
    hist = np.arange(n, dtype=np.int32)
    for rp in [1.1, 0.9, 1.0000001, 3.0, 1e-3, 1e3, 1.7e-30, 6.0e29]:
        r = np.float32(rp)
        got = orc.apply_window_penalty(l, float(r), n, hist)
        with np.errstate(over="ignore", under="ignore", invalid="ignore"):
            want = np.where(l < 0, l * r, l / r).astype(np.float32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), rp


def _q8_0_numpy(x):
    """independent restatement of ggml quantize_row_q8_0_ref (text.rs:676-691)"""
    x = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1) / d, np.float32(0)).astype(np.float32)
    q = x * idv[:, None]
    q = np.where(q >= 0, np.floor(q + np.float32(0.5)), np.ceil(q - np.float32(0.5)))  # half away from zero
    q = np.clip(q, -128, 127).astype(np.int8)
    dh = d.astype(np.float16)
    blocks = np.concatenate([dh.view(np.uint8).reshape(-1, 2), q.view(np.uint8)], axis=1).ravel()
    return blocks, (q.astype(np.float32) * dh.astype(np.float32)[:, None]).ravel()


def test_quantizer_matches_ggml_restatement(orc, ocr):
    x = ocr.gauss(77, 32 * 4000, 0.3)
    x[:32] = 0.0  # an all-zero block: d = 0
    x[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[64] = 1e-3  # tiny amax
    b, deq = orc.quantize_q8_0(x)
    b2, deq2 = _q8_0_numpy(x)
    assert np.array_equal(b, b2)
    assert np.array_equal(deq.view(np.uint32), deq2.view(np.uint32))
    assert np.array_equal(orc.dequantize_q8_0(b, x.size), deq)


def test_gguf_block_known_answer(orc):
    # ocr-gguf/src/lib.rs:568-592: d = 0.5 (f16), q = i - 16 → values -8.0 … 7.5
    blk = np.concatenate([np.frombuffer(np.float16(0.5).tobytes(), np.uint8),
                          (np.arange(32) - 16).astype(np.int8).view(np.uint8)])
    v = orc.dequantize_q8_0(blk, 32)
    assert (v[0], v[31]) == (-8.0, 7.5)


def test_f16_round_to_nearest_even(orc):
    rs = np.random.RandomState(0)
    x = (rs.randn(20000) * 10.0 ** rs.uniform(-9, 5, 20000)).astype(np.float32)
    x = np.concatenate([x, np.array([0, -0.0, 65504, 65519.99, 65520, 2.9802322e-08, 5.96e-8, np.inf, -np.inf],
                                    np.float32)])
    with np.errstate(over="ignore"):
        assert np.array_equal(orc.f16_from_f32(x), x.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("seed", [1, 12345, 2**63 + 7])
def test_generators_match(orc, ocr, seed):
    assert np.array_equal(orc.gauss(seed, 50000, 0.02).view(np.uint32), ocr.gauss(seed, 50000, 0.02).view(np.uint32))
    assert np.array_equal(orc.fill_ids(seed, 999, 151936), ocr.fill_ids(seed, 999, 151936))
    assert orc.substream(seed, 5) == ocr.substream(seed, 5)
    g = ocr.gauss(seed, 200000)
    assert abs(g.mean()) < 0.01 and abs(g.std() - 1.0) < 0.01


def test_rope_table_matches_reference_formula(orc):
    # text.rs:132-142 (f32 theta, f32 cos / sin); the f64 rotation check of rope_neox_matches_cpu (text.rs:768-792)
    t = orc.rope_table(1e6, 128, 1005)
    for pos in (0, 1, 1000, 1004):
        for i in (0, 1, 31, 63):
            theta = pos * (1e6 ** (-(2 * i) / 128))
            assert abs(t[pos, i, 0] - np.cos(theta)) < 5e-4 and abs(t[pos, i, 1] - np.sin(theta)) < 5e-4


def test_oracle_decoder_is_deterministic_and_causal(orc):
    cfg = dict(n_layer=2, dim=256, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000)
    m = orc.Model(cfg, seed=5)
    a = m.session(40)
    ids = orc.fill_ids(9, 12, 1000)
    la = a.prefill(ids, None, 12)
    # the same prompt fed as prefill 8 + 4 steps gives the same last logits (prefill ≡ steps, causal)
    b = m.session(40)
    b.prefill(ids[:8], None, 8)
    for t in ids[8:]:
        lb = b.step(int(t))
    assert np.allclose(la, lb, rtol=1e-4, atol=1e-4 * np.abs(la).max())


def decoder_np(orc, m, cfg: dict, ids) -> np.ndarray:
    """An independent numpy restatement of the Qwen3 prefill (text.rs:4-10, 437-521: RMSNorm → q / k / v → per-head
    q / k RMSNorm → NEOX RoPE → K / V rounded to f16 → causal softmax attention / sqrt(128) → o + residual → RMSNorm →
    SwiGLU → down + residual; output_norm and the tied head), in f64 on the dequantised tensors: the last row's
    logits"""
    d, H, G, dh, f, V = cfg["dim"], cfg["n_head"], cfg["n_kv"], cfg["d_head"], cfg["n_ff"], cfg["n_vocab"]
    eps = cfg.get("eps", 1e-6)

    def q8(layer, kind, rows, cols):
        return orc.dequantize_q8_0(m.tensor(layer, kind), rows * cols).reshape(rows, cols).astype(np.float64)

    def vec(layer, kind):
        return m.tensor(layer, kind).view(np.float32).astype(np.float64)

    def norm(x, w):
        return x / np.sqrt((x * x).mean(axis=-1, keepdims=True) + eps) * w

    n = len(ids)
    emb = q8(-1, 0, V, d)
    x = emb[np.asarray(ids)]
    cs = orc.rope_table(cfg.get("rope_base", 1e6), dh, n).astype(np.float64)  # [pos][dh/2][2]
    c, s = cs[:, None, :, 0], cs[:, None, :, 1]

    def rope(v):  # [n][heads][dh], NEOX pairs (i, i + dh/2)
        a, b = v[..., :dh // 2], v[..., dh // 2:]
        return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)

    for l in range(cfg["n_layer"]):
        h = norm(x, vec(l, orc.ATTN_NORM))
        q = (h @ q8(l, orc.Q, H * dh, d).T).reshape(n, H, dh)
        k = (h @ q8(l, orc.K, G * dh, d).T).reshape(n, G, dh)
        v = (h @ q8(l, orc.V, G * dh, d).T).reshape(n, G, dh)
        q = rope(norm(q, vec(l, orc.Q_NORM)))
        k = rope(norm(k, vec(l, orc.K_NORM))).astype(np.float16).astype(np.float64)
        v = v.astype(np.float16).astype(np.float64)
        kk, vv = np.repeat(k, H // G, axis=1), np.repeat(v, H // G, axis=1)
        sc = np.einsum("qhd,khd->hqk", q, kk) / np.sqrt(dh)
        sc = np.where(np.tril(np.ones((n, n), bool))[None], sc, -np.inf)
        p = np.exp(sc - sc.max(axis=2, keepdims=True))
        a = np.einsum("hqk,khd->qhd", p / p.sum(axis=2, keepdims=True), vv).reshape(n, H * dh)
        x = x + a @ q8(l, orc.O, d, H * dh).T
        h = norm(x, vec(l, orc.FFN_NORM))
        g, u = h @ q8(l, orc.GATE, f, d).T, h @ q8(l, orc.UP, f, d).T
        x = x + (g / (1 + np.exp(-g)) * u) @ q8(l, orc.DOWN, d, f).T
    out_norm = m.tensor(-1, 1).view(np.float32).astype(np.float64)
    return norm(x[-1], out_norm) @ emb.T


def test_oracle_decoder_matches_a_numpy_restatement(orc):
    cfg = dict(n_layer=2, dim=256, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000, eps=1e-6, rope_base=1e6)
    m = orc.Model(cfg, seed=13, sigma_w=0.2, sigma_e=1.0)
    ids = [int(t) for t in orc.fill_ids(3, 17, 1000)]
    got = m.session(32).prefill(ids, None, len(ids))
    want = decoder_np(orc, m, cfg, ids)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= 1e-5, f"{err:.2e}"  # (7e-7 here: the C oracle's f32 roundings)
    assert int(np.argmax(got)) == int(np.argmax(want))
