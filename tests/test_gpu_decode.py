"""The whole decode path on a B200 through the C ABI, against the CPU oracle.

- the seeded synthetic generator on the device gives the oracle's weights bit for bit; a GGUF written from the
  oracle's tensors loads (stream + repack) to the same device bytes (ocr_model_checksum)
- prefill, the CPU-choice step loop and the device-choice run-ahead decode of a small qwen3-shaped model match the
  oracle: logits within 2e-3 of max |logit| (the acceptance bound) and 1e-3 relative L2; greedy ids identical
  (kv_growth_matches_presized_cache's checks, app/crates/ocr-wgpu/src/text.rs:1329-1379, on this engine's
  preallocated cache)
- batched decode equals one slot at a time; a callback that stops ends the read where it says
- BASELINE config 2 at full size: the 512 greedy ids equal the oracle's (tests/golden/config2_greedy.json)
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import gguf_writer as W

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"

# the reference's tiny_text_model shape (text.rs:1297-1323): 5 layers, dim 256, 2 q heads on 1 kv head, ffn 512
TINY = dict(n_layer=5, dim=256, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000, eps=1e-6, rope_base=1e6)


def text_config(ocr, c, n_ctx_train=40960):
    return ocr.TextConfig(c["n_layer"], c["dim"], c["n_head"], c["n_kv"], c["d_head"], c["n_ff"], c["n_vocab"],
                          n_ctx_train, c.get("eps", 1e-6), c.get("rope_base", 1e6))


def close_logits(got, want):
    """the acceptance bound (2e-3 of max |logit|) and relative L2 1e-3: the f16 KV store turns f32 differences of
    summation order into occasional one-step f16 differences (2^-11 relative) that the next layers carry"""
    m = np.abs(want).max()
    assert np.abs(got - want).max() <= 2e-3 * m, np.abs(got - want).max() / m
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 1e-3, rel


@pytest.fixture(scope="module")
def tiny(ocr, orc, ctx):
    om = orc.Model(TINY, seed=31, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, TINY), 31, 0.2, 1.0)
    return om, gm


def test_synthetic_weights_are_the_oracles(ocr, orc, tiny):
    om, gm = tiny
    for layer in range(TINY["n_layer"]):
        for kind in range(11):
            assert gm.tensor_gguf(layer, kind) == om.tensor(layer, kind).tobytes(), (layer, kind)
    assert gm.tensor_gguf(-1, 0) == om.tensor(-1, 0).tobytes()
    assert gm.tensor_gguf(-1, 1) == om.tensor(-1, 1).tobytes()


def test_gguf_load_equals_synthetic(ocr, orc, ctx, tiny, tmp_path):
    om, gm = tiny
    data = W.text_model(om)
    p = tmp_path / "tiny.gguf"
    p.write_bytes(data)
    a = ocr.TextModel.load(ctx, str(p))
    b = ocr.TextModel.from_bytes(ctx, W.text_model(om, alignment=64))
    assert a.checksum() == gm.checksum() == b.checksum()
    assert a.cfg.n_vocab == 1000 and a.cfg.n_layer == 5


def test_prefill_step_decode_match_oracle(ocr, orc, ctx, tiny):
    om, gm = tiny
    prompt = [int(t) for t in orc.fill_ids(5, 20, TINY["n_vocab"])]
    n_new, n_steps = 150, 40
    n_ctx = len(prompt) + n_new
    # the CPU-choice path: prefill, then steps of the greedy token, logits every step
    gs = gm.session(n_ctx)
    osn = om.session(n_ctx)
    lg = gs.prefill(0, ids=prompt)
    lo = osn.prefill(prompt, None, len(prompt))
    close_logits(lg, lo)
    for _ in range(n_steps):
        t = int(np.argmax(lo))
        lg = gs.step([t])[0]
        lo = osn.step(t)
        close_logits(lg, lo)
    assert gs.n_past(0) == len(prompt) + n_steps
    # the device choice, run ahead, from the prompt's logits
    gs2 = gm.session(n_ctx)
    gs2.prefill(0, ids=prompt, logits=False)
    preset = ocr.Preset("greedy_rp1.1", 0.0, 1.0, 1.1, 20, 0.0, n_new)
    got = gs2.decode_gpu(0, preset, prompt)
    assert len(got) == n_new
    assert gs2.n_past(0) == n_ctx - 1  # the last choice needs no row
    os2 = om.session(n_ctx)
    first = os2.prefill(prompt, None, len(prompt))
    want, margins = os2.decode(first, 1.1, 20, 0.0, prompt, n_new)
    k = next((i for i in range(n_new) if got[i] != want[i]), None)
    assert k is None, f"first divergence at choice {k}: device {got[k]} vs oracle {want[k]} (oracle top-2 margin {margins[k]})"


def test_frequency_penalty_decode_matches_oracle(ocr, orc, ctx, tiny):
    om, gm = tiny
    prompt = [int(t) for t in orc.fill_ids(6, 12, TINY["n_vocab"])]
    n_new = 60
    gs = gm.session(len(prompt) + n_new)
    gs.prefill(0, ids=prompt, logits=False)
    got = gs.decode_gpu(0, ocr.Preset("greedy_rp1.1_fp0.1", 0.0, 1.0, 1.1, 20, 0.1, n_new), prompt)
    os_ = om.session(len(prompt) + n_new)
    first = os_.prefill(prompt, None, len(prompt))
    want, margins = os_.decode(first, 1.1, 20, 0.1, prompt, n_new)
    assert got == want.tolist()


def test_embedding_rows_and_batch_equal_single(ocr, orc, ctx, tiny):
    """Input::Embeddings rows mixed with tokens; decode_batch == each slot decoded alone (same session shape)"""
    om, gm = tiny
    B, n_new = 3, 24
    rows = [int(t) for t in orc.fill_ids(8, 10, TINY["n_vocab"])]
    prompts = []
    for b in range(B):
        ids = np.array(rows[: 4 + b] + [-1] * 6 + rows[4 + b:], np.int32)
        embd = np.zeros((ids.size, TINY["dim"]), np.float32)
        embd[ids < 0] = ocr.gauss(100 + b, int((ids < 0).sum()) * TINY["dim"]).reshape(-1, TINY["dim"])
        prompts.append((ids, embd))
    preset = ocr.Preset("t", 0.0, 1.0, 1.15, 8, 0.0, n_new)
    hist = np.full((B, 8), 151655 % TINY["n_vocab"], np.int32)
    sa = gm.session(64, batch=B)
    sb = gm.session(64, batch=B)
    for b, (ids, embd) in enumerate(prompts):
        la = sa.prefill(b, ids=ids, embd=embd)
        sb.prefill(b, ids=ids, embd=embd, logits=False)
        os_ = om.session(64)
        lo = os_.prefill(ids, embd, ids.size)
        close_logits(la, lo)
    batch = sa.decode_batch(preset, hist)
    for b in range(B):
        single = sb.decode_gpu(b, preset, hist[b])
        assert single == batch[b].tolist(), b


def test_wide_batch_matches_oracle(ocr, orc, ctx):
    """a batch whose (slot, kv head) pairs outnumber the 16- and 8-CTA cluster splits (5 slots x 8 kv heads: 4-CTA
    clusters, one wave of 40): its first step and greedy choices as the oracle's per slot"""
    cfg = dict(n_layer=2, dim=256, n_head=16, n_kv=8, d_head=128, n_ff=512, n_vocab=1000, eps=1e-6, rope_base=1e6)
    B, n_new = 5, 12
    om = orc.Model(cfg, seed=43, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 43, 0.2, 1.0)
    prompts = [[int(t) for t in orc.fill_ids(20 + b, 10, cfg["n_vocab"])] for b in range(B)]
    sess = gm.session(48, batch=B)
    wants = []
    for b, prompt in enumerate(prompts):
        lg = sess.prefill(b, ids=prompt)
        os_ = om.session(48)
        lo = os_.prefill(prompt, None, len(prompt))
        close_logits(lg, lo)
        wants.append(os_.decode(lo, 1.1, 8, 0.0, prompt, n_new)[0].tolist())
    got = sess.decode_batch(ocr.Preset("t", 0.0, 1.0, 1.1, 8, 0.0, n_new), np.array(prompts, np.int32))
    for b in range(B):
        assert got[b].tolist() == wants[b], b


@pytest.mark.parametrize("shape", [
    dict(n_layer=2, dim=256, n_head=16, n_kv=16, d_head=128, n_ff=512, n_vocab=1000),  # 16 kv heads: unfused o-proj
    dict(n_layer=2, dim=1280, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000),   # dim > 1024: wide staging
])
def test_unfused_layer_matches_oracle(ocr, orc, ctx, shape):
    """shapes outside the fused layer (more than 8 kv heads, or rows wider than one float4 per staging thread) take
    the separate o-projection kernel and the multi-pass activation staging: step logits and greedy ids as the
    oracle's"""
    cfg = dict(shape, eps=1e-6, rope_base=1e6)
    om = orc.Model(cfg, seed=41, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 41, 0.2, 1.0)
    prompt = [int(t) for t in orc.fill_ids(15, 12, cfg["n_vocab"])]
    gs, osn = gm.session(48), om.session(48)
    lg, lo = gs.prefill(0, ids=prompt), osn.prefill(prompt, None, len(prompt))
    close_logits(lg, lo)
    for _ in range(6):
        t = int(np.argmax(lo))
        close_logits(gs.step([t])[0], lo := osn.step(t))
    gs2 = gm.session(48)
    gs2.prefill(0, ids=prompt, logits=False)
    got = gs2.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1.1, 20, 0.0, 30), prompt)
    os2 = om.session(48)
    want, margins = os2.decode(os2.prefill(prompt, None, len(prompt)), 1.1, 20, 0.0, prompt, 30)
    assert got == want.tolist()


def test_short_prefill_matches_oracle(ocr, orc, ctx, tiny):
    """prompts of up to 4 rows run as decode steps of their slot: token and embedding rows after a long prefill, and
    one row alone after a rewind (the benchmark's step) — logits as the oracle's prefill of the whole prompt"""
    om, gm = tiny
    dim = TINY["dim"]
    rows = [int(t) for t in orc.fill_ids(14, 12, TINY["n_vocab"])]
    ids = np.array(rows[:9] + [-1, rows[9], -1], np.int32)
    embd = np.zeros((ids.size, dim), np.float32)
    embd[ids < 0] = ocr.gauss(140, 2 * dim).reshape(-1, dim)
    lo = om.session(32).prefill(ids, embd, ids.size)
    gs = gm.session(32, batch=2)
    gs.prefill(1, ids=ids[:9], embd=embd[:9], logits=False)  # slot 1: the other slot must stay untouched
    lg = gs.prefill(1, ids=ids[9:], embd=embd[9:])
    close_logits(lg, lo)
    assert gs.n_past(1) == ids.size and gs.n_past(0) == 0
    gs.rewind(1, ids.size - 1)
    close_logits(gs.prefill(1, ids=ids[-1:], embd=embd[-1:]), lo)


def test_callback_stops_the_read(ocr, orc, ctx, tiny):
    om, gm = tiny
    prompt = [int(t) for t in orc.fill_ids(9, 16, TINY["n_vocab"])]
    preset = ocr.Preset("t", 0.0, 1.0, 1.1, 20, 0.0, 80)
    s1 = gm.session(120)
    s1.prefill(0, ids=prompt, logits=False)
    full = s1.decode_gpu(0, preset, prompt)
    seen = []
    s2 = gm.session(120)
    s2.prefill(0, ids=prompt, logits=False)
    got = s2.decode_gpu(0, preset, prompt, on_token=lambda t: (seen.append(t), len(seen) < 37)[1])
    assert got == full[:37] and seen == full[:37]


def test_profile_step_matches_step(ocr, orc, ctx, tiny):
    """the per-dispatch profiler runs the same step: 2 kernels per layer (the qkv and o projections fused into the
    attention, the FFN one kernel) + the LM head, positive times, the slot advances, and the logits it leaves equal a
    plain step's"""
    om, gm = tiny
    prompt = [int(t) for t in orc.fill_ids(12, 10, TINY["n_vocab"])]
    a, b = gm.session(32), gm.session(32)
    a.prefill(0, ids=prompt, logits=False)
    b.prefill(0, ids=prompt, logits=False)
    rec = a.profile_step([7])
    assert len(rec) == 2 * TINY["n_layer"] + 1
    assert [r["name"] for r in rec[:2]] == ["qkv + attention + o-proj", "ffn (gate|up, swiglu, down)"]
    assert rec[-1]["layer"] == -1 and all(r["us"] > 0 and r["bytes"] > 0 for r in rec)
    assert a.n_past(0) == b.n_past(0) + 1
    lb = b.step([7])[0]
    la = a.step([9])  # a's next step runs from the profiled step's state
    lb2 = b.step([9])[0]
    assert np.array_equal(la[0], lb2) and np.isfinite(lb).all()


def test_timeline_step_matches_step(ocr, orc, ctx, tiny):
    """the in-chain timeline of the one-slot step: the profiler's kernels, chained; positive in-chain times; the next
    step's logits equal a plain session's"""
    om, gm = tiny
    prompt = [int(t) for t in orc.fill_ids(12, 10, TINY["n_vocab"])]
    a, b = gm.session(32), gm.session(32)
    a.prefill(0, ids=prompt, logits=False)
    b.prefill(0, ids=prompt, logits=False)
    rec = a.timeline_step([7], reps=2)
    assert [r["name"] for r in rec] == [r["name"] for r in b.profile_step([7])]
    assert all(r["us"] > 0 for r in rec) and a.n_past(0) == b.n_past(0)
    assert np.array_equal(a.step([9])[0], b.step([9])[0])


def test_handles_release_in_any_order(ocr, orc):
    """a context outlives its handle while a model or session made in it lives (a garbage collector may release
    them in any order): the session still steps after the context and model handles are gone"""
    c = ocr.Context(0)
    m = ocr.TextModel.synthetic(c, text_config(ocr, TINY), 31, 0.2, 1.0)
    s = m.session(16)
    s.prefill(0, ids=[1, 2, 3], logits=False)
    c.close()
    m.close()
    lg = s.step([4])
    assert np.isfinite(lg).all() and s.n_past(0) == 4
    s.close()


def test_session_errors(ocr, ctx, tiny):
    om, gm = tiny
    s = gm.session(30)
    with pytest.raises(ocr.OcrError, match="no logits"):
        s.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1.1, 20, 0.0, 5), [1])
    with pytest.raises(ocr.OcrError, match="outside the vocabulary"):
        s.prefill(0, ids=[5, 1000])
    with pytest.raises(ocr.OcrError, match="overflow"):
        s.prefill(0, ids=list(range(31)))
    s.prefill(0, ids=list(range(25)), logits=False)
    with pytest.raises(ocr.OcrError, match="overflows"):
        s.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1.1, 20, 0.0, 10), [1])
    with pytest.raises(ocr.OcrError, match="positive normal"):
        s.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1e-40, 20, 0.0, 2), [1])
    with pytest.raises(ocr.OcrError, match="trained on"):
        gm.session(50000)


def test_config2_greedy_ids_match_oracle(ocr, ctx):
    """BASELINE config 2 at full size: 28 layers, 2048-row prefix, 512 greedy ids with rp 1.15 / window 64"""
    fx = json.loads((GOLDEN / "config2_greedy.json").read_text())
    from tests.golden.make_golden import config2_inputs

    seed, prefix, history = config2_inputs()
    assert seed == fx["seed"]
    m = ocr.TextModel.synthetic(ctx, text_config(ocr, fx["config"]), seed, fx["sigma_w"], fx["sigma_e"])
    s = m.session(2048 + 512)
    first = s.prefill(0, embd=prefix)
    top = np.argsort(-first, kind="stable")[:8]
    assert abs(float(np.abs(first).max()) - fx["first_max_abs"]) <= 2e-3 * fx["first_max_abs"]
    assert top[0] == fx["first_top8"][0]
    got = s.decode_gpu(0, ocr.Preset("c2", 0.0, 1.0, fx["rp"], fx["window"], 0.0, fx["max_new"]), history)
    want = fx["ids"]
    k = next((i for i in range(len(want)) if got[i] != want[i]), None)
    assert k is None, f"first divergence at choice {k}: device {got[k]} vs oracle {want[k]} (margin {fx['margins'][k]})"


def test_contexts_on_two_devices(ocr, orc, torch_cuda):
    """kernel attributes (the opt-in shared memory, 16-CTA clusters) are set per device: a process with a context on
    each of two GPUs decodes on both, the same ids as the oracle's"""
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    om = orc.Model(TINY, seed=31, sigma_w=0.2, sigma_e=1.0)
    prompt = [int(t) for t in orc.fill_ids(5, 20, TINY["n_vocab"])]
    os_ = om.session(64)
    want, _ = os_.decode(os_.prefill(prompt, None, len(prompt)), 1.1, 20, 0.0, prompt, 16)
    for dev in (1, 0):
        c = ocr.Context(dev)
        m = ocr.TextModel.synthetic(c, text_config(ocr, TINY), 31, 0.2, 1.0)
        s = m.session(64)
        s.prefill(0, ids=prompt, logits=False)
        got = s.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1.1, 20, 0.0, 16), prompt)
        assert got == want.tolist(), dev
        s.close()
        m.close()
        c.close()


@pytest.mark.parametrize("batch,slots", [(1, (0,)), (32, (0, 17))])
def test_config2_decode_logits_match_oracle_on_the_same_cache(ocr, orc, ctx, batch, slots):
    """BASELINE config 2's decode kernels at full size (28 x 1024, 16/8 heads, ffn 3072, vocab 151936), logits checked
    step by step (fused_decode_kernels_match_cpu, app/crates/ocr-wgpu/src/text.rs:863-975): the device's 2048-row
    prefill cache is copied into the oracle's session, then 4 decode steps on both — logits within 2e-3 of max |logit|
    and relative L2 1e-3 each step. batch 1 runs the compiled one-slot kernels (fused qkv + attention + o-projection,
    fused FFN, LM head); batch 32 with two live slots runs the tensor-core contractions and the batched attention."""
    from tests.golden.make_golden import CONFIG2, IMAGE_PAD, config2_inputs

    seed, prefix, _ = config2_inputs()
    m = ocr.TextModel.synthetic(ctx, text_config(ocr, CONFIG2), seed, 0.02, 0.02)
    om = orc.Model(CONFIG2, seed=seed, sigma_w=0.02, sigma_e=0.02)
    n_ctx, n_pre = 2048 + 8, 2048
    s = m.session(n_ctx, batch=batch)
    oss = {}
    for b in slots:
        rows = prefix if b == 0 else prefix[::-1].copy()  # two different prefixes
        s.prefill(b, embd=rows, logits=False)
        os_ = om.session(n_ctx)
        for layer in range(CONFIG2["n_layer"]):
            k, v = s.kv(layer, b, 0, n_pre)
            os_.set_kv(layer, 0, k, v)
        os_.n_past = n_pre
        oss[b] = os_
    toks = {b: IMAGE_PAD for b in slots}
    for _ in range(4):
        feed = [toks.get(b, -1) for b in range(batch)]
        lg = s.step(feed)
        for b in slots:
            lo = oss[b].step(toks[b])
            close_logits(lg[b], lo)
            toks[b] = int(np.argmax(lo))
