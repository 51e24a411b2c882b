"""The batched decode path on the tensor cores (tcgen05) through the C ABI, against the CPU oracle.

Batches of more than 8 slots run their contractions (qkv, gate|up + SwiGLU, down + residual, the LM head + choice) as
skinny GEMMs on the tensor cores with f16 hi / lo splits of both operands (k_bgemm.cu). Checked here:
- ocr_op_matvec_q8_0 with nb > 8 (the same contraction with a plain store or residual add) against the oracle's
  matvec: within 1e-5 of sum |w x| per output, the CUDA-core matvec's bound (q8_0_matvec_and_matmul_match_cpu_dequant,
  app/crates/ocr-wgpu/src/text.rs:706-741) — partial 128-row tiles, two slot groups, K from 256 to 4096;
- whole decode steps of batches of 12 and 33 slots on a small qwen3-shaped model: prefill logits, per-step logits
  within the acceptance bound (2e-3 of max |logit|, relative L2 1e-3), and greedy ids equal to the oracle's and to the
  same slots decoded one at a time (the CUDA-core path).
"""
from __future__ import annotations

import numpy as np
import pytest

from test_gpu_decode import close_logits, text_config

pytestmark = pytest.mark.gpu


def dev(torch, a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def host(torch, t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("rows,cols,nb,norm,acc", [
    (512, 1024, 32, False, True), (4096, 1024, 32, True, False), (6144, 1024, 20, True, False),
    (1024, 3072, 32, False, True), (1000, 2048, 33, True, True), (300, 4096, 9, False, False),
    (130, 256, 16, True, False), (20011, 1024, 32, True, False),
])
def test_tensor_core_matvec_matches_oracle(ocr, orc, ctx, torch_cuda, rows, cols, nb, norm, acc):
    torch = torch_cuda
    w = orc.synth_q8_0(rows * cols, 91 + rows + cols, 0.02)
    wd = dev(torch, ocr.q8_rows_from_blocks(w, rows, cols))
    x = ocr.gauss(15 + nb, nb * cols, 1.0).reshape(nb, cols)
    x[:, ::17] *= 40.0  # a spread of magnitudes, so the hi / lo split of the activations matters
    nw = (1.0 + 0.1 * ocr.gauss(16, cols)).astype(np.float32)
    base = ocr.gauss(17, nb * rows, 1.0).reshape(nb, rows)
    xd, nwd, yd = dev(torch, x), dev(torch, nw), dev(torch, base.copy())
    ocr.op_matvec_q8_0(ctx, wd.data_ptr(), rows, cols, xd.data_ptr(), nwd.data_ptr() if norm else None, 1e-6, nb,
                       yd.data_ptr(), acc)
    ctx.sync()
    got = host(torch, yd)
    xn = np.stack([r * np.float32(orc.rms_scale(r, 1e-6)) * nw for r in x]).astype(np.float32) if norm else x
    deq = orc.dequantize_q8_0(w, rows * cols).reshape(rows, cols).astype(np.float64)
    worst = 0.0
    for b in range(nb):
        want = orc.matvec_q8_0(w, rows, cols, xn[b], base[b] if acc else None)
        absdot = np.abs(deq) @ np.abs(xn[b].astype(np.float64))
        err = np.abs(got[b].astype(np.float64) - want)
        bound = 1e-5 * absdot + 1e-6 + (np.abs(base[b]) * 1e-7 if acc else 0)
        assert (err <= bound).all(), (b, float((err / bound).max()))
        worst = max(worst, float((err / (absdot + 1e-30)).max()))
    print(f"worst |err| / sum|w x| = {worst:.2e}")


BATCH_CFG = dict(n_layer=3, dim=256, n_head=16, n_kv=8, d_head=128, n_ff=512, n_vocab=1000, eps=1e-6, rope_base=1e6)


@pytest.mark.parametrize("B,heads", [(12, (16, 8)), (33, (16, 8)), (9, (8, 8)), (10, (16, 4))])
def test_tensor_core_batch_decode_matches_oracle(ocr, orc, ctx, B, heads):
    """B slots of a 3-layer model (dim 256, ffn 512; 16/8, 8/8 or 16/4 heads: 1, 2 or 4 q heads per kv head, one CTA
    or several per (slot, kv head)): each slot's prompt prefilled, then (a) four CPU-choice
    steps of the whole batch — every slot's logits against the oracle's — and (b) the device-choice batched decode,
    whose ids must equal the oracle's greedy ids and those of the slots decoded one at a time"""
    cfg = dict(BATCH_CFG, n_head=heads[0], n_kv=heads[1])
    n_new, n_steps = 20, 4
    om = orc.Model(cfg, seed=47, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 47, 0.2, 1.0)
    prompts = [[int(t) for t in orc.fill_ids(60 + b, 8 + b % 5, cfg["n_vocab"])] for b in range(B)]
    n_ctx = 64
    # (a) the CPU-choice steps
    sa = gm.session(n_ctx, batch=B)
    osns, los = [], []
    for b, prompt in enumerate(prompts):
        lg = sa.prefill(b, ids=prompt)
        os_ = om.session(n_ctx)
        lo = os_.prefill(prompt, None, len(prompt))
        close_logits(lg, lo)
        osns.append(os_)
        los.append(lo)
    for _ in range(n_steps):
        toks = [int(np.argmax(lo)) for lo in los]
        lgs = sa.step(toks)
        for b in range(B):
            los[b] = osns[b].step(toks[b])
            close_logits(lgs[b], los[b])
    # (b) the device choice for the whole batch from the prompts' logits
    sb = gm.session(n_ctx, batch=B)
    wants = []
    for b, prompt in enumerate(prompts):
        sb.prefill(b, ids=prompt, logits=False)
        os_ = om.session(n_ctx)
        lo = os_.prefill(prompt, None, len(prompt))
        wants.append(os_.decode(lo, 1.1, 8, 0.0, prompt[-8:], n_new)[0].tolist())
    hist = np.array([p[-8:] for p in prompts], np.int32)
    got = sb.decode_batch(ocr.Preset("t", 0.0, 1.0, 1.1, 8, 0.0, n_new), hist)
    single = gm.session(n_ctx, batch=1)
    for b in range(B):
        assert got[b].tolist() == wants[b], (b, got[b].tolist(), wants[b])
        if b % 8 == 0:
            single.rewind(0, 0)
            single.prefill(0, ids=prompts[b], logits=False)
            assert single.decode_gpu(0, ocr.Preset("t", 0.0, 1.0, 1.1, 8, 0.0, n_new), hist[b]) == wants[b], b


@pytest.mark.parametrize("B", [12, 32])
def test_batched_attention_over_many_tiles(ocr, orc, ctx, B):
    """the batched attention's K/V ring wraps (260-row prefixes: 5 tiles of 64 keys for one CTA per (slot, kv head) at
    B = 32, several per CTA of a 3-way split at B = 12): four CPU-choice steps, every slot's logits against the
    oracle's"""
    cfg = BATCH_CFG
    om = orc.Model(cfg, seed=53, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 53, 0.2, 1.0)
    n_pre, n_ctx = 260, 272
    s = gm.session(n_ctx, batch=B)
    osns, los = [], []
    for b in range(B):
        embd = ocr.gauss(500 + b, n_pre * cfg["dim"]).reshape(n_pre, cfg["dim"])
        lg = s.prefill(b, embd=embd)
        os_ = om.session(n_ctx)
        lo = os_.prefill(None, embd, n_pre)
        close_logits(lg, lo)
        osns.append(os_)
        los.append(lo)
    for _ in range(4):
        toks = [int(np.argmax(lo)) for lo in los]
        lgs = s.step(toks)
        for b in range(B):
            los[b] = osns[b].step(toks[b])
            close_logits(lgs[b], los[b])


LAYER = ["qkv (tcgen05)", "attention (batched)", "o + residual (tcgen05)", "gate|up + swiglu (tcgen05)",
         "down + residual (tcgen05)"]


def test_tensor_core_profile_step(ocr, orc, ctx):
    """the profiler sees the batched step's kernels: layer 0's operand prep (the tokens' embedding rows, attn_norm),
    then per layer qkv, the batched attention, the o-projection, gate|up, down — the later norms built inside the
    qkv and gate|up contractions from the sums of squares the residual-adding ones leave — then the LM head's prep
    and contraction"""
    cfg = BATCH_CFG
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 47, 0.2, 1.0)
    s = gm.session(32, batch=16)
    for b in range(16):
        s.prefill(b, ids=[1 + b, 2, 3, 4, 5], logits=False)
    rec = s.profile_step([7] * 16)
    names = [r["name"] for r in rec]
    assert names == ["prep (embed, norm, hi/lo)"] + LAYER * cfg["n_layer"] + ["prep (norm, hi/lo)", "lm head (tcgen05)"]
    assert all(r["us"] > 0 for r in rec)


def test_prefill_attention_tensor_cores_match_f32_kernel(ocr, ctx, monkeypatch):
    """the prefill's causal attention on the tensor cores (Q and the probabilities split f16 hi / lo, two softmax
    passes) against the f32 kernel (OCR_PF_ATTN=0): a 200-row prefill then 173 embedding rows continuing at position
    200 (tiles of 128 queries and 64 keys, neither size a multiple), logits within 1e-5 of max |logit| after each,
    then the same 16 greedy choices"""
    cfg = BATCH_CFG
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 57, 0.2, 1.0)
    ids = [int(t) for t in ocr.fill_ids(58, 200, cfg["n_vocab"])]
    rows = ocr.gauss(59, 173 * cfg["dim"], 1.0).reshape(173, cfg["dim"])
    out = []
    for env in ("1", "0"):
        monkeypatch.setenv("OCR_PF_ATTN", env)
        s = gm.session(400)
        l1 = s.prefill(0, ids=ids)
        l2 = s.prefill(0, embd=rows)
        pre = ocr.Preset("t", 0.0, 1.0, 1.1, 16, 0.0, 16)
        out.append((l1, l2, s.decode_gpu(0, pre, ids[-16:])))
        s.close()
    monkeypatch.delenv("OCR_PF_ATTN")
    (a1, a2, ai), (b1, b2, bi) = out
    for a, b in ((a1, b1), (a2, b2)):
        m = np.abs(b).max()
        assert np.abs(a - b).max() <= 1e-5 * m, np.abs(a - b).max() / m
    assert ai == bi


def test_step_embd_equals_per_slot_prefill(ocr, ctx):
    """ocr_step_embd (one embedding row for every active slot in one step) leaves what a one-row prefill of each slot
    leaves: the same logits bit for bit, the same positions; an inactive slot does not move"""
    cfg = BATCH_CFG
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 51, 0.2, 1.0)
    a, b = gm.session(32, batch=16), gm.session(32, batch=16)
    for s in (a, b):
        for k in range(16):
            s.prefill(k, ids=[2 + k, 4, 6, 8, 10], logits=False)
    rows = ocr.gauss(77, 16 * cfg["dim"], 1.0).reshape(16, cfg["dim"])
    act = [1] * 16
    act[5] = 0
    la = a.step_embd(rows, act, logits=True)
    for k in range(16):
        if act[k]:
            lb = b.prefill(k, embd=rows[k:k + 1])
            assert np.array_equal(la[k], lb), k
    assert a.n_past(5) == 5 and a.n_past(0) == b.n_past(0) == 6
    nxt_a, nxt_b = a.step([9] * 16), b.step([9] * 16)
    assert np.array_equal(nxt_a, nxt_b)


def test_norms_inside_contractions_match_separate_prep(ocr, orc, ctx, monkeypatch):
    """the norms built inside the contractions (sums of squares per 128-row tile from the residual-adding
    contraction, added in tile order) against the separate prep kernel (OCR_NORM_IN=0; one CTA's sum per row): the
    same operand up to the order of the f32 sum of squares — logits within 1e-5 of max |logit| over 3 steps, and the
    same greedy ids over 24 choices for every slot"""
    cfg = BATCH_CFG
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 49, 0.2, 1.0)
    sa = gm.session(64, batch=16)
    monkeypatch.setenv("OCR_NORM_IN", "0")
    sb = gm.session(64, batch=16)
    monkeypatch.delenv("OCR_NORM_IN")
    assert len(sb.profile_step([-1] * 16)) == 7 * cfg["n_layer"] + 2  # (no slot active: the launches only)
    for s in (sa, sb):
        for b in range(16):
            s.prefill(b, ids=[3 + b, 5, 7, 11, 13, 17], logits=False)
    for t in range(3):
        la, lb = sa.step([20 + t] * 16), sb.step([20 + t] * 16)
        m = np.abs(lb).max()
        assert np.abs(la - lb).max() <= 1e-5 * m, np.abs(la - lb).max() / m
    pre = ocr.Preset("t", 0.0, 1.0, 1.1, 8, 0.0, 24)
    hist = np.full((16, 8), 3, np.int32)
    assert np.array_equal(sa.decode_batch(pre, hist), sb.decode_batch(pre, hist))


def test_tensor_core_timeline_step(ocr, orc, ctx):
    """the in-chain timeline runs the same launches as the profiler (chained, three times in one graph), every launch
    of the last repetition ends after the one before it, and the step leaves the state a plain step leaves: the next
    step's logits equal those of a session that took the step without the timeline"""
    cfg = BATCH_CFG
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 47, 0.2, 1.0)
    a, b = gm.session(32, batch=16), gm.session(32, batch=16)
    for s in (a, b):
        for k in range(16):
            s.prefill(k, ids=[1 + k, 2, 3, 4, 5], logits=False)
    rec = a.timeline_step([7] * 16, reps=3)
    prof = b.profile_step([7] * 16)
    assert [r["name"] for r in rec] == [r["name"] for r in prof]
    assert all(r["us"] > 0 for r in rec) and all(r["bytes"] == p["bytes"] for r, p in zip(rec, prof))
    assert a.n_past(0) == b.n_past(0) == 6
    la, lb = a.step([9] * 16), b.step([9] * 16)
    assert np.array_equal(la, lb)


# Below this top-2 gap (logit units; about 3e-5 of the largest |logit| here) the order of f32 summation decides the
# greedy choice: the oracle sums in f64, the device in f32 in another order. A device sequence may leave the oracle's at
# such a step only by taking the oracle's runner-up there (the comparison ends at that step); anywhere else the ids
# must be identical (read.rs:324-331 reports a divergence the same way: the step and both margins).
NEAR_TIE = 1e-4


def first_divergence(got, want):
    """None when identical; else the step where the device took the oracle's runner-up at a near-tie (asserts so)"""
    k = next((i for i in range(len(want["ids"])) if got[i] != want["ids"][i]), None)
    if k is not None:
        assert want["margins"][k] < NEAR_TIE and got[k] == want["runner_up"][k], (
            f"first divergence at choice {k}: device {got[k]} vs oracle {want['ids'][k]} (runner-up "
            f"{want['runner_up'][k]}, oracle top-2 margin {want['margins'][k]:.3g})")
    return k


def test_config3_batch_ids_match_oracle_and_single_slot(ocr, ctx):
    """BASELINE config 3 at full size: 32 slots, each a 3072-row prefix, 1024 greedy tokens with rp 1.15 over a
    64-token window, decoded as one batch on the tensor-core path. For the fixture's slots (0, 15, 31) the ids must be
    the oracle's (tests/golden/config3_greedy.json) — up to a swap at a near-tie — and so must the same slot's ids
    decoded alone (the one-slot CUDA-core path); at least one slot matches over all 1024 choices."""
    import json
    from pathlib import Path

    from tests.golden.make_golden import CONFIG2, CONFIG3_NEW, CONFIG3_PREFIX, config3_inputs

    fx = json.loads((Path(__file__).resolve().parent / "golden" / "config3_greedy.json").read_text())
    seed = fx["seed"]
    m = ocr.TextModel.synthetic(ctx, text_config(ocr, CONFIG2), seed, fx["sigma_w"], fx["sigma_e"])
    B = fx["batch"]
    s = m.session(CONFIG3_PREFIX + CONFIG3_NEW, batch=B)
    for b in range(B):
        _, prefix, history = config3_inputs(b)
        s.prefill(b, embd=prefix, logits=False)
    hist = np.full((B, 64), history[0], np.int32)
    preset = ocr.Preset("c3", 0.0, 1.0, fx["rp"], fx["window"], 0.0, fx["max_new"])
    got = s.decode_batch(preset, hist)
    s.close()
    one = m.session(CONFIG3_PREFIX + CONFIG3_NEW, batch=1)
    full = 0
    for key, want in fx["slots"].items():
        b = int(key)
        kb = first_divergence(got[b].tolist(), want)
        _, prefix, history = config3_inputs(b)
        one.rewind(0, 0)
        one.prefill(0, embd=prefix, logits=False)
        k1 = first_divergence(one.decode_gpu(0, preset, history), want)
        print(f"slot {b}: batch {'identical' if kb is None else f'near-tie swap at {kb}'}, one slot "
              f"{'identical' if k1 is None else f'near-tie swap at {k1}'}")
        full += kb is None
    assert full >= 1


@pytest.mark.parametrize("B", [12, 3])
def test_page_engine_matches_oracle_per_page(ocr, orc, ctx, B):
    """ocr_read_pages: 30 pages of different prompt lengths (token rows, some with embedding rows) and budgets
    through B slots, continuously batched (slots refilled as pages finish, budgets counted down on the device); every
    page's ids equal the oracle's greedy decode of that page alone"""
    cfg = BATCH_CFG
    om = orc.Model(cfg, seed=47, sigma_w=0.2, sigma_e=1.0)
    gm = ocr.TextModel.synthetic(ctx, text_config(ocr, cfg), 47, 0.2, 1.0)
    jobs = []
    for p in range(30):
        n = 3 + (p * 7) % 17  # 3 … 19 rows (a few of them short prompts, run as decode steps)
        ids = np.array([int(t) for t in orc.fill_ids(200 + p, n, cfg["n_vocab"])], np.int32)
        embd = None
        if p % 4 == 1:  # rows 1 and 2 as embeddings (Input::Embeddings)
            ids[1:3] = -1
            embd = np.zeros((n, cfg["dim"]), np.float32)
            embd[1:3] = ocr.gauss(300 + p, 2 * cfg["dim"]).reshape(2, -1)
        jobs.append(ocr.PageJob(p, embd, max_new=1 + (p * 5) % 23, ids=ids, history=[int(t) for t in ids[-8:] if t >= 0]))
    queue = list(jobs)
    done = {}
    sess = gm.session(64, batch=B)
    ocr.read_pages(sess, ocr.Preset("t", 0.0, 1.0, 1.1, 8, 0.0, 32), lambda: queue.pop(0) if queue else None,
                   lambda j: done.__setitem__(j.id, j.out.tolist()) or True, max_new_cap=32, chunk=5)
    assert sorted(done) == list(range(30))
    for j in jobs:
        os_ = om.session(64)
        lo = os_.prefill(j.ids, j.embd, j.ids.size)
        want = os_.decode(lo, 1.1, 8, 0.0, j.history, j.max_new)[0].tolist()
        assert done[j.id] == want, (j.id, done[j.id], want)
