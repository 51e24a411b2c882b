"""The sm_100a kernels through the C ABI against the CPU oracle (B200 only).

Ports of the reference's GPU tests (app/crates/ocr-wgpu/src/text.rs): q8_0_matvec_and_matmul_match_cpu_dequant
(706-741), fused_decode_kernels_match_cpu (863-975), gpu_choice_matches_choose (1000-1054), choose_pen_is_exact
(1061-1099), the split decode attention of f16_paths_match_cpu (1258-1291); plus the repack's identity and the
reference penalty fixture. Tolerances: a dot product within 1e-5 of sum |w x| (f32 accumulation in another order);
attention relative L2 < 1e-5 (as text.rs:1291); the sampler and the penalty bit for bit.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def dev(torch, a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def host(torch, t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def device_matrix(torch, ocr, orc, rows, cols, seed, sigma):
    """(GGUF blocks, the device row layout built on the host)"""
    w = orc.synth_q8_0(rows * cols, seed, sigma)
    return w, dev(torch, ocr.q8_rows_from_blocks(w, rows, cols))


def test_repack_holds_the_same_values(ocr, orc, ctx, torch_cuda):
    torch = torch_cuda
    for rows, cols in [(37, 96), (3, 1024), (64, 3072)]:
        w = orc.synth_q8_0(rows * cols, 1234 + rows, 0.3)
        buf = torch.zeros(w.size + 2, dtype=torch.uint8, device="cuda")
        buf[2:] = torch.from_numpy(w).cuda()  # blocks at a 2-byte (not 4-byte) boundary
        stride = ocr.q8_row_bytes(cols)
        out = torch.full((rows * stride,), 0xAB, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ocr.op_repack_q8_0(ctx, buf.data_ptr() + 2, rows, cols, out.data_ptr())
        ctx.sync()
        got = host(torch, out).reshape(rows, stride)
        want = ocr.q8_rows_from_blocks(w, rows, cols)
        assert np.array_equal(got[:, :cols + cols // 16], want[:, :cols + cols // 16])
        b = w.reshape(rows, cols // 32, 34)
        assert np.array_equal(got[:, :cols].view(np.int8), b[:, :, 2:].reshape(rows, cols).view(np.int8))


def _norm_rows(orc, x, nw, eps):
    return np.stack([r * np.float32(orc.rms_scale(r, eps)) * nw for r in x]).astype(np.float32)


@pytest.mark.parametrize("rows,cols,nb,norm,acc", [
    (37, 96, 1, False, False), (37, 96, 1, True, True), (4096, 1024, 1, True, False), (1024, 3072, 1, False, True),
    (1024, 2048, 2, False, True), (6144, 1024, 4, True, False), (1000, 256, 8, True, False), (512, 1024, 32, False, True),
    (3, 3072, 3, True, False), (20011, 1024, 1, True, False), (151936, 1024, 1, False, False),
])
def test_matvec_matches_oracle(ocr, orc, ctx, torch_cuda, rows, cols, nb, norm, acc):
    torch = torch_cuda
    w, wd = device_matrix(torch, ocr, orc, rows, cols, 77 + rows + cols, 0.02)
    x = ocr.gauss(5 + nb, nb * cols, 1.0).reshape(nb, cols)
    nw = (1.0 + 0.1 * ocr.gauss(6, cols)).astype(np.float32)
    base = ocr.gauss(7, nb * rows, 1.0).reshape(nb, rows)
    xd, nwd, yd = dev(torch, x), dev(torch, nw), dev(torch, base.copy())
    ocr.op_matvec_q8_0(ctx, wd.data_ptr(), rows, cols, xd.data_ptr(), nwd.data_ptr() if norm else None, 1e-6, nb,
                       yd.data_ptr(), acc)
    ctx.sync()
    got = host(torch, yd)
    xn = _norm_rows(orc, x, nw, 1e-6) if norm else x
    deq = orc.dequantize_q8_0(w, rows * cols).reshape(rows, cols).astype(np.float64)
    for b in range(nb):
        want = orc.matvec_q8_0(w, rows, cols, xn[b], base[b] if acc else None)
        absdot = np.abs(deq) @ np.abs(xn[b].astype(np.float64))
        err = np.abs(got[b].astype(np.float64) - want)
        assert (err <= 1e-5 * absdot + 1e-6 + (np.abs(base[b]) * 1e-7 if acc else 0)).all(), (b, err.max())


def _lcg_uniform(ocr, seed, n):
    return ocr.gauss(seed, n, 1.0) / 3.0  # roughly [-1, 1]; any seeded spread serves


def choose_modes(ocr, seed, vocab, mode):
    u = _lcg_uniform(ocr, seed, 2 * vocab)
    if mode == 0:
        return np.round(u[:vocab] * 3).astype(np.float32)  # ties everywhere, -0 / +0 among them
    if mode == 1:
        return (u[:vocab] * 20).astype(np.float32)
    if mode == 2:
        l = (np.round(u[vocab:] * 2) - 1).astype(np.float32)
        l[u[:vocab] > 0.6] = -np.inf
        return l
    return (u[:vocab] * 1e-3).astype(np.float32)


CHOOSE_CASES = [
    (151936, 1.1, 20, 0.0, [5] * 30),
    (151936, 1.1, 20, 0.1, [3, 3, 9]),
    (1000, 1.0, 20, 0.0, []),
    (1000, 1.3, 1, 0.0, [1, 2]),
    (1000, 0.7, 7, 0.37, [0, 999, 0, 4, 4, 4, 17, 999]),
    (1000, 1.1, 64, 0.1, [(i * 7) % 13 for i in range(100)]),
    (257, 2.5, 3, 1.5, [256]),
]


@pytest.mark.parametrize("case", range(len(CHOOSE_CASES)))
def test_gpu_choice_matches_choose(ocr, orc, ctx, torch_cuda, case):
    """gpu_choice_matches_choose (text.rs:1000-1054): device choice vs ocr-decode's choose, step after step"""
    torch = torch_cuda
    vocab, rp, window, fp, seed_hist = CHOOSE_CASES[case]
    preset = ocr.Preset("t", 0.0, 1.0, rp, window, fp, 40)
    history = list(seed_hist)
    counts: dict[int, int] = {}
    for i in range(40):
        mode = i % 4
        l = choose_modes(ocr, 1000 * case + i, vocab, mode)
        if i == 7:
            l[:] = -np.inf  # all -inf: token 0
        if history:
            m = np.max(l)
            l[history[-1]] = np.float32(m + np.float32(0.05))  # the last token dominates: the penalties decide
        d = dev(torch, l)
        got = ocr.choose_gpu(ctx, d.data_ptr(), vocab, preset, history, counts)
        want, _ = orc.choose_greedy(l, rp, window, fp, history, counts)
        assert got == want, (case, i, mode)
        assert np.array_equal(host(torch, d).view(np.uint32), l.view(np.uint32))  # logits left unchanged
        history.append(want)
        counts[want] = counts.get(want, 0) + 1


def test_choose_nan_rules(ocr, orc, ctx, torch_cuda):
    torch = torch_cuda
    p = ocr.Preset("t", 0.0, 1.0, 1.0, 1, 0.0, 1)
    for l in ([1, np.nan, 5, np.nan], [np.nan, 1, 5], [np.nan] * 9, [-0.0, 0.0, -1.0], [2, 7, 7, 1]):
        a = np.array(l, np.float32)
        assert ocr.choose_gpu(ctx, dev(torch, a).data_ptr(), a.size, p, []) == orc.choose_greedy(a, 1.0, 1, 0.0, [])[0]


def test_penalty_is_exact(ocr, ctx, torch_cuda):
    """choose_pen_is_exact (text.rs:1061-1099), every product / quotient compared bit for bit"""
    torch = torch_cuda
    n = 8192
    s = np.uint64(3)
    bits = []
    with np.errstate(over="ignore"):
        for _i in range(n):
            s = s * np.uint64(6364136223846793005) + np.uint64(1442695040888963407)
            bits.append(int(s >> np.uint64(32)))
    l = np.empty(n, np.float32)
    for i, b in enumerate(bits):
        v = 0x0D800000 + b % (0x7F000000 - 0x0D800000) if i % 3 == 2 else b % 0x7F800000
        l[i] = np.array([v], np.uint32).view(np.float32)[0] * (-1 if i % 3 == 2 else 1)
    l[:6] = np.array([0.0, -0.0, np.inf, np.finfo(np.float32).max, np.uint32(1).view(np.float32),
                      np.finfo(np.float32).tiny], np.float32)
    hist = dev(torch, np.arange(n, dtype=np.int32))
    for rp in [1.1, 0.9, 1.0000001, 3.0, 1e-3, 1e3, 1.7e-30, 6.0e29]:
        r = np.float32(rp)
        d = dev(torch, l)
        ocr.op_penalize(ctx, d.data_ptr(), n, float(r), n, hist.data_ptr(), n)
        ctx.sync()
        with np.errstate(over="ignore", under="ignore", invalid="ignore"):
            want = np.where(l < 0, l * r, l / r).astype(np.float32)
        got = host(torch, d)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), rp


def test_penalty_matches_reference_fixture(ocr, ctx, torch_cuda):
    torch = torch_cuda
    from tests.golden.make_golden import penalty_logits

    fx = json.loads((GOLDEN / "penalty_ref.json").read_text())
    for c in fx["cases"]:
        l = penalty_logits(c["seed"], c["vocab"])
        hist = np.array(c["tail"] + c["out"], np.int32)
        d = dev(torch, l)
        h = dev(torch, hist)
        ocr.op_penalize(ctx, d.data_ptr(), c["vocab"], c["rp"], c["window"], h.data_ptr(), hist.size)
        ctx.sync()
        got = host(torch, d)
        changed = np.nonzero(got.view(np.uint32) != l.view(np.uint32))[0]
        assert changed.tolist() == c["changed"]
        assert got[changed].view(np.uint32).tolist() == c["values_bits"]
        p = ocr.Preset("t", 0.0, 1.0, c["rp"], c["window"], 0.0, 1)
        assert ocr.choose_gpu(ctx, dev(torch, l).data_ptr(), c["vocab"], p, hist.tolist()) == c["argmax"]


@pytest.mark.parametrize("vocab,window,rp", [(151936, 64, 1.15), (1000, 20, 1.1), (4099, 7, 0.7)])
def test_lm_head_sample_matches_oracle(ocr, orc, ctx, torch_cuda, vocab, window, rp):
    """dmv_norm + choose: logits within 2e-3 max|logit| (and 1e-5 sum|w x|); the token is choose() of those logits"""
    torch = torch_cuda
    dim = 1024
    w, wd = device_matrix(torch, ocr, orc, vocab, dim, 4242 + vocab, 0.02)
    x = ocr.gauss(17, dim, 1.0)
    nw = orc.fill_norm(18, dim)
    hist = ocr.fill_ids(19, 70, vocab)
    xd, nwd = dev(torch, x), dev(torch, nw)
    want = orc.matvec_q8_0(w, vocab, dim, x * np.float32(orc.rms_scale(x, 1e-6)) * nw)
    hist[-1] = int(np.argmax(want))  # the best token sits in the window: the penalty decides
    hd = dev(torch, np.concatenate([hist, np.zeros(4, np.int32)]))
    lend = dev(torch, np.array([hist.size], np.int32))
    tokd = dev(torch, np.zeros(1, np.int32))
    logits = torch.zeros(vocab, dtype=torch.float32, device="cuda")
    for rep in range(2):  # twice: the self-resetting counters
        lend.fill_(hist.size)
        torch.cuda.synchronize()
        ocr.op_lm_head_sample(ctx, wd.data_ptr(), vocab, dim, xd.data_ptr(), nwd.data_ptr(), 1e-6, rp, window,
                              hd.data_ptr(), lend.data_ptr(), tokd.data_ptr(), logits.data_ptr())
        ctx.sync()
        got = host(torch, logits)
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()
        deq = orc.dequantize_q8_0(w, vocab * dim).reshape(vocab, dim)
        absdot = np.abs(deq).astype(np.float64) @ np.abs(x * np.float32(orc.rms_scale(x, 1e-6)) * nw)
        assert (np.abs(got - want) <= 1e-5 * absdot + 1e-6).all()
        tok = int(host(torch, tokd)[0])
        assert tok == orc.choose_greedy(got, rp, window, 0.0, hist.tolist())[0]
        assert int(host(torch, lend)[0]) == hist.size + 1
        assert int(host(torch, hd)[hist.size]) == tok


ATTN_CASES = [(16, 8, 2560, 2303), (16, 8, 300, 299), (4, 2, 300, 0), (4, 2, 300, 127), (4, 2, 300, 128),
              (2, 1, 129, 128), (16, 8, 4096, 4095), (8, 8, 200, 150), (8, 1, 200, 199), (16, 4, 513, 511)]


@pytest.mark.parametrize("n_head,n_kv,n_ctx,pos", ATTN_CASES)
def test_attention_decode_matches_oracle(ocr, orc, ctx, torch_cuda, n_head, n_kv, n_ctx, pos):
    """qkv_post + attn_decode + attn_merge: out rel L2 < 1e-5, V row exact, K row within one f16 step"""
    torch = torch_cuda
    D = 128
    seed = n_head * 1000 + n_ctx + pos
    raw = (ocr.gauss(seed, (n_head + 2 * n_kv) * D, 3.0)).reshape(n_head + 2 * n_kv, D)
    qn, kn = orc.fill_norm(seed + 1, D), orc.fill_norm(seed + 2, D)
    cs = orc.rope_table(1e6, D, n_ctx)
    kf = ocr.gauss(seed + 3, n_kv * n_ctx * D, 2.0).reshape(n_kv, n_ctx, D)
    vf = ocr.gauss(seed + 4, n_kv * n_ctx * D, 1.0).reshape(n_kv, n_ctx, D)
    k16, v16 = kf.astype(np.float16), vf.astype(np.float16)
    kd, vd = dev(torch, k16.view(np.uint16).view(np.int16)), dev(torch, v16.view(np.uint16).view(np.int16))
    rawd, qnd, knd, csd = dev(torch, raw), dev(torch, qn), dev(torch, kn), dev(torch, cs)
    out = torch.zeros(n_head * D, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ocr.op_attention_decode(ctx, rawd.data_ptr(), qnd.data_ptr(), knd.data_ptr(), csd.data_ptr(), kd.data_ptr(),
                            vd.data_ptr(), n_head, n_kv, n_ctx, pos, 1e-6, out.data_ptr())
    ctx.sync()
    got = host(torch, out).reshape(n_head, D)
    gk = host(torch, kd).view(np.uint16).reshape(n_kv, n_ctx, D)
    gv = host(torch, vd).view(np.uint16).reshape(n_kv, n_ctx, D)
    # the oracle: the new rows, then softmax(q k / sqrt(128)) v over keys 0..pos
    kc, vc = k16.view(np.uint16).copy(), v16.view(np.uint16).copy()
    for j in range(n_kv):
        kr = orc.head_norm_rope(raw[n_head + j], kn, cs[pos], 1e-6)
        kc[j, pos] = orc.f16_from_f32(kr)
        vc[j, pos] = orc.f16_from_f32(raw[n_head + n_kv + j])
    assert np.array_equal(gv[:, pos], vc[:, pos])
    dk = np.abs(gk[:, pos].view(np.float16).astype(np.float32) - kc[:, pos].view(np.float16).astype(np.float32))
    assert (dk <= np.abs(kc[:, pos].view(np.float16).astype(np.float32)) * 2 ** -10 + 1e-7).all()
    # untouched rows stay
    keep = np.ones(n_ctx, bool)
    keep[pos] = False
    assert np.array_equal(gk[:, keep], kc[:, keep]) and np.array_equal(gv[:, keep], vc[:, keep])
    kc[:, pos] = gk[:, pos]  # attend over the device's own new key (checked above to one f16 step)
    g = n_head // n_kv
    want = np.stack([orc.attend(orc.head_norm_rope(raw[h], qn, cs[pos], 1e-6), kc[h // g].ravel(), vc[h // g].ravel(),
                                pos + 1, D, 1.0 / np.sqrt(128.0)) for h in range(n_head)])
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 1e-5, rel


def test_bounded_wait_runs_out_and_context_recovers(ocr, orc, torch_cuda):
    """a device wait that cannot complete gives up after its limit (no hang, no fault): the kernel reports it, the host
    sees OCR_ERR_DEVICE once, and the same context then runs normal work (the reference's Health rule: a device
    failure is an error, app/crates/ocr-wgpu/src/gpu.rs:901-970)"""
    torch = torch_cuda
    c = ocr.Context(0)
    try:
        assert ocr.op_wait_probe(c, 50) is True
        with pytest.raises(ocr.OcrError, match="bounded wait") as e:
            c.sync()
        assert e.value.code == 6
        c.sync()  # the flag was cleared with the report
        w = orc.synth_q8_0(64 * 256, 3, 0.02)
        wd = dev(torch, ocr.q8_rows_from_blocks(w, 64, 256))
        x = ocr.gauss(4, 256, 1.0)
        xd, yd = dev(torch, x), torch.zeros(64, device="cuda")
        ocr.op_matvec_q8_0(c, wd.data_ptr(), 64, 256, xd.data_ptr(), None, 1e-6, 1, yd.data_ptr(), False)
        c.sync()
        want = orc.matvec_q8_0(w, 64, 256, x, None)
        assert np.allclose(host(torch, yd), want, rtol=0, atol=1e-4)
    finally:
        c.close()
