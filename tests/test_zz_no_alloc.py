"""ocr_op_lm_head_sample_noalloc through the C ABI, against ocr_op_lm_head_sample (the scratch-allocating entry
point it mirrors): the same logits bit for bit, the same token, history and length, on two calls in a row (the
completion ticket must be back at zero for the second), and no device memory taken by the call.

Named to be collected last: it must pass both alone and after every other test has used the device.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    torch.cuda.synchronize()
    return t


def _host(torch, t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("vocab,window,rp", [(151936, 64, 1.15), (4099, 7, 0.7)])
def test_noalloc_lm_head_equals_lm_head(ocr, orc, torch_cuda, vocab, window, rp):
    torch = torch_cuda
    dim = 1024
    w = orc.synth_q8_0(vocab * dim, 777 + vocab, 0.02)
    wd = _dev(torch, ocr.q8_rows_from_blocks(w, vocab, dim))
    xd = _dev(torch, ocr.gauss(27, dim, 1.0))
    nwd = _dev(torch, orc.fill_norm(28, dim))
    hist = ocr.fill_ids(29, 70, vocab)

    def state():
        return (_dev(torch, np.concatenate([hist, np.zeros(4, np.int32)])),
                _dev(torch, np.array([hist.size], np.int32)), _dev(torch, np.zeros(1, np.int32)),
                torch.zeros(vocab, dtype=torch.float32, device="cuda"))

    ctx = ocr.Context(0)  # a fresh context: its memory ledger shows what the call allocates
    try:
        # one call on a throwaway state first: with lazy module loading the first launch loads the kernels' module
        # (and with it the static array, which the library holds from then on); the checks below are on later calls
        hw, lw, tw, gw = state()
        ocr.op_lm_head_sample_noalloc(ctx, wd.data_ptr(), vocab, dim, xd.data_ptr(), nwd.data_ptr(), 1e-6, rp,
                                      window, hw.data_ptr(), lw.data_ptr(), tw.data_ptr(), gw.data_ptr())
        ctx.sync()
        ha, la, ta, ga = state()
        hb, lb, tb, gb = state()
        for call in range(2):  # two in a row on the same state: the second decodes one token further
            before = ctx.memory()
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]  # the driver's count: sees any cudaMalloc, tracked or not
            ocr.op_lm_head_sample_noalloc(ctx, wd.data_ptr(), vocab, dim, xd.data_ptr(), nwd.data_ptr(), 1e-6, rp,
                                          window, ha.data_ptr(), la.data_ptr(), ta.data_ptr(), ga.data_ptr())
            ctx.sync()
            torch.cuda.synchronize()
            assert ctx.memory() == before, "the no-alloc call took device memory"
            assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc call changed the device's free memory"
            ocr.op_lm_head_sample(ctx, wd.data_ptr(), vocab, dim, xd.data_ptr(), nwd.data_ptr(), 1e-6, rp, window,
                                  hb.data_ptr(), lb.data_ptr(), tb.data_ptr(), gb.data_ptr())
            ctx.sync()
            assert np.array_equal(_host(torch, ga).view(np.uint32), _host(torch, gb).view(np.uint32)), call
            assert int(_host(torch, ta)[0]) == int(_host(torch, tb)[0]), call
            assert int(_host(torch, la)[0]) == int(_host(torch, lb)[0]) == hist.size + 1 + call
            assert np.array_equal(_host(torch, ha), _host(torch, hb)), call
        # and the second call's token is the CPU choice over its logits and the history the first one extended
        h = _host(torch, ha)
        want = orc.choose_greedy(_host(torch, ga), rp, window, 0.0, hist.tolist() + [int(h[hist.size])])[0]
        assert int(h[hist.size + 1]) == want
    finally:
        ctx.close()


def test_noalloc_rejects_null_and_bad_shape(ocr, torch_cuda):
    ctx = ocr.Context(0)
    try:
        with pytest.raises(ocr.OcrError, match="null"):
            ocr.op_lm_head_sample_noalloc(ctx, 0, 10, 64, 0, 0, 1e-6, 1.1, 4, 0, 0, 0, None)
        buf = torch_cuda.zeros(4096, dtype=torch_cuda.uint8, device="cuda")
        p = buf.data_ptr()
        with pytest.raises(ocr.OcrError, match="bad shape"):
            ocr.op_lm_head_sample_noalloc(ctx, p, 10, 48, p, 0, 1e-6, 1.1, 4, p, p, p, None)
    finally:
        ctx.close()
