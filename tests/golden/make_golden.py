"""Generate the committed golden fixtures under tests/golden/ (run here, in the container that mounts the reference).

    python tests/golden/make_golden.py penalty --reference-root DIR     → penalty_ref.json
    python tests/golden/make_golden.py config2                          → config2_greedy.json
    python tests/golden/make_golden.py config3                          → config3_greedy.json

penalty: the reference's own windowed repetition penalty — hf/window_rep_penalty.py's WindowRepetitionPenalty.apply
(b-straub/historic-htr-ocr, hf/window_rep_penalty.py:65-86) — run on torch CPU float32 logits. vllm is not installed,
so a stub provides the three names the module imports (SamplingParams, BatchUpdate / LogitsProcessor,
process_dict_updates); apply() itself runs unmodified. The logits are regenerated in the tests from their seed
(ocr_b200.gauss); the fixture holds the changed entries as f32 bit patterns and the greedy choice after the penalty.

config2: the CPU oracle's greedy decode of BASELINE config 2 (28 layers, dim 1024, 16/8 heads, ffn 3072, vocab
151936; q8_0 weights sigma 0.02 from the model seed; a 2048-row N(0,1) embedding prefix; 512 tokens with rp 1.15 over
a 64-token window seeded with 64 x <|image_pad|> = 151655). The fixture holds the ids and each step's top-2 margin, so
the GPU test needs no oracle run on the GPU host.

config3: the same oracle decode for slots 0, 15 and 31 of BASELINE config 3 (32 sequences on the config-2 decoder; slot
b's prefix is 3072 rows of gauss(substream(seed + b, 200000)); 1024 tokens each, rp 1.15, window 64 seeded with 64 x
<|image_pad|>), with each choice's top-2 margin and runner-up token: the batched GPU path's ids for those slots must
equal them (a swap at a near-tie is told apart from an error by the runner-up).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "historic-htr-ocr_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import ocr_b200 as P  # noqa: E402  (the synthetic data spec only: gauss / fill_ids / substream)

# BASELINE config 2 — shared with bench.py and the GPU tests
CONFIG2 = dict(n_layer=28, dim=1024, n_head=16, n_kv=8, d_head=128, n_ff=3072, n_vocab=151936, eps=1e-6,
               rope_base=1e6)
IMAGE_PAD = 151655


def config2_inputs():
    seed = P.SEED_BASE + 2
    prefix = P.gauss(P.substream(seed, 200000), 2048 * 1024, 1.0).reshape(2048, 1024)
    history = [IMAGE_PAD] * 64
    return seed, prefix, history


# ---- the reference's penalty ------------------------------------------------------------------------------------------
def _stub_vllm():
    vllm = types.ModuleType("vllm")

    class SamplingParams:  # the two fields the module reads
        def __init__(self, repetition_penalty=1.0, extra_args=None):
            self.repetition_penalty = repetition_penalty
            self.extra_args = extra_args

    vllm.SamplingParams = SamplingParams
    lp = types.ModuleType("vllm.v1.sample.logits_processor")

    class LogitsProcessor:
        pass

    class BatchUpdate:
        pass

    lp.LogitsProcessor = LogitsProcessor
    lp.BatchUpdate = BatchUpdate
    builtin = types.ModuleType("vllm.v1.sample.logits_processor.builtin")
    builtin.process_dict_updates = lambda reqs, batch_update, new_state: None
    for name, mod in [("vllm", vllm), ("vllm.v1", types.ModuleType("vllm.v1")),
                      ("vllm.v1.sample", types.ModuleType("vllm.v1.sample")),
                      ("vllm.v1.sample.logits_processor", lp),
                      ("vllm.v1.sample.logits_processor.builtin", builtin)]:
        sys.modules[name] = mod


def penalty_logits(seed: int, vocab: int) -> np.ndarray:
    """the test logits: N(0, 2) values, every 7th rounded to an integer (ties, ±0 among them)"""
    l = P.gauss(seed, vocab, 2.0)
    l[::7] = np.round(l[::7])
    l[3::11] = -l[3::11]
    return l.astype(np.float32)


PENALTY_CASES = [
    # (vocab, rp, window, prompt tail, output so far)
    (1000, 1.1, 20, [5] * 30, []),
    (1000, 1.1, 20, [3, 3, 9], [17, 3, 998]),
    (1000, 1.3, 1, [1, 2], [7]),
    (1000, 0.7, 7, [0, 999, 0, 4, 4, 4, 17, 999], [4, 0]),
    (1000, 1.15, 64, [int(x) for x in P.fill_ids(11, 100, 1000)], [int(x) for x in P.fill_ids(12, 40, 1000)]),
    (257, 2.5, 3, [256], [0, 256]),
    (151936, 1.15, 64, [151655] * 64, [int(x) for x in P.fill_ids(13, 70, 151936)]),
    (151936, 1.1, 20, [151655] * 20 + [151645, 198, 151644], [int(x) for x in P.fill_ids(14, 5, 151936)]),
]


def make_penalty(reference_root: Path) -> dict:
    import torch

    _stub_vllm()
    sys.path.insert(0, str(reference_root / "hf"))
    import window_rep_penalty as wrp  # the reference module, unmodified

    cases = []
    for i, (vocab, rp, win, tail, out) in enumerate(PENALTY_CASES):
        seed = 1000 + i
        l = penalty_logits(seed, vocab)
        proc = wrp.WindowRepetitionPenalty(None, torch.device("cpu"), False)
        proc.reqs = {0: (rp, win, list(tail[-win:]), list(out))}
        t = torch.from_numpy(l.copy()).reshape(1, vocab)
        got = proc.apply(t).reshape(vocab).numpy()
        changed = np.nonzero(got.view(np.uint32) != l.view(np.uint32))[0]
        best = 0
        for k in range(vocab):  # ocr-decode's argmax: the first maximum
            if got[k] > got[best]:
                best = k
        cases.append(dict(seed=seed, vocab=vocab, rp=rp, window=win, tail=list(tail), out=list(out),
                          changed=changed.tolist(), values_bits=got[changed].view(np.uint32).tolist(),
                          argmax=int(best)))
    return dict(source="hf/window_rep_penalty.py WindowRepetitionPenalty.apply (torch CPU f32, vllm stubbed)",
                logits="tests.golden.make_golden.penalty_logits(seed, vocab)", cases=cases)


def make_config2() -> dict:
    import oracle as O

    seed, prefix, history = config2_inputs()
    t0 = time.time()
    m = O.Model(CONFIG2, seed=seed, sigma_w=0.02, sigma_e=0.02)
    s = m.session(2048 + 512)
    first = s.prefill(None, prefix, 2048)
    t1 = time.time()
    ids, margins = s.decode(first, 1.15, 64, 0.0, history, 512)
    t2 = time.time()
    order = np.argsort(-first, kind="stable")[:8]
    return dict(config=CONFIG2, seed=seed, sigma_w=0.02, sigma_e=0.02, prefix="gauss(substream(seed, 200000), "
                "2048*1024, 1.0)", history=history, rp=1.15, window=64, max_new=512, ids=ids.tolist(),
                margins=[float(x) for x in margins], first_top8=order.tolist(),
                first_top8_logits=[float(first[k]) for k in order], first_max_abs=float(np.abs(first).max()),
                oracle_seconds=dict(prefill=round(t1 - t0, 1), decode=round(t2 - t1, 1)), threads=O.num_threads())


# 32 sequences on the config-2 decoder, each a 3072-row prefix and 1024 greedy tokens.
# The oracle decodes a subset of the slots at full length; the GPU test runs the whole batch and compares those.
CONFIG3_SLOTS = (0, 15, 31)
CONFIG3_PREFIX, CONFIG3_NEW = 3072, 1024


def config3_inputs(slot: int):
    """(model seed, slot's prefix rows, history): slot b's prefix is gauss(substream(seed + b, 200000)) rows"""
    seed = P.SEED_BASE + 2
    prefix = P.gauss(P.substream(seed + slot, 200000), CONFIG3_PREFIX * 1024, 1.0).reshape(CONFIG3_PREFIX, 1024)
    return seed, prefix, [IMAGE_PAD] * 64


def make_config3() -> dict:
    import oracle as O

    seed = P.SEED_BASE + 2
    m = O.Model(CONFIG2, seed=seed, sigma_w=0.02, sigma_e=0.02)
    slots = {}
    for b in CONFIG3_SLOTS:
        _, prefix, history = config3_inputs(b)
        t0 = time.time()
        s = m.session(CONFIG3_PREFIX + CONFIG3_NEW)
        first = s.prefill(None, prefix, CONFIG3_PREFIX)
        t1 = time.time()
        ids, margins, second = s.decode_top2(first, 1.15, 64, 0.0, history, CONFIG3_NEW)
        t2 = time.time()
        order = np.argsort(-first, kind="stable")[:8]
        slots[str(b)] = dict(ids=ids.tolist(), margins=[float(x) for x in margins], runner_up=second.tolist(),
                             first_top8=order.tolist(),
                             first_top8_logits=[float(first[k]) for k in order],
                             first_max_abs=float(np.abs(first).max()),
                             oracle_seconds=dict(prefill=round(t1 - t0, 1), decode=round(t2 - t1, 1)))
        print("slot", b, "done", round(t2 - t0, 1), "s", flush=True)
    return dict(config=CONFIG2, seed=seed, sigma_w=0.02, sigma_e=0.02, batch=32, prefix_rows=CONFIG3_PREFIX,
                prefix="slot b: gauss(substream(seed + b, 200000), 3072*1024, 1.0)", history=[IMAGE_PAD] * 64,
                rp=1.15, window=64, max_new=CONFIG3_NEW, slots=slots, threads=O.num_threads())


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["penalty", "config2", "config3"])
    ap.add_argument("--reference-root", default=os.environ.get("OCR_REFERENCE_ROOT"),
                    help="the reference checkout (or OCR_REFERENCE_ROOT); needed for `penalty` only")
    a = ap.parse_args()
    if a.what == "penalty":
        if not a.reference_root:
            ap.error("penalty needs --reference-root DIR (or OCR_REFERENCE_ROOT): the reference's hf/ directory")
        out = make_penalty(Path(a.reference_root))
        (HERE / "penalty_ref.json").write_text(json.dumps(out, indent=1))
    elif a.what == "config2":
        out = make_config2()
        (HERE / "config2_greedy.json").write_text(json.dumps(out))
    else:
        out = make_config3()
        (HERE / "config3_greedy.json").write_text(json.dumps(out))
    print("ok", a.what)
