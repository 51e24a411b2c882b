"""bench.py — decode throughput of the B200 q8_0 text-decode engine (libocrcuda.so).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3|2|1|5]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P \
        bench.py --gpus N --steps K --warmup W

Default workload (config 3, BASELINE.json configs[2] — the largest single-GPU decode config, the per-B200 figure): a
Qwen3-0.6B-shaped decoder (28 layers, dim 1024, 16/8 heads of 128, ffn 3072, vocab 151936, tied head) with seeded
synthetic q8_0 weights (sigma 0.02) generated on the device; 32 sequences per GPU, each with its f16 KV cache
prefilled (untimed) from 3072 seeded N(0,1) embedding rows; one step = a full greedy decode of 1024 tokens for all 32
sequences with the windowed repetition penalty (rp 1.15, window 64, seeded with 64 x <|image_pad|>) through the C ABI
(ocr_decode_batch: host history in, host ids out), preceded by re-feeding each prefix's last row (so every step starts
from the same logits). Pages are independent: at N GPUs every rank decodes its own batch (weak scaling, no data-path
collective); ranks only meet for the timing barrier and the max-over-ranks (gloo, host memory). The bytes streamed
per step (633 MB of weights, 13 GB of KV rows) exceed the 126 MB L2, so no flush is needed between steps. At one GPU
the line also carries config 2 (`config2`: one sequence, 2048-row prefix, 512 tokens) measured in the same run.

--config 2: one sequence per GPU, 2048-row prefix, 512 tokens.
--config 1: the LM head + windowed penalty + greedy argmax alone (ocr_op_lm_head_sample),
x N(0,1) [1024], W [151936 x 1024] N(0, 0.02) q8_0, history 512 uniform ids, penalty 1.15 over the last 64.
--config 4: one synthetic page end to end at batch 1 — a 1540 x 1100 RGB image (uniform bytes) baked
(white-padded to 1540 x 1120) and encoded by the Pixtral-shaped q8_0 vision encoder + projector (24 layers, 8800
patches → 2200 image tokens), prefilled between 7 + 7 prompt ids, then 1500 greedy tokens; time to first token
(encode + prefill + choice 0) and the decode rate reported separately.
--config 5: the page sweep — 512 seeded pages (prefix U[1500,3072] rows, U[800,1500] tokens) claimed
from a shared queue by one page engine per GPU (prefill included; strong scaling).

--impl reference: the reference's own path cannot run here (Rust + WGSL on wgpu: no Rust toolchain, no graphics
adapter), so the reference arm times the CPU restatement of it (oracle/, OpenMP on all host cores) on a bounded
sample of the same workload (decode steps at positions spread over the decode), on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "historic-htr-ocr_b200"))

CONFIG2 = dict(n_layer=28, dim=1024, n_head=16, n_kv=8, d_head=128, n_ff=3072, n_vocab=151936, eps=1e-6,
               rope_base=1e6)
IMAGE_PAD = 151655
PREFIX, NEW = 2048, 512


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def max_over_ranks(values, dist=None):
    """each value's maximum over the ranks (a gloo all-reduce of a host tensor; no data-path collective: the replicas
    only meet here and at the timing barrier) — the values themselves for one process"""
    import torch

    t = torch.tensor([float(v) for v in values], dtype=torch.float64)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def workload_config(config, B, new, prefix_len, world):
    """the `config` object of both arms' JSON lines"""
    return {"workload": f"BASELINE config {config}: greedy decode of {new} tokens per sequence, {B} sequence(s) per "
                        f"GPU, {prefix_len}-row prefilled f16 KV cache, rp 1.15 window 64",
            "model": "Qwen3-0.6B-shaped text decoder (28 x 1024, 16/8 heads, ffn 3072, vocab 151936, tied head)",
            "global_batch": B * world, "seq_len": prefix_len + new,
            "parallelism": f"replicas x{world} (pages partitioned, no collectives)",
            "l2": "inputs larger than L2 (633 MB of weights streamed per token)"}


def whole_job_rate(world, units_per_rank, seconds):
    """units of all replicas (weak scaling: each rank decodes its own sequences) over the slowest rank's time"""
    return world * units_per_rank / seconds


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, max, throttle reasons)"""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------------------------------------------------------------
# the LM head + sampler kernel timed alone (config 1, and the roofline of the dominant kernel)
# ---------------------------------------------------------------------------------------------------------------------
def lm_head_kernel(ocr, ctx, torch, reps: int, flush_bytes: int = 256 << 20):
    """(mean µs per launch, algorithmic bytes per launch): W 151936 x 1024 q8_0 (165,306,368 B) + x (4 KB) + norm
    (4 KB) + logits written (607,744 B) + the 64-token window; L2 flushed between launches (a 256 MB read)"""
    V, D = 151936, 1024
    g = torch.Generator(device="cuda").manual_seed(1)
    stride = ocr.q8_row_bytes(D)
    w = torch.zeros(V, stride, dtype=torch.uint8, device="cuda")
    w[:, :D] = torch.randint(-127, 128, (V, D), dtype=torch.int8, device="cuda", generator=g).view(torch.uint8)
    w[:, D:D + D // 16] = (torch.rand(V, D // 32, device="cuda", generator=g) * 0.0003 + 0.0001).half() \
        .view(torch.uint8)
    x = torch.randn(D, device="cuda", generator=g)
    nw = torch.ones(D, device="cuda")
    hist = torch.randint(0, V, (512 + reps + 8,), dtype=torch.int32, device="cuda", generator=g)
    ln = torch.tensor([512], dtype=torch.int32, device="cuda")
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    logits = torch.empty(V, device="cuda")
    flush = torch.zeros(flush_bytes // 4, device="cuda")
    stream = torch.cuda.ExternalStream(ctx.stream())
    torch.cuda.synchronize()
    times = []
    for i in range(reps + 3):
        float(flush.sum())  # a read larger than L2 (a write would leave dirty lines to drain during the launch)
        ln.fill_(512)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ocr.op_lm_head_sample(ctx, w.data_ptr(), V, D, x.data_ptr(), nw.data_ptr(), 1e-6, 1.15, 64, hist.data_ptr(),
                              ln.data_ptr(), tok.data_ptr(), logits.data_ptr())
        b.record(stream)
        b.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b) * 1e3)
    ctx.sync()
    algo = V * D + V * (D // 32) * 2 + 2 * D * 4 + V * 4 + 64 * 4
    return sum(times) / len(times), algo


def kernel_classes(sess, B, prefix_len, last_rows, steps=4):
    """in-chain per-kernel times of the decode step (ocr_timeline_step: the step's launches chained as the timed
    graph chains them, %globaltimer at every CTA's end; a launch's time is its latest CTA end less the previous
    launch's, the last of 3 chained repetitions), grouped by kernel class: launches, mean µs, algorithmic bytes per
    launch, share of the step"""
    for b in range(B):
        sess.rewind(b, prefix_len - 1)
        sess.prefill(b, embd=last_rows[b], logits=False)
    agg = {}
    for i in range(steps):
        for k in sess.timeline_step([IMAGE_PAD] * B, reps=3):
            a = agg.setdefault(k["name"], [0, 0.0, 0.0])
            a[0] += 1
            a[1] += k["us"]
            a[2] += k["bytes"]
    tot = sum(a[1] for a in agg.values())
    peak, _ = peaks()
    out = []
    for name, (n, us, by) in sorted(agg.items(), key=lambda x: -x[1][1]):
        gbs = by / (us * 1e-6) / 1e9
        out.append({"kernel": name, "launches": n, "us_per_launch": round(us / n, 2),
                    "bytes_per_launch": round(by / n), "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                    "share": round(us / tot, 4)})
    return out


def kernel_roofline(classes):
    """the roofline object for the dominant class (largest share of the step's device time)"""
    peak, which = peaks()
    top = classes[0]
    traffic = None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get(top["kernel"])
    return {"kernel": top["kernel"], "bound": "hbm", "achieved": top["achieved_gbs"], "peak": peak, "unit": "GB/s",
            "frac": top["frac"], "peak_source": f"{which} hbm_gbs (of {which})", "traffic": traffic,
            "us_per_launch": top["us_per_launch"], "algorithmic_bytes_per_launch": top["bytes_per_launch"],
            "share_of_step": top["share"], "timing": "in-chain (%globaltimer per CTA, ocr_timeline_step)"}


# ---------------------------------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------------------------------
# the decode workloads: slots per GPU, prefix rows per slot, tokens decoded per slot (BASELINE configs[1] and [2])
WORKLOADS = {2: dict(B=1, prefix=PREFIX, new=NEW), 3: dict(B=32, prefix=3072, new=1024),
             4: dict(B=1, prefix=2214, new=1500), 5: dict(B=32, prefix=2286, new=1150)}  # (config 5: its mean page, for the CPU samples' positions)


def decode_workload(ocr, ctx, torch, config, steps, warmup, pg, local, tokens=0, prefix=0, profile_range=False):
    """one replica's decode throughput on a config: the model, each slot's prefix prefilled (untimed), then `steps`
    timed steps of a full greedy decode of every slot through the C ABI (host history in, host ids out). Returns the
    timing and the session (for the per-kernel profile). `tokens` / `prefix` shrink the workload for profiler
    captures; `profile_range` brackets the first timed step with cudaProfilerStart / Stop (ncu
    --profile-from-start off captures that step's launches only)."""
    w = WORKLOADS[config]
    B, prefix_len, new = w["B"], prefix or w["prefix"], tokens or w["new"]
    seed = ocr.SEED_BASE + 2
    model = ocr.TextModel.synthetic(ctx, ocr.TextConfig(**CONFIG2), seed, 0.02, 0.02)
    sess = model.session(prefix_len + new, batch=B)
    # the prefill of every slot's prefix (untimed for the decode metric; its own time reported beside it: device
    # events around each slot's prefill, the rows generated on the host before)
    stream0 = torch.cuda.ExternalStream(ctx.stream())
    pf_ms = 0.0
    for b in range(B):
        embd = ocr.gauss(ocr.substream(seed + b, 200000), prefix_len * 1024, 1.0).reshape(prefix_len, 1024)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream0)
        sess.prefill(b, embd=embd, logits=False)
        e1.record(stream0)
        e1.synchronize()
        pf_ms += e0.elapsed_time(e1)
    last_rows = [ocr.gauss(ocr.substream(seed + b, 200000), 1024, 1.0, start=(prefix_len - 1) * 1024)
                 for b in range(B)]
    preset = ocr.Preset("bench", 0.0, 1.0, 1.15, 64, 0.0, new)
    hist = np.full((B, 64), IMAGE_PAD, np.int32)
    stream = torch.cuda.ExternalStream(ctx.stream())

    last_block = np.stack(last_rows).astype(np.float32)

    def step():
        # every slot back to its prefix, the last prefix row re-fed (every step starts from the same logits): one
        # batched step of all slots' rows (ocr_step_embd), or the slot's one-row prefill
        for b in range(B):
            sess.rewind(b, prefix_len - 1)
        if B > 1:
            sess.step_embd(last_block)
        else:
            sess.prefill(0, embd=last_rows[0], logits=False)
        if B == 1:
            return sess.decode_gpu(0, preset, hist[0])
        return sess.decode_batch(preset, hist)

    for _ in range(warmup):
        step()
    ctx.sync()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        ev0.record(stream)
        for i in range(steps):
            if profile_range and i == 0:
                torch.cuda.profiler.start()
            step()
            if profile_range and i == 0:
                torch.cuda.synchronize()
                torch.cuda.profiler.stop()
        ev1.record(stream)
        ev1.synchronize()
        wall = time.perf_counter() - t0
    dev_s, wall = max_over_ranks([ev0.elapsed_time(ev1) / 1e3, wall], pg)
    return dict(B=B, prefix=prefix_len, new=new, dev_s=dev_s, wall=wall, clocks=clk.summary(), sess=sess,
                model=model, last_rows=last_rows,
                prefill={"rows": B * prefix_len, "rows_per_slot": prefix_len, "ms": round(pf_ms, 1),
                         "rows_per_s": round(B * prefix_len / (pf_ms * 1e-3), 1),
                         "note": "each slot's prefix prefilled through ocr_prefill (Input::Embeddings rows): the "
                                 "projections on the tensor cores (three groups of 32 rows per CTA), the causal "
                                 "attention on the tensor cores; device time, untimed for the decode metric"})


def run_ours(args):
    import torch

    import ocr_b200 as ocr

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        pg = dist
    ctx = ocr.Context(local)
    if args.config == 1:
        return run_config1(args, ocr, ctx, torch, pg, rank, world)
    if args.config == 5:
        return run_config5(args, ocr, ctx, torch, pg if pg else None, rank, world, local)
    if args.config == 4:
        return run_config4(args, ocr, ctx, torch, pg, rank, world, local)
    r = decode_workload(ocr, ctx, torch, args.config, args.steps, args.warmup, pg, local, args.tokens, args.prefix,
                        args.profile_range)
    B, prefix_len, new, dev_s, wall = r["B"], r["prefix"], r["new"], r["dev_s"], r["wall"]
    tokens = world * B * new * args.steps
    out = None
    if rank == 0:
        classes = kernel_classes(r["sess"], B, prefix_len, r["last_rows"])
        # per step: the re-feed of the slots' last prefix rows (one batched step), choice 0, then new - 1 decode
        # steps; a decode step's launches as the timeline counted them (kernels per layer + the LM head / choice)
        launches_per_token = sum(k["launches"] for k in classes) // 4
        launches = args.steps * (launches_per_token + 1 + (new - 1) * launches_per_token)
        roof = kernel_roofline(classes)
        out = {
            "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
            "value": round(whole_job_rate(world, B * new * args.steps, dev_s), 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_s / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights x f32 activations, f16 KV",
            "data": "synthetic (seeded q8_0 weights sigma 0.02, N(0,1) prefix embeddings; no checkpoint)",
            "config": workload_config(args.config, B, new, prefix_len, world),
            "e2e": {"value": round(tokens / wall, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": B * (64 * 4 + 1024 * 4), "d2h_bytes_per_step": B * new * 4},
            "gpu_launches": int(launches),
            "roofline": roof,
            "kernels": classes,
            "clocks": r["clocks"],
            "prefill": r["prefill"],
        }
    r["sess"].close()
    r["model"].close()
    if rank == 0:
        lm_us, lm_bytes = lm_head_kernel(ocr, ctx, torch, 10)
        out["lm_head_alone"] = {"us_per_launch": round(lm_us, 2), "achieved_gbs": round(lm_bytes / lm_us / 1e3, 1),
                                "note": "the LM head + penalty + argmax kernel timed alone after a 256 MB L2 read"}
        if world == 1 and args.config == 3 and not args.no_secondary:
            # BASELINE config 2 (one sequence per GPU) measured in the same run, reported beside the headline
            r2 = decode_workload(ocr, ctx, torch, 2, 3, 3, None, local)
            c2 = kernel_classes(r2["sess"], 1, r2["prefix"], r2["last_rows"])
            out["config2"] = {"value": round(r2["new"] * 3 / r2["dev_s"], 1), "unit": "tok/s",
                              "ms_per_step": round(r2["dev_s"] / 3 * 1e3, 3), "steps": 3, "warmup": 3,
                              "workload": workload_config(2, 1, r2["new"], r2["prefix"], 1)["workload"],
                              "roofline": kernel_roofline(c2), "kernels": c2}
            r2["sess"].close()
            r2["model"].close()
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline_sample(args.config, tokens_sample=16)
        print(json.dumps(out), flush=True)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    ctx.close()
    return out


def run_config5(args, ocr, ctx, torch, pg, rank, world, local):
    """the page sweep. 512 seeded pages (prefix rows uniform on [1500, 3072], 800 … 1500 tokens
    each) claimed by the ranks from a shared queue (the process group's store: no data-path collective), each rank
    reading its pages through its GPU's page engine (ocr_read_pages: 32 slots, continuous batching; prefill of each
    page's rows included). Whole-box tokens over the slowest rank's device time; strong scaling (the pages are fixed)."""
    import pages as P

    seed = ocr.SEED_BASE + 5
    n_pages = args.pages or P.N_PAGES
    specs = P.page_specs(seed, n_pages)
    pool = P.page_pool(seed, CONFIG2["dim"])
    model = ocr.TextModel.synthetic(ctx, ocr.TextConfig(**CONFIG2), ocr.SEED_BASE + 2, 0.02, 0.02)
    sess = model.session(P.PREFIX_MAX + P.GEN_MAX, batch=32)
    preset = ocr.Preset("c5", 0.0, 1.0, 1.15, 64, 0.0, P.GEN_MAX)
    hist = [IMAGE_PAD] * 64
    store = pg.distributed_c10d._get_default_store() if pg else P.LocalStore()
    stream = torch.cuda.ExternalStream(ctx.stream())

    def sweep(ns, page_ids):
        q = P.PageQueue(store, rank, world, len(page_ids), ns=ns)

        def read(claim, done):
            def source():
                i = claim()
                if i is None:
                    return None
                sp = specs[page_ids[i]]
                return ocr.PageJob(i, pool[sp.row0: sp.row0 + sp.prefix], sp.new, history=hist)

            def on_done(job):
                return done(job.id, len(job.out))

            ocr.read_pages(sess, preset, source, on_done, max_new_cap=P.GEN_MAX, chunk=16)

        mine = P.run_worker(read, q)
        return q, mine

    # warm-up: a few pages (one-time setup, graph capture)
    sweep("warm/", [p % n_pages for p in range(2 * world)])
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        ev0.record(stream)
        q, mine = sweep("sweep/", list(range(n_pages)))
        ev1.record(stream)
        ev1.synchronize()
        wall = time.perf_counter() - t0
    dev_s, wall = max_over_ranks([ev0.elapsed_time(ev1) / 1e3, wall], pg)
    tokens = q.tokens()
    out = None
    if rank == 0:
        out = {
            "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
            "value": round(tokens / dev_s, 1), "unit": "tok/s", "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": round(dev_s * 1e3, 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q8_0 weights x f32 activations, f16 KV",
            "data": "synthetic (seeded q8_0 weights, N(0,1) prefix rows; no checkpoint)",
            "config": {"workload": f"BASELINE config 5: {n_pages} pages (prefix U[1500,3072] rows, U[800,1500] tokens), "
                                   "prefill + greedy decode, 32 slots per GPU, continuous batching",
                       "model": "Qwen3-0.6B-shaped text decoder (28 x 1024, 16/8 heads, ffn 3072, vocab 151936)",
                       "global_batch": 32 * world, "parallelism": f"replicas x{world}, pages claimed from a shared queue"},
            "pages": n_pages, "tokens": tokens, "prefix_rows": sum(s.prefix for s in specs),
            "pages_read_rank0": mine,
            "e2e": {"value": round(tokens / wall, 1), "unit": "tok/s",
                    "h2d_bytes_per_step": sum(s.prefix for s in specs) * CONFIG2["dim"] * 4 + n_pages * 64 * 4,
                    "d2h_bytes_per_step": tokens * 4},
            "clocks": clk.summary()}
        print(json.dumps(out), flush=True)
    P.PageQueue(store, rank, world, n_pages, ns="sweep/").leave()
    sess.close()
    model.close()
    return out


PAGE_W, PAGE_H, PROMPT_PRE, PROMPT_POST = 1540, 1100, 7, 7


def run_config4(args, ocr, ctx, torch, pg, rank, world, local):
    """one page end to end at batch 1 (Engine::read_text, engine.rs:447-524). A step: the page's
    bytes (pinned host memory) baked and encoded (ocr_vision_encode_page: the white pad inside the patch gather, 24
    encoder layers on 8800 patches, the projector → 2200 rows left on the device), the prompt [7 ids, 2200 image
    rows, 7 ids] prefilled from the device rows, choice 0, then 1500 greedy choices (ocr_decode: host history in,
    host ids out). TTFT = encode + prefill (device events); the decode rate over the 1500 choices after it."""
    seed = ocr.SEED_BASE + 4
    vcfg = ocr.VisionConfig()
    vision = ocr.Vision.synthetic(ctx, vcfg, seed, 0.02)
    model = ocr.TextModel.synthetic(ctx, ocr.TextConfig(**CONFIG2), ocr.SEED_BASE + 2, 0.02, 0.02)
    g = 28
    sw, sh, left, top, right, bottom = ocr.bake_plan(vcfg.image_size, g, PAGE_W, PAGE_H)
    n_img = ((sw + left + right) // g) * ((sh + top + bottom) // g)
    rng = np.random.default_rng(seed)
    page = torch.from_numpy(rng.integers(0, 256, (PAGE_H, PAGE_W, 3), dtype=np.uint8)).pin_memory()
    ids_pre = [int(t) for t in rng.integers(0, CONFIG2["n_vocab"], PROMPT_PRE)]
    ids_post = [int(t) for t in rng.integers(0, CONFIG2["n_vocab"], PROMPT_POST)]
    ids = ids_pre + [-1] * n_img + ids_post
    n_prompt, new = len(ids), args.tokens or WORKLOADS[4]["new"]
    rows = torch.zeros((n_prompt, CONFIG2["dim"]), dtype=torch.float32, device="cuda")
    img_rows = rows[PROMPT_PRE:PROMPT_PRE + n_img]
    sess = model.session(n_prompt + new)
    preset = ocr.Preset("page", 0.0, 1.0, 1.15, 64, 0.0, new)
    history = [IMAGE_PAD] * n_img + ids_post
    stream = torch.cuda.ExternalStream(ctx.stream())
    page_np = page.numpy()

    def read(ev):
        sess.rewind(0, 0)
        ev[0].record(stream)
        vision.encode_page(page_np, out=img_rows)
        ev[1].record(stream)
        sess.prefill(0, ids=ids, embd=rows, logits=False)
        ev[2].record(stream)
        out = sess.decode_gpu(0, preset, history)
        ev[3].record(stream)
        ev[3].synchronize()
        return out

    def events():
        return [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    for _ in range(args.warmup):
        read(events())
    torch.cuda.synchronize()
    enc, pf, dec, tot = [], [], [], []
    with Clocks(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ev = events()
            out = read(ev)
            assert len(out) == new
            enc.append(ev[0].elapsed_time(ev[1]))
            pf.append(ev[1].elapsed_time(ev[2]))
            dec.append(ev[2].elapsed_time(ev[3]))
            tot.append(ev[0].elapsed_time(ev[3]))
        wall = time.perf_counter() - t0
    k = args.steps
    dev_s = sum(tot) / 1e3
    dev_s, wall = max_over_ranks([dev_s, wall], pg)
    decode_rate = new * k / (sum(dec) / 1e3)
    ttft = (sum(enc) + sum(pf)) / k
    out = None
    if rank == 0:
        flops_vit = 24 * (2 * 8800 * (4 * 1024 * 1024 + 3 * 4096 * 1024) + 4 * 8800 * 8800 * 1024)
        out = {
            "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
            "value": round(world * decode_rate, 1), "unit": "tok/s", "n_gpus": world, "steps": k,
            "warmup": args.warmup, "ms_per_step": round(dev_s / k * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights x f32 activations (f16 hi/lo tensor-core "
                                                           "operands), f16 KV",
            "data": "synthetic (seeded 1540x1100 RGB page, uniform bytes; seeded q8_0 vision and text weights)",
            "config": {"workload": f"BASELINE config 4: one page end to end at batch 1 — bake to {sw + left + right}x"
                                   f"{sh + top + bottom}, Pixtral-shaped q8_0 encoder (24 x 1024, 16 heads of 64, "
                                   f"ffn 4096) + projector → {n_img} image rows, prompt {n_prompt} rows, {new} greedy "
                                   "tokens (rp 1.15, window 64)",
                       "model": "vision: Pixtral ViT + LightOnOCR projector; text: Qwen3-0.6B-shaped decoder",
                       "global_batch": world, "seq_len": n_prompt + new, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (633 MB of text weights per token; 0.86 GB of vision weights and "
                             "activations per page)"},
            "ttft": {"ms": round(ttft, 2), "encode_ms": round(sum(enc) / k, 2), "prefill_ms": round(sum(pf) / k, 2),
                     "image_rows": n_img, "prompt_rows": n_prompt,
                     "encode_tflops": round(flops_vit / (sum(enc) / k * 1e-3) / 1e12, 1),
                     "note": "device events on the library's stream: encode (the page's host-to-device copy, the bake's "
                             "pad fused into the patch gather, 24 layers, the projector) + prefill (the prompt's last "
                             "logits); choice 0 is the decode's first kernel"},
            "decode": {"tok_per_s": round(decode_rate, 1), "ms": round(sum(dec) / k, 1), "tokens": new},
            "e2e": {"value": round(world * new * k / wall, 1), "unit": "tok/s (whole page read, TTFT included)",
                    "h2d_bytes_per_step": PAGE_W * PAGE_H * 3 + len(ids) * 4 + len(history) * 4,
                    "d2h_bytes_per_step": new * 4},
            "clocks": clk.summary()}
        if not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_baseline_sample(4, tokens_sample=16)
            enc = cpu_encode_sample()
            n_patches = ((sw + left + right) // vcfg.patch) * ((sh + top + bottom) // vcfg.patch)
            enc["gpu_patches_per_s"] = round(n_patches / (out["ttft"]["encode_ms"] * 1e-3), 1)
            out["cpu_encode"] = enc
        print(json.dumps(out), flush=True)
    sess.close()
    model.close()
    vision.close()
    return out


def run_config1(args, ocr, ctx, torch, pg, rank, world):
    us_list = []
    with Clocks(int(os.environ.get("LOCAL_RANK", 0))) as clk:
        us, algo = lm_head_kernel(ocr, ctx, torch, args.steps)
    peak, which = peaks()
    if rank == 0:
        gbs = algo / (us * 1e-6) / 1e9
        print(json.dumps({
            "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
            "value": round(world * 1e6 / us, 1), "unit": "choices/s", "n_gpus": world, "steps": args.steps,
            "warmup": 3, "ms_per_step": round(us / 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q8_0 x f32", "data": "synthetic",
            "config": {"workload": "BASELINE config 1: LM head 151936 x 1024 q8_0 + windowed penalty + argmax",
                       "l2": "flushed between launches (a 256 MB read)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": which, "traffic": None},
            "cpu_baseline": None if args.no_cpu_baseline else cpu_baseline_sample(1, 200),
            "clocks": clk.summary()}), flush=True)
    del us_list
    return None


# ---------------------------------------------------------------------------------------------------------------------
# the CPU baseline (the oracle: the reference's path restated, OpenMP on all host cores)
# ---------------------------------------------------------------------------------------------------------------------
def cpu_positions(config: int, n: int) -> list[int]:
    """n decode positions spread evenly over the config's decode (prefix .. prefix + new - 1): the sampled tokens see
    the same mean key count as the GPU arm's full decode"""
    w = WORKLOADS[config]
    return [w["prefix"] + (w["new"] * i) // n for i in range(n)]


class CpuDecode:
    """the oracle's decode (the reference's path restated, OpenMP on all host cores) on a config's model: timed runs of
    single-token steps at positions spread over the config's decode, one sequence at a time"""

    def __init__(self, config: int):
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O

        import ocr_b200 as ocr

        self.config, self.O = config, O
        w = WORKLOADS[config]
        self.model = O.Model(CONFIG2, seed=ocr.SEED_BASE + 2, sigma_w=0.02, sigma_e=0.02)
        self.s = self.model.session(w["prefix"] + w["new"])
        self.s.n_past = w["prefix"]
        self.s.step(IMAGE_PAD)  # warm-up

    def run(self, n_tokens: int):
        """(seconds, sample text) for n_tokens steps"""
        pos = cpu_positions(self.config, n_tokens)
        t0 = time.perf_counter()
        for i, p in enumerate(pos):
            self.s.n_past = p  # the cache rows' values do not change the work of a step
            self.s.step((IMAGE_PAD + 7 * i) % CONFIG2["n_vocab"])
        dt = time.perf_counter() - t0
        sample = (f"{n_tokens} config-{self.config} decode steps at positions {pos[0]}..{pos[-1]} (spread evenly over "
                  f"the decode, mean {sum(pos) / len(pos) + 1:.0f} keys), one sequence at a time, oracle/oracle.c "
                  "(OpenMP)")
        return dt, sample

    def cores(self) -> int:
        return self.O.num_threads()


class CpuLmHead:
    """config 1 on the host cores: the oracle's LM head (151936 x 1024 q8_0 matvec of the output-normed row, OpenMP)
    and its choose() (windowed penalty rp 1.15 over 64 history ids, greedy), the seeded inputs of the GPU arm's shape"""

    def __init__(self):
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle as O

        self.O = O
        V, D = CONFIG2["n_vocab"], CONFIG2["dim"]
        self.V, self.D = V, D
        self.w = O.synth_q8_0(V * D, 4242, 0.02)
        x = O.gauss(17, D, 1.0)
        self.xn = (x * np.float32(O.rms_scale(x, 1e-6)) * O.fill_norm(18, D)).astype(np.float32)
        self.hist = [int(t) for t in O.fill_ids(19, 64, V)]

    def run(self, n: int):
        """(seconds, sample text) for n choices"""
        t0 = time.perf_counter()
        for _ in range(n):
            logits = self.O.matvec_q8_0(self.w, self.V, self.D, self.xn)
            self.O.choose_greedy(logits, 1.15, 64, 0.0, self.hist)
        dt = time.perf_counter() - t0
        return dt, (f"{n} choices: the LM head matvec ({self.V} x {self.D} q8_0) and choose() (rp 1.15, window 64, "
                    "greedy), oracle/oracle.c (OpenMP)")

    def cores(self) -> int:
        return self.O.num_threads()


def cpu_encode_sample(side: int = 280):
    """the vision encoder on the host cores: the oracle's encode (OpenMP) of a side x side page with the full
    24-layer LightOnOCR-shaped encoder — a bounded sample of config 4's encode (8800 patches), reported per patch"""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O

    import ocr_b200 as ocr

    cfg = ocr.VisionConfig().as_dict()
    v = O.Vision(cfg, ocr.SEED_BASE + 4, 0.02)
    img = np.random.default_rng(4).integers(0, 256, (side, side, 3), dtype=np.uint8)
    t0 = time.perf_counter()
    v.encode(img)
    dt = time.perf_counter() - t0
    n = (side // 14) ** 2
    return {"value": round(n / dt, 1), "unit": "patches/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"the oracle's encode of a {side} x {side} page ({n} patches, 24 layers, the projector), "
                      f"{dt:.1f} s, oracle/vision.c (OpenMP); config 4's page has 8800 patches"}


def cpu_baseline_sample(config: int, tokens_sample: int = 16):
    if config == 1:
        cl = CpuLmHead()
        cl.run(1)  # warm-up
        dt, sample = cl.run(tokens_sample)
        return {"value": round(tokens_sample / dt, 2), "unit": "choices/s", "cores": cl.cores(), "kind": "port",
                "sample": sample}
    cd = CpuDecode(config)
    dt, sample = cd.run(tokens_sample)
    return {"value": round(tokens_sample / dt, 2), "unit": "tok/s", "cores": cd.cores(), "kind": "port",
            "sample": sample}


def run_reference(args):
    rank, local, world = dist_env()
    if rank != 0:
        return
    if args.config == 1:
        # config 1: the oracle's LM head + choose() on the host cores, on our arm's metric and unit
        cl = CpuLmHead()
        cl.run(1)
        dt, n = 0.0, 4
        for i in range(args.warmup + args.steps):
            t, sample = cl.run(n)
            if i >= args.warmup:
                dt += t
        v = round(n * args.steps / dt, 3)
        print(json.dumps({
            "impl": "reference", "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
            "value": v, "unit": "choices/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q8_0 x f32", "data": "synthetic",
            "config": {"workload": "BASELINE config 1: LM head 151936 x 1024 q8_0 + windowed penalty + argmax"},
            "cpu_baseline": {"value": v, "unit": "choices/s", "cores": cl.cores(), "kind": "port",
                             "sample": sample + " — the reference's Rust/WGSL path cannot run here; timed is its CPU "
                                                "restatement"},
            "e2e": {"value": v, "unit": "choices/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)
        return
    config = args.config
    w = WORKLOADS[config]
    per_step = 4  # tokens per step: a bounded sample of the decode
    cd = CpuDecode(config)
    cores = cd.cores()
    dt = 0.0
    for i in range(args.warmup + args.steps):
        t, sample = cd.run(per_step)
        if i >= args.warmup:
            dt += t
    v = round(per_step * args.steps / dt, 3)
    sample = (sample.replace(f"{per_step} config", f"{per_step} (per step) config") +
              " — the reference's Rust/WGSL path cannot run here (no Rust toolchain, no graphics adapter); timed is "
              "its CPU restatement")
    print(json.dumps({
        "impl": "reference", "metric": "decode tok/s per B200 & per box (q8_0 1B VLM); matvec HBM GB/s vs peak",
        "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q8_0 weights x f32 activations, f16 KV", "data": "synthetic",
        "config": workload_config(config, w["B"], w["new"], w["prefix"], world),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4, 5], default=3)
    ap.add_argument("--pages", type=int, default=0, help="config 5: pages in the sweep (default 512)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true", help="config 3: skip the config-2 measurement beside it")
    ap.add_argument("--tokens", type=int, default=0,
                    help="decode this many tokens per step instead of the config's (short runs for ncu captures)")
    ap.add_argument("--prefix", type=int, default=0,
                    help="prefix rows per slot instead of the config's (small cases for ncu captures)")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the first timed step with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
