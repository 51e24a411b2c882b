"""libocrcuda.so on the host (no GPU): it loads, exports every entry point include/ocr_cuda.h declares, refuses bad
arguments with a message, and its GGUF reader follows the reference's rules (app/crates/ocr-gguf/src/lib.rs tests
parses_kvs_tensors_and_data / rejects_unknown_type_and_truncation, 577-606; TextConfig::from_gguf and
TextModel::load's checks, app/crates/ocr-wgpu/src/text.rs:51-82, 111-128, 332-375).
"""
from __future__ import annotations

import ctypes as C
import re
import struct
from pathlib import Path

import numpy as np
import pytest

import gguf_writer as W

HEADER = Path(__file__).resolve().parent.parent / "include" / "ocr_cuda.h"


def declared():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:ocr_status|const char\*|int)\s+(ocr_\w+)\s*\(", txt, re.M)))


def test_library_exports_every_declared_symbol(ocr):
    names = declared()
    assert len(names) >= 30
    lib = ocr.lib()
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(ocr.EXPORTS) == names
    assert "sm_100a" in ocr.version()
    assert ocr.q8_row_bytes(1024) == 1088 and ocr.q8_row_bytes(96) == 112 and ocr.q8_row_bytes(33) == 0


def test_host_argument_errors(ocr):
    lib = ocr.lib()
    assert lib.ocr_session_create(None, 10, 1, None) == 1
    assert "null" in lib.ocr_last_error().decode()
    assert lib.ocr_prefill(None, 0, None, None, 0, None) == 1
    assert lib.ocr_sample_logits(None, None, 0, None, None, 0, None, None, 0, None) == 1
    # sampled presets stay on the CPU (text.rs:151-163)
    with pytest.raises(ocr.OcrError, match="sampled"):
        ocr.Preset("sampled_T0.1_p0.9", temperature=0.1, top_p=0.9, repetition_penalty=1.0).sampler()


def tiny_generic(alignment=None):
    """lib.rs:522-575's tiny GGUF: 3 KVs (u32, string array, f32 array) + bf16 [3,2] + q8_0 [32]"""
    q = np.frombuffer(np.float16(0.5).tobytes(), np.uint8).tobytes() + (np.arange(32) - 16).astype(np.int8).tobytes()
    return W.write(
        [("a.n", W.U32, 7), ("a.names", W.ARR, (W.STR, ["x", "yz"])), ("a.mean", W.ARR, (W.F32, [0.5, 0.25, -1.0]))],
        [("w", [3, 2], W.T_BF16, W.bf16_bytes([1.0, -2.0, 0.5, 3.0, 0.0, 1.5])), ("q", [32], W.T_Q8_0, q)],
        alignment)


@pytest.mark.parametrize("al", [None, 64])
def test_parses_kvs_tensors_and_data(ocr, al):
    g = ocr.Gguf(data=tiny_generic(al))
    h = g.header()
    assert h["version"] == 3 and h["n_tensors"] == 2
    assert g.u32("a.n") == 7
    assert g.f32_array("a.mean") == [0.5, 0.25, -1.0]
    w = g.info("w")
    assert (w["shape"], w["type"]) == ([3, 2], 30)
    assert g.to_f32("w").tolist() == [1.0, -2.0, 0.5, 3.0, 0.0, 1.5]
    q = g.to_f32("q")
    assert len(q) == 32 and (q[0], q[31]) == (-8.0, 7.5)
    assert h["data_offset"] % (al or 32) == 0


def test_rejects_unknown_type_and_truncation(ocr):
    b = bytearray(tiny_generic())
    pos = bytes(b).index(bytes([1, 0, 0, 0, 32, 0, 0, 0, 0, 0, 0, 0])) + 12  # the q tensor's type: Q8_0 → Q4_K
    b[pos] = 12
    with pytest.raises(ocr.OcrError, match="not supported"):
        ocr.Gguf(data=bytes(b))
    t = tiny_generic()
    with pytest.raises(ocr.OcrError):
        ocr.Gguf(data=t[:-1])
    with pytest.raises(ocr.OcrError, match="magic"):
        ocr.Gguf(data=b"GGUX")
    v4 = bytearray(tiny_generic())
    v4[4] = 4
    with pytest.raises(ocr.OcrError, match="version"):
        ocr.Gguf(data=bytes(v4))


TINY = dict(n_layer=2, dim=256, n_head=2, n_kv=1, d_head=128, n_ff=512, n_vocab=1000)


@pytest.fixture(scope="module")
def tiny_model_bytes(orc):
    return W.text_model(orc.Model(TINY, seed=11))


def test_text_config_from_gguf(ocr, tiny_model_bytes):
    c = ocr.Gguf(data=tiny_model_bytes).text_config()
    assert (c.n_layer, c.dim, c.n_head, c.n_kv, c.d_head, c.n_ff, c.n_vocab) == (2, 256, 2, 1, 128, 512, 1000)
    assert abs(c.eps - 1e-6) < 1e-12 and c.rope_base == 1e6 and c.n_ctx_train == 40960


def _edit(orc, mutate_kvs=None, mutate_tensors=None):
    m = orc.Model(TINY, seed=11)
    kvs = W.text_model_kvs(m.cfg)
    ts = W.text_model_tensors(m)
    if mutate_kvs:
        kvs = mutate_kvs(kvs)
    if mutate_tensors:
        ts = mutate_tensors(ts)
    return W.write(kvs, ts)


@pytest.mark.parametrize("case,match", [
    ("arch", "qwen3 only"),
    ("head_dim", "written for 128"),
    ("heads", "kv heads"),
    ("rope_scaling", "rope scaling"),
    ("bias", "not part of this engine's graph"),
    ("fused_qkv", "fused attn_qkv"),
    ("output_weight", "ties the output"),
    ("f16_weight", "read q8_0 weights"),
    ("bad_shape", "shape"),
    ("norm_type", "expected F32"),
    ("missing", "no tensor"),
])
def test_text_model_checks(ocr, orc, case, match):
    def kv_set(key, ty, val):
        return lambda kvs: [(k, t, v) if k != key else (k, ty, val) for k, t, v in kvs]

    def add_tensor(name, shape, ty, data):
        return lambda ts: ts + [(name, shape, ty, data)]

    q_blk = b"\0" * 34
    edits = {
        "arch": dict(mutate_kvs=kv_set("general.architecture", W.STR, "llama")),
        "head_dim": dict(mutate_kvs=kv_set("qwen3.attention.key_length", W.U32, 64)),
        "heads": dict(mutate_kvs=kv_set("qwen3.attention.head_count_kv", W.U32, 3)),
        "rope_scaling": dict(mutate_kvs=lambda kvs: kvs + [("qwen3.rope.scaling.type", W.STR, "yarn")]),
        "bias": dict(mutate_tensors=add_tensor("blk.0.attn_q.bias", [256], W.T_F32, b"\0" * 1024)),
        "fused_qkv": dict(mutate_tensors=add_tensor("blk.1.attn_qkv.weight", [32], W.T_Q8_0, q_blk)),
        "output_weight": dict(mutate_tensors=add_tensor("output.weight", [32], W.T_Q8_0, q_blk)),
        "f16_weight": dict(mutate_tensors=lambda ts: [(n, s, W.T_F16 if n == "blk.0.attn_k.weight" else t,
                                                       b"\0" * (s[0] * s[1] * 2) if n == "blk.0.attn_k.weight" else d)
                                                      for n, s, t, d in ts]),
        "bad_shape": dict(mutate_tensors=lambda ts: [(n, [s[1], s[0]] if n == "blk.1.ffn_down.weight" else s, t, d)
                                                     for n, s, t, d in ts]),
        "norm_type": dict(mutate_tensors=lambda ts: [(n, s, W.T_F16 if n == "blk.0.ffn_norm.weight" else t,
                                                      d[: len(d) // 2] if n == "blk.0.ffn_norm.weight" else d)
                                                     for n, s, t, d in ts]),
        "missing": dict(mutate_tensors=lambda ts: [x for x in ts if x[0] != "blk.1.attn_v.weight"]),
    }
    data = _edit(orc, **edits[case])
    with pytest.raises(ocr.OcrError, match=match):
        ocr.Gguf(data=data).text_config()


def test_gguf_file_roundtrip(ocr, tiny_model_bytes, tmp_path):
    p = tmp_path / "text-q8_0.gguf"
    p.write_bytes(tiny_model_bytes)
    g = ocr.Gguf(path=str(p))
    assert g.str("general.architecture") == "qwen3"
    info = g.info("token_embd.weight")
    assert info["shape"] == [256, 1000] and info["type"] == 8
    with pytest.raises(ocr.OcrError, match="cannot open"):
        ocr.Gguf(path=str(tmp_path / "absent.gguf"))
