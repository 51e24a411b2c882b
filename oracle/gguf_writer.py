"""gguf_writer.py — write GGUF v3 files (TEST INFRASTRUCTURE): a qwen3 text model from the oracle's tensors, or raw
key/value + tensor lists for the reader's format tests. The byte layout is GGUF's (ggml gguf.cpp; the reader rules of
b-straub/historic-htr-ocr app/crates/ocr-gguf/src/lib.rs:341-401): header, KVs, tensor infos, data aligned.
"""
from __future__ import annotations

import struct
from typing import Iterable, Optional

import numpy as np

# GGUF value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
# ggml tensor types
T_F32, T_F16, T_Q8_0, T_BF16 = 0, 1, 8, 30


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _val(ty: int, v) -> bytes:
    if ty == STR:
        return _s(v)
    if ty == ARR:
        ety, items = v
        return struct.pack("<IQ", ety, len(items)) + b"".join(_val(ety, x) for x in items)
    fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}[ty]
    return struct.pack(fmt, v)


def write(kvs: Iterable[tuple[str, int, object]], tensors: Iterable[tuple[str, list[int], int, bytes]],
          alignment: Optional[int] = None, version: int = 3) -> bytes:
    """kvs: (key, value type, value); tensors: (name, shape in ggml order, ggml type, raw bytes)"""
    kvs = list(kvs)
    tensors = list(tensors)
    if alignment is not None:
        kvs.append(("general.alignment", U32, alignment))
    al = alignment or 32
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs)))
    for k, ty, v in kvs:
        out += _s(k) + struct.pack("<I", ty) + _val(ty, v)
    off = 0
    offsets = []
    for name, shape, ty, data in tensors:
        offsets.append(off)
        out += _s(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        out += struct.pack("<IQ", ty, off)
        off = (off + len(data) + al - 1) // al * al
    while len(out) % al:
        out.append(0)
    base = len(out)
    for (name, shape, ty, data), o in zip(tensors, offsets):
        while len(out) < base + o:
            out.append(0)
        out += data
    return bytes(out)


KIND_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm", "ffn_norm",
              "ffn_gate", "ffn_up", "ffn_down")


def text_model_kvs(cfg: dict, n_ctx_train: int = 40960) -> list:
    return [
        ("general.architecture", STR, "qwen3"),
        ("qwen3.block_count", U32, cfg["n_layer"]),
        ("qwen3.context_length", U32, n_ctx_train),
        ("qwen3.embedding_length", U32, cfg["dim"]),
        ("qwen3.feed_forward_length", U32, cfg["n_ff"]),
        ("qwen3.attention.head_count", U32, cfg["n_head"]),
        ("qwen3.attention.head_count_kv", U32, cfg["n_kv"]),
        ("qwen3.attention.key_length", U32, cfg["d_head"]),
        ("qwen3.attention.value_length", U32, cfg["d_head"]),
        ("qwen3.attention.layer_norm_rms_epsilon", F32, cfg.get("eps", 1e-6)),
        ("qwen3.rope.freq_base", F32, cfg.get("rope_base", 1e6)),
    ]


def text_model_tensors(model) -> list:
    """(name, shape, type, bytes) of an oracle.Model, in GGUF's order: token_embd, layers, output_norm"""
    c = model.cfg
    qd, kvd = c["n_head"] * c["d_head"], c["n_kv"] * c["d_head"]
    shapes = {
        "attn_norm": [c["dim"]], "attn_q": [c["dim"], qd], "attn_k": [c["dim"], kvd], "attn_v": [c["dim"], kvd],
        "attn_output": [qd, c["dim"]], "attn_q_norm": [c["d_head"]], "attn_k_norm": [c["d_head"]],
        "ffn_norm": [c["dim"]], "ffn_gate": [c["dim"], c["n_ff"]], "ffn_up": [c["dim"], c["n_ff"]],
        "ffn_down": [c["n_ff"], c["dim"]],
    }
    out = [("token_embd.weight", [c["dim"], c["n_vocab"]], T_Q8_0, model.tensor(-1, 0).tobytes())]
    for layer in range(c["n_layer"]):
        for kind, name in enumerate(KIND_NAMES):
            ty = T_F32 if len(shapes[name]) == 1 else T_Q8_0
            out.append((f"blk.{layer}.{name}.weight", shapes[name], ty, model.tensor(layer, kind).tobytes()))
    out.append(("output_norm.weight", [c["dim"]], T_F32, model.tensor(-1, 1).tobytes()))
    return out


def text_model(model, n_ctx_train: int = 40960, alignment: Optional[int] = None) -> bytes:
    return write(text_model_kvs(model.cfg, n_ctx_train), text_model_tensors(model), alignment)


def bf16_bytes(vals) -> bytes:
    a = np.asarray(vals, np.float32).view(np.uint32)
    r = ((a + 0x7FFF + ((a >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
    return r.tobytes()
