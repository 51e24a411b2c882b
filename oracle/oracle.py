"""oracle.py — ctypes wrapper of the CPU oracle (oracle.c). TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg may import this module, and
only as the checker or the timed CPU baseline — never as part of the product path. See oracle.h for the reference
file:line each function restates.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

ATTN_NORM, Q, K, V, O, Q_NORM, K_NORM, FFN_NORM, GATE, UP, DOWN = range(11)
TOK_EMBD_STREAM, OUTPUT_NORM_STREAM = 100000, 100001


class VCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "dim", "n_head", "n_ff", "patch", "merge", "image_size",
                                         "proj_dim")] + [("eps", C.c_float), ("rope_theta", C.c_float),
                                                         ("mean", C.c_float * 3), ("std", C.c_float * 3)]


class Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "dim", "n_head", "n_kv", "d_head", "n_ff", "n_vocab")] + [
        ("eps", C.c_float), ("rope_base", C.c_float)]


_P = C.c_void_p
_SIGS = {
    "orc_splitmix64_at": (C.c_uint64, [C.c_uint64, C.c_uint64]),
    "orc_substream": (C.c_uint64, [C.c_uint64, C.c_uint64]),
    "orc_gauss": (C.c_float, [C.c_uint64, C.c_uint64]),
    "orc_fill_gauss": (None, [_P, C.c_size_t, C.c_uint64, C.c_float]),
    "orc_fill_norm": (None, [_P, C.c_size_t, C.c_uint64]),
    "orc_fill_ids": (None, [_P, C.c_size_t, C.c_uint64, C.c_uint32]),
    "orc_f16_from_f32": (C.c_uint16, [C.c_float]),
    "orc_f32_from_f16": (C.c_float, [C.c_uint16]),
    "orc_quantize_q8_0": (None, [_P, C.c_size_t, _P, _P]),
    "orc_dequantize_q8_0": (None, [_P, C.c_size_t, _P]),
    "orc_synth_q8_0": (None, [_P, C.c_size_t, C.c_uint64, C.c_float]),
    "orc_rope_table": (None, [C.c_float, C.c_int, C.c_int, _P]),
    "orc_rms_scale": (C.c_float, [_P, C.c_int, C.c_float]),
    "orc_matvec_q8_0": (None, [_P, C.c_int, C.c_int, _P, _P, C.c_int]),
    "orc_head_norm_rope": (None, [_P, _P, _P, C.c_int, C.c_float, _P]),
    "orc_attend": (None, [_P, _P, _P, C.c_int, C.c_int, C.c_int, C.c_float, _P]),
    "orc_choose_greedy": (C.c_int32, [_P, C.c_int, C.c_float, C.c_int, C.c_float, _P, C.c_int, _P, _P, C.c_int]),
    "orc_apply_window_penalty": (None, [_P, C.c_float, C.c_int, _P, C.c_int]),
    "orc_model_synthetic": (_P, [C.POINTER(Cfg), C.c_uint64, C.c_float, C.c_float]),
    "orc_model_alloc": (_P, [C.POINTER(Cfg)]),
    "orc_model_free": (None, [_P]),
    "orc_model_tensor": (_P, [_P, C.c_int, C.c_int, C.POINTER(C.c_size_t)]),
    "orc_session_new": (_P, [_P, C.c_int]),
    "orc_session_free": (None, [_P]),
    "orc_session_n_past": (C.c_int, [_P]),
    "orc_session_set_n_past": (None, [_P, C.c_int]),
    "orc_prefill": (C.c_int, [_P, _P, _P, C.c_int, _P]),
    "orc_step": (C.c_int, [_P, C.c_int32, _P]),
    "orc_decode": (C.c_int, [_P, _P, C.c_float, C.c_int, C.c_float, _P, C.c_int, C.c_int, _P, _P]),
    "orc_decode_top2": (C.c_int, [_P, _P, C.c_float, C.c_int, C.c_float, _P, C.c_int, C.c_int, _P, _P, _P]),
    "orc_session_k": (_P, [_P, C.c_int]),
    "orc_session_v": (_P, [_P, C.c_int]),
    "orc_session_set_kv": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, _P, _P]),
    "orc_num_threads": (C.c_int, []),
    "orc_vision_patch_cols": (C.c_int, [_P]),
    "orc_synth_q8_0_padded": (None, [_P, C.c_int, C.c_int, C.c_int, C.c_uint64, C.c_float]),
    "orc_vision_synthetic": (_P, [_P, C.c_uint64, C.c_float]),
    "orc_vision_free": (None, [_P]),
    "orc_pixel_lut": (None, [_P, _P]),
    "orc_rope2d_table": (None, [C.c_float, C.c_int, C.c_int, _P]),
    "orc_gelu_tanh": (C.c_float, [C.c_float]),
    "orc_vision_encode": (C.c_int, [_P, _P, C.c_int, C.c_int, C.c_int, _P]),
    "orc_vision_layer1_rows": (C.c_int, [_P, _P, C.c_int, C.c_int, _P, C.c_int, _P]),
    "orc_bake_plan": (None, [C.c_int, C.c_int, C.c_int, C.c_int, _P]),
    "orc_bake_pad": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
    "orc_resize_taps": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), _P, C.c_int]),
    "orc_resize_lanczos3": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
    "orc_bake": (C.c_int, [_P, C.c_int, C.c_int, C.c_int, C.c_int, _P]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            import importlib.util
            spec = importlib.util.spec_from_file_location("oracle_build", HERE / "build.py")
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build()
        L = C.CDLL(str(LIB))
        for n, (r, a) in _SIGS.items():
            f = getattr(L, n)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


# ---- data ------------------------------------------------------------------------------------------------------------
def gauss(seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_gauss(_p(out), n, seed, sigma)
    return out


def fill_norm(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_fill_norm(_p(out), n, seed)
    return out


def fill_ids(seed: int, n: int, n_vocab: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().orc_fill_ids(_p(out), n, seed, n_vocab)
    return out


def substream(seed: int, k: int) -> int:
    return int(lib().orc_substream(seed, k))


def f16_from_f32(x: np.ndarray) -> np.ndarray:
    f = lib().orc_f16_from_f32
    return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)


def quantize_q8_0(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(GGUF blocks as uint8 [n/32*34], dequantized f32 [n])"""
    x = np.ascontiguousarray(x, np.float32).ravel()
    blocks = np.empty(x.size // 32 * 34, np.uint8)
    deq = np.empty(x.size, np.float32)
    lib().orc_quantize_q8_0(_p(x), x.size, _p(blocks), _p(deq))
    return blocks, deq


def dequantize_q8_0(blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q8_0(_p(np.ascontiguousarray(blocks, np.uint8)), n, _p(out))
    return out


def synth_q8_0(n: int, seed: int, sigma: float) -> np.ndarray:
    blocks = np.empty(n // 32 * 34, np.uint8)
    lib().orc_synth_q8_0(_p(blocks), n, seed, sigma)
    return blocks


def rope_table(base: float, d_head: int, n_pos: int) -> np.ndarray:
    out = np.empty((n_pos, d_head // 2, 2), np.float32)
    lib().orc_rope_table(base, d_head, n_pos, _p(out))
    return out


def matvec_q8_0(blocks: np.ndarray, rows: int, k: int, x: np.ndarray, y: Optional[np.ndarray] = None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    acc = y is not None
    out = np.ascontiguousarray(y, np.float32).copy() if acc else np.empty(rows, np.float32)
    lib().orc_matvec_q8_0(_p(np.ascontiguousarray(blocks, np.uint8)), rows, k, _p(x), _p(out), 1 if acc else 0)
    return out


def rms_scale(x: np.ndarray, eps: float) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return float(lib().orc_rms_scale(_p(x), x.size, eps))


def head_norm_rope(head: np.ndarray, w: np.ndarray, cs: np.ndarray, eps: float) -> np.ndarray:
    head = np.ascontiguousarray(head, np.float32)
    out = np.empty_like(head)
    lib().orc_head_norm_rope(_p(head), _p(np.ascontiguousarray(w, np.float32)),
                             _p(np.ascontiguousarray(cs, np.float32)), head.size, eps, _p(out))
    return out


def attend(q: np.ndarray, k16: np.ndarray, v16: np.ndarray, n_keys: int, stride: int, scale: float) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    out = np.empty_like(q)
    lib().orc_attend(_p(q), _p(np.ascontiguousarray(k16, np.uint16)), _p(np.ascontiguousarray(v16, np.uint16)),
                     n_keys, stride, q.size, scale, _p(out))
    return out


def choose_greedy(logits: np.ndarray, rp: float, window: int, fp: float, history: Sequence[int],
                  counts: Optional[dict] = None) -> tuple[int, np.ndarray]:
    """ocr_decode::sampling::choose (greedy); returns (token, the penalised logits)"""
    l = np.ascontiguousarray(logits, np.float32).copy()
    h = np.ascontiguousarray(history, np.int32)
    ct = np.ascontiguousarray(list((counts or {}).keys()), np.int32)
    cn = np.ascontiguousarray(list((counts or {}).values()), np.uint32)
    t = lib().orc_choose_greedy(_p(l), l.size, rp, window, fp, _p(h) if h.size else None, h.size,
                                _p(ct) if ct.size else None, _p(cn) if cn.size else None, ct.size)
    return int(t), l


def apply_window_penalty(logits: np.ndarray, rp: float, window: int, history: Sequence[int]) -> np.ndarray:
    l = np.ascontiguousarray(logits, np.float32).copy()
    h = np.ascontiguousarray(history, np.int32)
    lib().orc_apply_window_penalty(_p(l), rp, window, _p(h) if h.size else None, h.size)
    return l


# ---- the decoder -----------------------------------------------------------------------------------------------------
class Model:
    def __init__(self, cfg: dict, seed: Optional[int] = None, sigma_w: float = 0.02, sigma_e: float = 0.02):
        self.cfg = dict(cfg)
        c = Cfg(cfg["n_layer"], cfg["dim"], cfg["n_head"], cfg["n_kv"], cfg["d_head"], cfg["n_ff"], cfg["n_vocab"],
                cfg.get("eps", 1e-6), cfg.get("rope_base", 1e6))
        self._c = c
        self.h = lib().orc_model_synthetic(C.byref(c), seed, sigma_w, sigma_e) if seed is not None else \
            lib().orc_model_alloc(C.byref(c))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def tensor(self, layer: int, kind: int) -> np.ndarray:
        """raw storage view (uint8) of a tensor: q8_0 blocks, or f32 bytes for norms"""
        n = C.c_size_t()
        p = lib().orc_model_tensor(self.h, layer, kind, C.byref(n))
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n.value,))

    def session(self, n_ctx: int) -> "Session":
        return Session(self, n_ctx)


class Session:
    def __init__(self, model: Model, n_ctx: int):
        self.model = model
        self.n_ctx = n_ctx
        self.h = lib().orc_session_new(model.h, n_ctx)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_session_free(self.h)
            self.h = None

    @property
    def n_past(self) -> int:
        return lib().orc_session_n_past(self.h)

    @n_past.setter
    def n_past(self, v: int) -> None:
        lib().orc_session_set_n_past(self.h, v)

    def prefill(self, ids: Optional[Sequence[int]], embd: Optional[np.ndarray], n: int) -> np.ndarray:
        V = self.model.cfg["n_vocab"]
        out = np.empty(V, np.float32)
        ida = None if ids is None else np.ascontiguousarray(ids, np.int32)
        ea = None if embd is None else np.ascontiguousarray(embd, np.float32)
        rc = lib().orc_prefill(self.h, _p(ida), _p(ea), n, _p(out))
        if rc != 0:
            raise RuntimeError(f"orc_prefill: {rc}")
        return out

    def step(self, tok: int) -> np.ndarray:
        out = np.empty(self.model.cfg["n_vocab"], np.float32)
        rc = lib().orc_step(self.h, tok, _p(out))
        if rc != 0:
            raise RuntimeError(f"orc_step: {rc}")
        return out

    def decode(self, first_logits: np.ndarray, rp: float, window: int, fp: float, history: Sequence[int],
               max_new: int) -> tuple[np.ndarray, np.ndarray]:
        ids = np.empty(max_new, np.int32)
        margins = np.empty(max_new, np.float32)
        h = np.ascontiguousarray(history, np.int32)
        rc = lib().orc_decode(self.h, _p(np.ascontiguousarray(first_logits, np.float32)), rp, window, fp,
                              _p(h) if h.size else None, h.size, max_new, _p(ids), _p(margins))
        if rc != 0:
            raise RuntimeError(f"orc_decode: {rc}")
        return ids, margins

    def decode_top2(self, first_logits: np.ndarray, rp: float, window: int, fp: float, history: Sequence[int],
                    max_new: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """decode, with each choice's top-2 margin and runner-up token"""
        ids = np.empty(max_new, np.int32)
        margins = np.empty(max_new, np.float32)
        second = np.empty(max_new, np.int32)
        h = np.ascontiguousarray(history, np.int32)
        rc = lib().orc_decode_top2(self.h, _p(np.ascontiguousarray(first_logits, np.float32)), rp, window, fp,
                                   _p(h) if h.size else None, h.size, max_new, _p(ids), _p(margins), _p(second))
        if rc != 0:
            raise RuntimeError(f"orc_decode_top2: {rc}")
        return ids, margins, second

    def kv(self, layer: int) -> tuple[np.ndarray, np.ndarray]:
        c = self.model.cfg
        n = self.n_ctx * c["n_kv"] * c["d_head"]
        k = np.ctypeslib.as_array(C.cast(lib().orc_session_k(self.h, layer), C.POINTER(C.c_uint16)), shape=(n,))
        v = np.ctypeslib.as_array(C.cast(lib().orc_session_v(self.h, layer), C.POINTER(C.c_uint16)), shape=(n,))
        return k.copy(), v.copy()

    def set_kv(self, layer: int, row0: int, k: np.ndarray, v: np.ndarray) -> None:
        """overwrite KV rows [row0, row0 + len(k)) of a layer (f16 bit patterns, [n][n_kv * d_head])"""
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        if lib().orc_session_set_kv(self.h, layer, row0, k.shape[0], _p(k), _p(v)) != 0:
            raise RuntimeError("orc_session_set_kv: rows outside the session")


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---- the vision encoder + projector (vision.c) --------------------------------------------------------------------------
V_LN1, V_Q, V_K, V_V, V_O, V_LN2, V_GATE, V_UP, V_DOWN = range(9)
V_LAYER_STREAM, V_PATCH_STREAM, V_PRE_LN_STREAM, V_INPUT_NORM_STREAM = 200000, 300000, 300001, 300002
V_MERGER_STREAM, V_MM1_STREAM, V_MM2_STREAM = 300003, 300004, 300005


def vcfg(d: dict) -> VCfg:
    return VCfg(d["n_layer"], d["dim"], d["n_head"], d["n_ff"], d["patch"], d["merge"], d["image_size"],
                d["proj_dim"], d["eps"], d["rope_theta"], (C.c_float * 3)(*d["mean"]), (C.c_float * 3)(*d["std"]))


class Vision:
    """the synthetic q8_0 encoder + projector of a config dict (the keys of VCfg)"""

    def __init__(self, cfg: dict, seed: int, sigma_w: float = 0.02):
        self.cfg = dict(cfg)
        self._c = vcfg(cfg)
        self.h = lib().orc_vision_synthetic(C.byref(self._c), seed, sigma_w)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_vision_free(self.h)
            self.h = None

    def grid(self, w: int, h: int) -> tuple[int, int]:
        return w // self.cfg["patch"], h // self.cfg["patch"]

    def encode(self, rgb: np.ndarray, layers: int = -1) -> np.ndarray:
        """rgb uint8 [h][w][3] (baked) → [n_tokens][proj_dim], or the residual [n_patches][dim] after `layers`"""
        h, w = rgb.shape[:2]
        px, py = self.grid(w, h)
        n = px * py
        m = self.cfg["merge"] ** 2
        out = np.empty((n, self.cfg["dim"]) if layers >= 0 else (n // m, self.cfg["proj_dim"]), np.float32)
        rc = lib().orc_vision_encode(self.h, _p(np.ascontiguousarray(rgb, np.uint8)), w, h, layers, _p(out))
        if rc < 0:
            raise ValueError(f"image {w}x{h} is not baked")
        return out

    def layer1_rows(self, rgb: np.ndarray, rows: Sequence[int]) -> np.ndarray:
        h, w = rgb.shape[:2]
        r = np.ascontiguousarray(rows, np.int32)
        out = np.empty((r.size, self.cfg["dim"]), np.float32)
        if lib().orc_vision_layer1_rows(self.h, _p(np.ascontiguousarray(rgb, np.uint8)), w, h, _p(r), r.size,
                                        _p(out)) < 0:
            raise ValueError("bad image or rows")
        return out


def rope2d_table(theta: float, d_head: int, max_pos: int) -> np.ndarray:
    out = np.empty((2, max_pos, d_head // 4, 2), np.float32)
    lib().orc_rope2d_table(theta, d_head, max_pos, _p(out))
    return out


def pixel_lut(cfg: dict) -> np.ndarray:
    out = np.empty((3, 256), np.float32)
    c = vcfg(cfg)
    lib().orc_pixel_lut(C.byref(c), _p(out))
    return out


def bake_plan(longest: int, grid: int, w0: int, h0: int) -> tuple[int, ...]:
    out = np.empty(6, np.int32)
    lib().orc_bake_plan(longest, grid, w0, h0, _p(out))
    return tuple(int(v) for v in out)


def bake_pad(rgb: np.ndarray, longest: int = 1540, grid: int = 28) -> np.ndarray:
    h0, w0 = rgb.shape[:2]
    sw, sh, left, top, right, bottom = bake_plan(longest, grid, w0, h0)
    out = np.empty((sh + top + bottom, sw + left + right, 3), np.uint8)
    if lib().orc_bake_pad(_p(np.ascontiguousarray(rgb, np.uint8)), w0, h0, longest, grid, _p(out)) != 0:
        raise ValueError("the bake of this image resizes it")
    return out


def resize_lanczos3(rgb: np.ndarray, w: int, h: int) -> np.ndarray:
    h0, w0 = rgb.shape[:2]
    out = np.empty((h, w, 3), np.uint8)
    if lib().orc_resize_lanczos3(_p(np.ascontiguousarray(rgb, np.uint8)), w0, h0, w, h, _p(out)) != 0:
        raise ValueError("resize out of range")
    return out


def resize_taps(n_in: int, n_out: int, o: int) -> tuple[int, np.ndarray]:
    w = np.empty(4096, np.float32)
    left = C.c_int()
    n = lib().orc_resize_taps(n_in, n_out, o, C.byref(left), _p(w), 4096)
    return left.value, w[:n].copy()


def bake(rgb: np.ndarray, longest: int = 1540, grid: int = 28) -> np.ndarray:
    """the whole bake: the Lanczos-3 resize when the plan scales, then the white pads"""
    h0, w0 = rgb.shape[:2]
    sw, sh, left, top, right, bottom = bake_plan(longest, grid, w0, h0)
    out = np.empty((sh + top + bottom, sw + left + right, 3), np.uint8)
    if lib().orc_bake(_p(np.ascontiguousarray(rgb, np.uint8)), w0, h0, longest, grid, _p(out)) != 0:
        raise ValueError("bake failed")
    return out
