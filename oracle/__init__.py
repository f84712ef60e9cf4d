"""ctypes bindings of the CPU oracle (oracle/oracle.c) — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker (and the timed CPU baseline). The product package
(malaga_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")

# Compiler recipe: no FMA contraction (fmaf() is explicit), OpenMP over rows.
CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
          "-Wall", "-Wno-unused-parameter", "-Wno-maybe-uninitialized"]


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["gcc", *CFLAGS, "-o", LIB_PATH, src, "-lm"])
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i, u32, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_float
        L.orc_load.argtypes = [ctypes.c_char_p]
        L.orc_load.restype = vp
        L.orc_free.argtypes = [vp]
        L.orc_config.argtypes = [vp, vp]
        L.orc_dequant.argtypes = [vp, ctypes.c_char_p, ctypes.c_long, ctypes.c_long]
        L.orc_dequant.restype = f
        L.orc_encode.argtypes = [vp, vp, vp, i, i]
        L.orc_encode.restype = vp
        L.orc_enc_free.argtypes = [vp]
        L.orc_enc_synthetic.argtypes = [vp, vp, i, i, ctypes.c_uint64]
        L.orc_enc_synthetic.restype = vp
        L.orc_enc_cross.argtypes = [vp, vp, i, i, vp]
        L.orc_greedy.argtypes = [vp, vp, u32, i, i, vp, vp]
        L.orc_beam.argtypes = [vp, vp, u32, i, f, i, vp, vp]
        L.orc_greedy_sl.argtypes = [vp, vp, vp, vp, i, u32, i, i, vp, i, i, vp]
        L.orc_exp.argtypes = [f]
        L.orc_exp.restype = f
        L.orc_log.argtypes = [f]
        L.orc_log.restype = f
        L.orc_threads.restype = i
        L.orc_set_threads.argtypes = [i]
        L.orc_matmul.argtypes = [i, vp, ctypes.c_long, ctypes.c_long, vp, i, i, i, vp]
        L.orc_matmul.restype = i
        L.orc_quantize_q81.argtypes = [vp, i, i, vp, vp, vp]
        L.orc_log_softmax_topk.argtypes = [vp, i, i, i, vp, vp]
        _lib = L
    return _lib


CFG_KEYS = ["vocab_size", "d_model", "encoder_layers", "decoder_layers", "encoder_heads", "decoder_heads",
            "encoder_ffn", "decoder_ffn", "max_pos", "pad", "eos", "start", "max_length", "scale_embedding"]


def pad_batch(src: list[list[int]], pad: int) -> tuple[np.ndarray, np.ndarray]:
    s = max(len(r) for r in src)
    ids = np.full((len(src), s), pad, np.uint32)
    for i, r in enumerate(src):
        ids[i, : len(r)] = r
    return ids, np.array([len(r) for r in src], np.uint32)


class Oracle:
    def __init__(self, path: str):
        self.h = lib().orc_load(path.encode())
        if not self.h:
            raise OSError(f"oracle cannot load {path}")
        out = (ctypes.c_int * 16)()
        n = lib().orc_config(self.h, out)
        self.cfg = dict(zip(CFG_KEYS, list(out)[:n]))

    def close(self):
        if self.h:
            lib().orc_free(self.h)
            self.h = None

    __del__ = close

    def encode(self, src: list[list[int]]):
        ids, lens = pad_batch(src, self.cfg["pad"])
        e = lib().orc_encode(self.h, ids.ctypes.data, lens.ctypes.data, ids.shape[0], ids.shape[1])
        return _Enc(e, ids.shape[0], ids.shape[1])

    def cross(self, enc, layer: int, which: int) -> np.ndarray:
        H, d = self.cfg["decoder_heads"], self.cfg["d_model"]
        out = np.empty((enc.b, H, enc.s, d // H), np.float32)
        lib().orc_enc_cross(self.h, enc.h, layer, which, out.ctypes.data)
        return out

    def greedy(self, src: list[list[int]], tgt: int, max_new: int, force: bool = False, logits: bool = False):
        """Raw greedy columns [b, max_new] (pad after eos) and optional logits [max_new, b, V]."""
        enc = self.encode(src)
        out = np.zeros((enc.b, max_new), np.uint32)
        lg = np.empty((max_new, enc.b, self.cfg["vocab_size"]), np.float32) if logits else None
        lib().orc_greedy(self.h, enc.h, tgt, max_new, int(force), out.ctypes.data,
                         lg.ctypes.data if logits else None)
        return (out, lg) if logits else out

    def greedy_shortlist(self, src: list[list[int]], tgt: int, max_new: int, sl_ids: list[int], s_bucket: int,
                         force: bool = False):
        """Raw greedy columns [b, max_new] over a vocabulary shortlist (sorted ids)
        and the source tokens, the state's source bucket being s_bucket."""
        enc = self.encode(src)
        ids, lens = pad_batch(src, self.cfg["pad"])
        sl = np.ascontiguousarray(sl_ids, np.uint32)
        out = np.zeros((enc.b, max_new), np.uint32)
        lib().orc_greedy_sl(self.h, enc.h, ids.ctypes.data, lens.ctypes.data, ids.shape[1], tgt, max_new, int(force),
                            sl.ctypes.data, len(sl), s_bucket, out.ctypes.data)
        return out

    def beam(self, src: list[list[int]], tgt: int, k: int, max_new: int, length_penalty: float = 1.0):
        enc = self.encode(src)
        out = np.zeros((enc.b, max_new), np.uint32)
        lens = np.zeros(enc.b, np.uint32)
        lib().orc_beam(self.h, enc.h, tgt, k, length_penalty, max_new, out.ctypes.data, lens.ctypes.data)
        return [list(out[i, : lens[i]]) for i in range(enc.b)]

    def decode_timing_sample(self, src: list[list[int]], tgt: int, steps: int) -> np.ndarray:
        """Forced greedy decode of `steps` tokens from synthetic cross K/V (no
        encoder pass): the CPU-baseline timing sample."""
        lens = np.array([len(r) for r in src], np.uint32)
        e = lib().orc_enc_synthetic(self.h, lens.ctypes.data, len(src), int(lens.max()), 1)
        enc = _Enc(e, len(src), int(lens.max()))
        out = np.zeros((enc.b, steps), np.uint32)
        lib().orc_greedy(self.h, enc.h, tgt, steps, 1, out.ctypes.data, None)
        return out

    def dequant(self, name: str, r: int, j: int) -> float:
        return lib().orc_dequant(self.h, name.encode(), r, j)


class _Enc:
    def __init__(self, h, b, s):
        self.h, self.b, self.s = h, b, s

    def __del__(self):
        if self.h:
            lib().orc_enc_free(self.h)
            self.h = None


def matmul(ggml_type: int, w: np.ndarray, n_rows: int, k: int, x: np.ndarray, mode: str, nw: int = 4) -> np.ndarray:
    """y = x . W^T for raw GGUF rows w ([n_rows, row_bytes] uint8): mode "mmvq"
    (the reference's vector kernel with nw warps) or "mmq"."""
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros((x.shape[0], n_rows), np.float32)
    if lib().orc_matmul(ggml_type, w.ctypes.data, n_rows, k, x.ctypes.data, x.shape[0],
                        0 if mode == "mmvq" else 1, nw, y.ctypes.data) != 0:
        raise ValueError("unsupported matmul shape")
    return y


def quantize_q81(x: np.ndarray):
    """q8_1 blocks of rows x: (q int8 [rows, K], d [rows, K/32], s [rows, K/32])."""
    x = np.ascontiguousarray(x, np.float32)
    rows, k = x.shape
    q = np.zeros((rows, k), np.int8)
    d = np.zeros((rows, k // 32), np.float32)
    s = np.zeros((rows, k // 32), np.float32)
    lib().orc_quantize_q81(x.ctypes.data, rows, k, q.ctypes.data, d.ctypes.data, s.ctypes.data)
    return q, d, s


def log_softmax_topk(x: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """Per row of x [rows, n] f32: log_softmax (SUM32 order) and its top k by k
    argmax passes (translator.rs:343-358). Returns (vals [rows, k], idx [rows, k])."""
    x = np.ascontiguousarray(x, np.float32)
    rows, n = x.shape
    vals = np.empty((rows, k), np.float32)
    idx = np.empty((rows, k), np.uint32)
    lib().orc_log_softmax_topk(x.ctypes.data, rows, n, k, vals.ctypes.data, idx.ctypes.data)
    return vals, idx


def strip_eos(row, eos: int) -> list[int]:
    out = []
    for t in row:
        if t == eos:
            break
        out.append(int(t))
    return out
