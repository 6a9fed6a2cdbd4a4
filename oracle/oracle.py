"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, as the checker.  The product (libboa_b200.so) never
loads it.  See boa_oracle.h for what each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_lib = None


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_load.restype = C.c_void_p
        L.orc_load.argtypes = [C.c_char_p, C.c_int, C.c_int, C.c_int]
        L.orc_free.argtypes = [C.c_void_p]
        L.orc_last_error.restype = C.c_char_p
        L.orc_logits.argtypes = [C.c_void_p, _u8p, C.c_int, C.c_int, C.c_int, _f32p]
        L.orc_cdf_rows.argtypes = [_f32p, C.c_int, C.c_float, _u32p]
        L.orc_rc_encode_cdf.argtypes = [_u32p, _u8p, C.c_int, _u32p, C.c_int]
        L.orc_rc_decode_cdf.argtypes = [_u32p, C.c_int, _u32p, C.c_int, _u8p]
        L.orc_compress.argtypes = [C.c_void_p, _u8p, C.c_size_t, C.c_uint32, C.c_float, C.c_int,
                                   _u8p, _u32p, C.c_uint32, _u32p]
        L.orc_decompress.argtypes = [C.c_void_p, _u32p, C.c_uint32, _u32p, _u8p, C.c_size_t,
                                     C.c_uint32, C.c_float, C.c_int, _u8p]
        L.orc_compress_warm.argtypes = [C.c_void_p, _u8p, C.c_size_t, C.c_uint32, C.c_uint32, C.c_float, C.c_int,
                                        _u8p, _u32p, C.c_uint32, _u32p]
        L.orc_decompress_warm.argtypes = [C.c_void_p, _u32p, C.c_uint32, _u32p, _u8p, C.c_size_t, C.c_uint32,
                                          C.c_uint32, C.c_float, C.c_int, _u8p]
        L.orc_pyrc_cdf_rows.argtypes = [_f32p, C.c_int, C.c_int, _u32p]
        L.orc_pyrc_encode.argtypes = [_f32p, _i32p, C.c_int, C.c_int, _u32p, C.c_int]
        L.orc_pyrc_decode.argtypes = [_f32p, C.c_int, C.c_int, _u32p, C.c_int, _i32p]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def pitch_words(chunk_len: int) -> int:
    """Per-chunk stream capacity in words, boa.cpp:338."""
    return (chunk_len * 10 + 4096 + 3) // 4


class OracleModel:
    def __init__(self, path: str, backbone: int = 0, d_model: int = 256, n_layers: int = 8):
        self.h = lib().orc_load(path.encode(), backbone, d_model, n_layers)
        if not self.h:
            raise RuntimeError(lib().orc_last_error().decode())

    def close(self):
        if self.h:
            lib().orc_free(self.h)
            self.h = None

    __del__ = close

    def logits(self, tokens: np.ndarray, mode: int = 0) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint8)
        B, L = tokens.shape
        out = np.empty((B, L, 256), np.float32)
        lib().orc_logits(self.h, _p(tokens, _u8p), B, L, mode, _p(out, _f32p))
        return out

    def compress(self, data: bytes, chunk_len: int, inv_temperature: float = 1.0, threads: int = 0,
                 warm: int = 0):
        n = len(data)
        nc = (n + chunk_len - 1) // chunk_len
        pw = pitch_words(chunk_len)
        arr = np.frombuffer(data, np.uint8) if n else np.zeros(1, np.uint8)
        fb = np.zeros(max(nc, 1), np.uint8)
        words = np.zeros(max(nc, 1) * pw, np.uint32)
        sizes = np.zeros(max(nc, 1), np.uint32)
        if warm:
            rc = lib().orc_compress_warm(self.h, _p(arr, _u8p), n, chunk_len, warm, inv_temperature,
                                         threads or os.cpu_count(), _p(fb, _u8p), _p(words, _u32p), pw,
                                         _p(sizes, _u32p))
        else:
            rc = lib().orc_compress(self.h, _p(arr, _u8p), n, chunk_len, inv_temperature,
                                    threads or os.cpu_count(), _p(fb, _u8p), _p(words, _u32p), pw,
                                    _p(sizes, _u32p))
        if rc != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        streams = [words[i * pw: i * pw + sizes[i]].copy() for i in range(nc)]
        return fb[:nc].copy(), streams

    def decompress(self, first_bytes, streams, n: int, chunk_len: int,
                   inv_temperature: float = 1.0, threads: int = 0, warm: int = 0) -> bytes:
        nc = len(streams)
        pw = pitch_words(chunk_len)
        words = np.zeros(max(nc, 1) * pw, np.uint32)
        sizes = np.zeros(max(nc, 1), np.uint32)
        for i, s in enumerate(streams):
            words[i * pw: i * pw + len(s)] = s
            sizes[i] = len(s)
        fb = np.ascontiguousarray(np.asarray(first_bytes, np.uint8))
        if fb.size == 0:
            fb = np.zeros(1, np.uint8)
        out = np.zeros(max(n, 1), np.uint8)
        if warm:
            lib().orc_decompress_warm(self.h, _p(words, _u32p), pw, _p(sizes, _u32p), _p(fb, _u8p), n,
                                      chunk_len, warm, inv_temperature, threads or os.cpu_count(), _p(out, _u8p))
        else:
            lib().orc_decompress(self.h, _p(words, _u32p), pw, _p(sizes, _u32p), _p(fb, _u8p), n,
                                 chunk_len, inv_temperature, threads or os.cpu_count(), _p(out, _u8p))
        return out[:n].tobytes()


def cdf_rows(logits: np.ndarray, inv_temperature: float = 1.0) -> np.ndarray:
    lg = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1, 256)
    Q = np.empty((lg.shape[0], 257), np.uint32)
    lib().orc_cdf_rows(_p(lg, _f32p), lg.shape[0], inv_temperature, _p(Q, _u32p))
    return Q


def rc_encode_cdf(Q: np.ndarray, syms: np.ndarray) -> np.ndarray:
    Q = np.ascontiguousarray(Q, dtype=np.uint32)
    syms = np.ascontiguousarray(syms, dtype=np.uint8)
    n = syms.size
    cap = 3 * n + 16
    out = np.zeros(cap, np.uint32)
    w = lib().orc_rc_encode_cdf(_p(Q, _u32p), _p(syms, _u8p), n, _p(out, _u32p), cap)
    if w < 0:
        raise RuntimeError("stream overflow")
    return out[:w].copy()


def rc_decode_cdf(Q: np.ndarray, words: np.ndarray, n: int) -> np.ndarray:
    Q = np.ascontiguousarray(Q, dtype=np.uint32)
    words = np.ascontiguousarray(words, dtype=np.uint32)
    wbuf = words if words.size else np.zeros(1, np.uint32)
    syms = np.zeros(max(n, 1), np.uint8)
    lib().orc_rc_decode_cdf(_p(Q, _u32p), n, _p(wbuf, _u32p), words.size, _p(syms, _u8p))
    return syms[:n]


# ---- the Python codec's coder (gpu_range_coder.py) -------------------------
def pyrc_cdf_rows(probs: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(probs, dtype=np.float32)
    K = p.shape[-1]
    p = p.reshape(-1, K)
    out = np.empty((p.shape[0], K + 1), np.uint32)
    lib().orc_pyrc_cdf_rows(_p(p, _f32p), p.shape[0], K, _p(out, _u32p))
    return out


def pyrc_encode(probs: np.ndarray, syms: np.ndarray) -> np.ndarray:
    """One stream: probs [n][K] float32, syms [n] int32 -> uint32 words."""
    p = np.ascontiguousarray(probs, dtype=np.float32)
    s = np.ascontiguousarray(syms, dtype=np.int32)
    n, K = p.shape
    cap = 3 * n + 16
    out = np.zeros(cap, np.uint32)
    w = lib().orc_pyrc_encode(_p(p, _f32p), _p(s, _i32p), n, K, _p(out, _u32p), cap)
    if w < 0:
        raise RuntimeError("stream overflow")
    return out[:w].copy()


def pyrc_decode(probs: np.ndarray, words: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(probs, dtype=np.float32)
    n, K = p.shape
    wd = np.ascontiguousarray(words, dtype=np.uint32)
    wbuf = wd if wd.size else np.zeros(1, np.uint32)
    out = np.zeros(max(n, 1), np.int32)
    lib().orc_pyrc_decode(_p(p, _f32p), n, K, _p(wbuf, _u32p), wd.size, _p(out, _i32p))
    return out[:n]
