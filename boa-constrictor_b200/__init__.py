"""boa_b200 -- B200-native BoaConstrictor compress/decompress (Python binding).

The product is ``libboa_b200.so`` (CUDA kernels for sm_100a behind the C ABI in
``include/boa_b200.h``) and the ``bin/boa_constrictor`` CLI.  This module is a
thin ctypes binding over that C ABI for tests and benchmarks; it has no
compute path of its own and raises if the library is missing.

The directory name contains a hyphen, so load it by path::

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location(
        "boa_b200", "boa-constrictor_b200/__init__.py",
        submodule_search_locations=["boa-constrictor_b200"])
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import subprocess

import numpy as np

from . import synth  # noqa: F401  (seeded inputs for tests and bench)
from . import sharding  # noqa: F401  (multi-rank chunk sharding)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libboa_b200.so")
CLI_PATH = os.path.join(HERE, "bin", "boa_constrictor")
HEADER = os.path.join(os.path.dirname(HERE), "include", "boa_b200.h")

BOA_OK, BOA_E_INVALID, BOA_E_CUDA, BOA_E_IO, BOA_E_FORMAT, BOA_E_DEVICE, BOA_E_NOMEM = 0, -1, -2, -3, -4, -5, -6
BOA_STREAM_FAILED = 0xFFFFFFFF  # size of a stream whose coding stopped (handle-free encoders)
BACKBONES = {"mamba": 0, "mambav1": 0, "lstm": 1, "gru": 2, "mingru": 3}
PROF_CLASSES = 12

_u8p, _u32p, _u64p, _f32p = (C.POINTER(C.c_uint8), C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                             C.POINTER(C.c_float))
_i32p = C.POINTER(C.c_int32)


class BoaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"boa error {code}: {msg}")
        self.code = code


def build(jobs: int = 8) -> str:
    """Compile libboa_b200.so and the CLI in-tree (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", HERE], check=True)
    return LIB_PATH


class boa2_info(C.Structure):
    _fields_ = [("total_size", C.c_uint64), ("chunk_len", C.c_uint32), ("n_chunks", C.c_uint32),
                ("last_chunk_len", C.c_uint32), ("flags", C.c_uint32), ("interleave_batch", C.c_uint32),
                ("index_version", C.c_uint32), ("payload_offset", C.c_uint64), ("payload_bytes", C.c_uint64),
                ("fp_len", C.c_uint32), ("fp", C.c_uint8 * 255)]


_LIB = None

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "boa_model_load": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "boa_model_free": (None, [C.c_void_p]),
    "boa_last_error": (C.c_char_p, [C.c_void_p]),
    "boa_set_temperature": (C.c_int, [C.c_void_p, C.c_float]),
    "boa_set_stream": (C.c_int, [C.c_void_p, C.c_void_p]),
    "boa_set_batch": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "boa_set_warm_start": (C.c_int, [C.c_void_p, C.c_uint32]),
    "boa_batch_geometry": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_int, _i32p, _i32p]),
    "boa_reserve": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "boa_stream_capacity_words": (C.c_uint32, [C.c_uint32]),
    "boa_compress_chunks": (C.c_int, [C.c_void_p, _u8p, C.c_size_t, C.c_uint32, C.c_uint32, C.c_uint32, _u8p,
                                      _u32p, C.c_size_t, _u32p, _u64p]),
    "boa_decompress_chunks": (C.c_int, [C.c_void_p, _u32p, _u32p, _u8p, _u32p, C.c_uint32, C.c_uint32, _u8p]),
    "boa_compress_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_void_p,
                                      C.c_void_p, C.c_uint64, C.c_void_p, C.c_void_p]),
    "boa_decompress_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64,
                                        C.c_uint32, C.c_uint32, C.c_void_p]),
    "boa_sync": (C.c_int, [C.c_void_p]),
    "boa_selftest_wait_timeout": (C.c_int, [C.c_int, C.c_uint32]),
    "boa_device_bytes": (C.c_uint64, [C.c_void_p]),
    "boa_set_profiling": (C.c_int, [C.c_void_p, C.c_int]),
    "boa_profile_read": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_double), _u64p]),
    "boa_profile_name": (C.c_char_p, [C.c_int]),
    "boa_launch_count": (C.c_uint64, [C.c_void_p]),
    "boa_model_logits": (C.c_int, [C.c_void_p, _u8p, C.c_int, C.c_int, C.c_int, _f32p]),
    "boa_rc_encode_cdf": (C.c_int, [C.c_void_p, _u32p, _u8p, C.c_int, C.c_int, _u32p, C.c_size_t, _u32p]),
    "boa_rc_decode_cdf": (C.c_int, [C.c_void_p, _u32p, C.c_int, C.c_int, _u32p, _u32p, _u8p]),
    "boa_rc_encode_cdf_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_uint32,
                                            C.c_void_p, C.c_void_p]),
    "boa_rc_state_bytes": (C.c_size_t, [C.c_int]),
    "boa_rc_encoder_init": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p]),
    "boa_rc_encode_cdf_steps": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                          C.c_uint32, C.c_void_p]),
    "boa_rc_encoder_finish": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_int, C.c_void_p]),
    "boa_rc_decoder_init": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "boa_rc_decode_cdf_steps": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p]),
    "boa_cdf_from_logits": (C.c_int, [C.c_void_p, _f32p, C.c_int, C.c_float, _u32p]),
    "boa_boa2_build": (C.c_int, [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _u8p,
                                 _u64p, _u8p, _u8p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "boa_boa2_build_fp": (C.c_int, [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _u8p, C.c_uint32,
                                    _u8p, _u64p, _u8p, _u8p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "boa_boa2_parse": (C.c_int, [_u8p, C.c_size_t, C.POINTER(boa2_info), _u8p, _u64p, _u64p]),
    "boa_pyrc_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "boa_pyrc_free": (None, [C.c_void_p]),
    "boa_pyrc_last_error": (C.c_char_p, [C.c_void_p]),
    "boa_pyrc_encode_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "boa_pyrc_finalize": (C.c_int, [C.c_void_p, C.c_void_p]),
    "boa_pyrc_read": (C.c_int, [C.c_void_p, _u32p, _i32p, C.c_void_p]),
    "boa_pyrc_load": (C.c_int, [C.c_void_p, _u32p, _i32p, C.c_void_p]),
    "boa_pyrc_init_decoder": (C.c_int, [C.c_void_p, C.c_void_p]),
    "boa_pyrc_decode_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
}


def lib():
    """The loaded libboa_b200.so.  Raises when it has not been built: there is
    no fallback implementation."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run boa_b200.build() (nvcc, sm_100a)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _p(a, t):
    return a.ctypes.data_as(t)


def _check(rc, h=None):
    if rc != 0:
        raise BoaError(rc, (lib().boa_last_error(h) or b"").decode())


def capacity_words(chunk_len: int) -> int:
    return int(lib().boa_stream_capacity_words(chunk_len))


class Model:
    """One library handle (one GPU).  Mirrors BoaPredictorGPU's construction
    from a .bin weight file plus the CLI's dims (boa.cpp:912-919)."""

    def __init__(self, path: str, backbone="mamba", d_model: int = 256, n_layers: int = 8, device: int = 0):
        h = C.c_void_p()
        bb = BACKBONES.get(backbone, -1) if isinstance(backbone, str) else int(backbone)
        rc = lib().boa_model_load(path.encode(), bb, d_model, n_layers, device, C.byref(h))
        if rc != 0:
            raise BoaError(rc, lib().boa_last_error(None).decode())
        self.h = h
        self.d_model, self.n_layers = d_model, n_layers

    def close(self):
        if getattr(self, "h", None):
            lib().boa_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_temperature(self, t: float):
        _check(lib().boa_set_temperature(self.h, t), self.h)

    def set_batch(self, chunks: int = 0, tile: int = 0):
        _check(lib().boa_set_batch(self.h, chunks, tile), self.h)

    def batch_geometry(self, n_chunks: int, chunk_len: int, compress: bool = True):
        """-> (chunks per batch, positions per compress tile) the next call would use."""
        b, t = C.c_int32(), C.c_int32()
        _check(lib().boa_batch_geometry(self.h, n_chunks, chunk_len, int(bool(compress)), C.byref(b), C.byref(t)),
               self.h)
        return b.value, t.value

    def reserve(self, n_chunks: int, chunk_len: int):
        """Allocate now what calls over this geometry will need."""
        _check(lib().boa_reserve(self.h, n_chunks, chunk_len), self.h)

    def set_warm_start(self, interleave_batch: int):
        _check(lib().boa_set_warm_start(self.h, interleave_batch), self.h)

    def set_stream(self, stream_ptr: int | None):
        _check(lib().boa_set_stream(self.h, C.c_void_p(stream_ptr or 0)), self.h)

    def sync(self):
        _check(lib().boa_sync(self.h), self.h)

    def device_bytes(self) -> int:
        return int(lib().boa_device_bytes(self.h))

    def set_profiling(self, on: bool):
        _check(lib().boa_set_profiling(self.h, int(bool(on))), self.h)

    def profile(self) -> dict:
        """{kernel class: (total ms, launches)} since the last read."""
        out = {}
        for c in range(PROF_CLASSES):
            ms, n = C.c_double(), C.c_uint64()
            _check(lib().boa_profile_read(self.h, c, C.byref(ms), C.byref(n)), self.h)
            out[lib().boa_profile_name(c).decode()] = (ms.value, n.value)
        return out

    def launch_count(self) -> int:
        return int(lib().boa_launch_count(self.h))

    # device-buffer API (ints are raw device pointers)
    def compress_device(self, d_data: int, n_bytes: int, chunk_len: int, n_chunks: int, d_first: int,
                        d_payload: int, cap_words: int, d_sizes: int, d_offsets: int):
        _check(lib().boa_compress_device(self.h, d_data, n_bytes, chunk_len, n_chunks, d_first, d_payload,
                                         cap_words, d_sizes, d_offsets), self.h)

    def decompress_device(self, d_payload: int, d_offsets: int, d_sizes: int, d_first: int, n_bytes: int,
                          chunk_len: int, n_chunks: int, d_out: int):
        _check(lib().boa_decompress_device(self.h, d_payload, d_offsets, d_sizes, d_first, n_bytes, chunk_len,
                                           n_chunks, d_out), self.h)

    # ---------------------------------------------------------------- codec
    def compress(self, data: bytes, chunk_len: int, first_chunk: int = 0, n_chunks: int | None = None):
        """-> (first_bytes u8[n], sizes u32[n] (words), payload u32[total])."""
        arr = np.frombuffer(data, np.uint8) if len(data) else np.zeros(1, np.uint8)
        total_chunks = (len(data) + chunk_len - 1) // chunk_len
        if n_chunks is None:
            n_chunks = total_chunks - first_chunk
        fb = np.zeros(max(n_chunks, 1), np.uint8)
        sizes = np.zeros(max(n_chunks, 1), np.uint32)
        cap = max(n_chunks, 1) * capacity_words(chunk_len)
        pay = np.zeros(cap, np.uint32)
        used = C.c_uint64()
        _check(lib().boa_compress_chunks(self.h, _p(arr, _u8p), len(data), chunk_len, first_chunk, n_chunks,
                                         _p(fb, _u8p), _p(pay, _u32p), cap, _p(sizes, _u32p), C.byref(used)),
               self.h)
        return fb[:n_chunks], sizes[:n_chunks], pay[:used.value].copy()

    def decompress(self, first_bytes, sizes, payload, chunk_lens, chunk_len: int) -> bytes:
        n = len(sizes)
        fb = np.ascontiguousarray(first_bytes, np.uint8)
        sz = np.ascontiguousarray(sizes, np.uint32)
        cl = np.ascontiguousarray(chunk_lens, np.uint32)
        pay = np.ascontiguousarray(payload, np.uint32)
        if pay.size == 0:
            pay = np.zeros(1, np.uint32)
        out = np.zeros(max(int(cl.sum()), 1), np.uint8)
        _check(lib().boa_decompress_chunks(self.h, _p(pay, _u32p), _p(sz, _u32p), _p(fb, _u8p), _p(cl, _u32p),
                                           chunk_len, n, _p(out, _u8p)), self.h)
        return out[:int(cl.sum())].tobytes()

    def logits(self, tokens: np.ndarray, mode: int = 0) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, np.uint8)
        B, L = tok.shape
        out = np.zeros((B, L, 256), np.float32)
        _check(lib().boa_model_logits(self.h, _p(tok, _u8p), B, L, mode, _p(out, _f32p)), self.h)
        return out

    def cdf_from_logits(self, logits: np.ndarray, inv_temperature: float = 1.0) -> np.ndarray:
        lg = np.ascontiguousarray(logits, np.float32).reshape(-1, 256)
        Q = np.zeros((lg.shape[0], 257), np.uint32)
        _check(lib().boa_cdf_from_logits(self.h, _p(lg, _f32p), lg.shape[0], inv_temperature, _p(Q, _u32p)),
               self.h)
        return Q

    def rc_encode_cdf(self, cdf: np.ndarray, syms: np.ndarray):
        """cdf [steps][streams][257], syms [steps][streams] -> (sizes, payload)."""
        Q = np.ascontiguousarray(cdf, np.uint32)
        S = np.ascontiguousarray(syms, np.uint8)
        nt, ns = S.shape
        cap = ns * capacity_words(nt + 1)
        pay = np.zeros(cap, np.uint32)
        sizes = np.zeros(ns, np.uint32)
        _check(lib().boa_rc_encode_cdf(self.h, _p(Q, _u32p), _p(S, _u8p), ns, nt, _p(pay, _u32p), cap,
                                       _p(sizes, _u32p)), self.h)
        return sizes, pay[:int(sizes.sum())].copy()

    def rc_decode_cdf(self, cdf: np.ndarray, sizes, payload) -> np.ndarray:
        Q = np.ascontiguousarray(cdf, np.uint32)
        nt, ns = Q.shape[0], Q.shape[1]
        sz = np.ascontiguousarray(sizes, np.uint32)
        pay = np.ascontiguousarray(payload, np.uint32)
        if pay.size == 0:
            pay = np.zeros(1, np.uint32)
        out = np.zeros((max(nt, 1), ns), np.uint8)
        _check(lib().boa_rc_decode_cdf(self.h, _p(Q, _u32p), ns, nt, _p(pay, _u32p), _p(sz, _u32p),
                                       _p(out, _u8p)), self.h)
        return out[:nt]


# -------------------------------------------------------------------- container
PYTHON_MODEL_CLASS = "BoaBytePredictor"  # the nn.Module that model.BoaConstrictor() returns (model.py:1754)


def python_fingerprint(class_name: str = PYTHON_MODEL_CLASS) -> bytes:
    """The fingerprint field Python BoaFile writes: blake2s of the model's class
    name, 16-byte digest (boa.py:107-109)."""
    return hashlib.blake2s(class_name.encode(), digest_size=16).digest()


def boa2_build(total_size: int, chunk_len: int, first_bytes, sizes_words, payload_words, warm_start: int = 0,
               fingerprint: bytes | None = None) -> bytes:
    """warm_start = interleave batch W of a warm-start container (flags bit0), 0 = off.
    fingerprint: bytes stored verbatim in the fingerprint field (e.g.
    python_fingerprint() for a file in the Python BoaFile dialect); None keeps
    the C++ writer's rule."""
    n = len(sizes_words)
    last = total_size - (n - 1) * chunk_len if n > 1 else total_size
    fb = np.ascontiguousarray(first_bytes, np.uint8)
    sb = np.ascontiguousarray(np.asarray(sizes_words, np.uint64) * 4)
    pay = np.ascontiguousarray(payload_words, np.uint32).view(np.uint8)
    if pay.size == 0:
        pay = np.zeros(1, np.uint8)
    if fb.size == 0:
        fb = np.zeros(1, np.uint8)
    if sb.size == 0:
        sb = np.zeros(1, np.uint64)
    ln = C.c_size_t()
    flags = 1 if warm_start else 0
    if fingerprint is None:
        def call(out, cap):
            return lib().boa_boa2_build(total_size, chunk_len, n, last, flags, warm_start, _p(fb, _u8p),
                                        _p(sb, _u64p), _p(pay, _u8p), out, cap, C.byref(ln))
    else:
        fp = np.frombuffer(bytes(fingerprint) or b"\0", np.uint8).copy()

        def call(out, cap):
            return lib().boa_boa2_build_fp(total_size, chunk_len, n, last, flags, _p(fp, _u8p), len(fingerprint),
                                           _p(fb, _u8p), _p(sb, _u64p), _p(pay, _u8p), out, cap, C.byref(ln))
    _check(call(None, 0))
    buf = np.zeros(ln.value, np.uint8)
    _check(call(_p(buf, _u8p), buf.size))
    return buf.tobytes()


def boa2_parse(blob: bytes) -> dict:
    arr = np.frombuffer(blob, np.uint8)
    info = boa2_info()
    rc = lib().boa_boa2_parse(_p(arr, _u8p), arr.size, C.byref(info), None, None, None)
    if rc != 0:
        raise BoaError(rc, "malformed BOA2 container")
    n = info.n_chunks
    fb = np.zeros(max(n, 1), np.uint8)
    off = np.zeros(max(n, 1), np.uint64)
    ln = np.zeros(max(n, 1), np.uint64)
    _check(lib().boa_boa2_parse(_p(arr, _u8p), arr.size, C.byref(info), _p(fb, _u8p), _p(off, _u64p),
                                _p(ln, _u64p)))
    base = info.payload_offset
    streams = [blob[base + int(o): base + int(o) + int(l)] for o, l in zip(off[:n], ln[:n])]
    return dict(total_size=info.total_size, chunk_len=info.chunk_len, n_chunks=n,
                last_chunk_len=info.last_chunk_len, flags=info.flags, interleave_batch=info.interleave_batch,
                index_version=info.index_version, first_bytes=fb[:n].copy(), streams=streams,
                fingerprint=bytes(info.fp[:info.fp_len]))
