"""Drop-in for the Python codec's GPU batch coder.

``gpu.queue.RangeCoderBatch`` here has the constructor, methods and
argument meaning of ``gpu_range_coder.gpu.queue.RangeCoderBatch``
(gpu_range_coder.py:466-550), which ``codec.compress_GPU`` /
``decompress_GPU`` (codec.py:11-151) drive once per position with
``torch.softmax`` rows.  The work runs in this package's sm_100a kernels
(the ``boa_pyrc_*`` entry points of libboa_b200.so) and the streams are bit
for bit the reference's for the same probabilities, so ``.boa`` files of the
Python path are written and read unchanged.  A codec switches with::

    from boa_b200 import pycoder as gr   # in place of: import gpu_range_coder as gr

Differences: work is enqueued on torch's current stream instead of being
followed by a device-wide synchronisation (the ``get_*`` calls synchronise),
and a stream that outgrows the pitch raises instead of writing past it.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import BoaError, lib, _i32p, _u32p, _p


class _RangeCoderBatch:
    def __init__(self, N: int, K: int, maxL: int, pitch_bytes: int | None = None):
        import torch
        if pitch_bytes is None:
            pitch_bytes = max(256, maxL * 8)
        self.N, self.K, self.maxL = int(N), int(K), int(maxL)
        self.pitch = (int(pitch_bytes) + 3) // 4
        self.device = torch.cuda.current_device()
        self._torch = torch
        self.h = None
        h = C.c_void_p()
        rc = lib().boa_pyrc_create(self.N, self.K, self.pitch, self.device, C.byref(h))
        if rc != 0:
            raise BoaError(rc, (lib().boa_pyrc_last_error(None) or b"").decode())
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib().boa_pyrc_free(self.h)
            self.h = None

    def _check(self, rc: int):
        if rc != 0:
            raise BoaError(rc, (lib().boa_pyrc_last_error(self.h) or b"").decode())

    def _stream(self):
        return C.c_void_p(self._torch.cuda.current_stream(self.device).cuda_stream)

    def _mask_ptr(self, mask):
        if mask is None:
            return None, None
        assert mask.is_cuda and mask.shape == (self.N,)
        if mask.dtype not in (self._torch.uint8, self._torch.bool):
            mask = mask.to(self._torch.uint8)
        mask = mask.contiguous()
        return mask, C.c_void_p(mask.data_ptr())

    def load_compressed_list(self, compressed_list):
        if len(compressed_list) != self.N:
            raise RuntimeError("compressed_list length must equal N")
        words = np.zeros((self.N, self.pitch), np.uint32)
        sizes = np.zeros(self.N, np.int32)
        for i, arr in enumerate(compressed_list):
            a = np.asarray(arr)
            if a.ndim != 1 or a.dtype.itemsize != 4 or a.dtype.kind != "u":
                raise RuntimeError("Each compressed item must be uint32[?]")
            if a.size > self.pitch:
                raise RuntimeError("Compressed stream exceeds pitch; increase pitch")
            words[i, :a.size] = a
            sizes[i] = a.size
        self._check(lib().boa_pyrc_load(self.h, _p(words, _u32p), _p(sizes, _i32p), self._stream()))

    def encode_step(self, symbols_gpu, probs_gpu, mask=None):
        torch = self._torch
        assert symbols_gpu.is_cuda and probs_gpu.is_cuda
        assert symbols_gpu.numel() == self.N and probs_gpu.shape == (self.N, self.K)
        syms = symbols_gpu.to(torch.int32).contiguous()
        probs = probs_gpu.to(torch.float32).contiguous()
        mask, mp = self._mask_ptr(mask)
        self._check(lib().boa_pyrc_encode_step(self.h, C.c_void_p(syms.data_ptr()), C.c_void_p(probs.data_ptr()),
                                               mp, self._stream()))

    def finalize(self):
        self._check(lib().boa_pyrc_finalize(self.h, self._stream()))

    def get_compressed_list(self):
        words = np.zeros((self.N, self.pitch), np.uint32)
        sizes = np.zeros(self.N, np.int32)
        self._check(lib().boa_pyrc_read(self.h, _p(words, _u32p), _p(sizes, _i32p), self._stream()))
        return [words[i, :sizes[i]].copy() for i in range(self.N)]

    def get_sizes_list(self):
        sizes = np.zeros(self.N, np.int32)
        self._check(lib().boa_pyrc_read(self.h, None, _p(sizes, _i32p), self._stream()))
        return sizes.tolist()

    def init_decoder(self):
        self._check(lib().boa_pyrc_init_decoder(self.h, self._stream()))

    def decode_step(self, probs_gpu, out_symbols_gpu, mask=None):
        torch = self._torch
        assert probs_gpu.is_cuda and out_symbols_gpu.is_cuda
        assert probs_gpu.shape == (self.N, self.K) and out_symbols_gpu.numel() == self.N
        assert out_symbols_gpu.dtype == torch.int32 and out_symbols_gpu.is_contiguous()
        probs = probs_gpu.to(torch.float32).contiguous()
        mask, mp = self._mask_ptr(mask)
        self._check(lib().boa_pyrc_decode_step(self.h, C.c_void_p(probs.data_ptr()),
                                               C.c_void_p(out_symbols_gpu.data_ptr()), mp, self._stream()))


class gpu:
    class queue:
        RangeCoderBatch = _RangeCoderBatch
