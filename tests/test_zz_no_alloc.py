"""The allocation-free encoder entry point (boa_rc_encode_cdf_noalloc).

Callers that cannot allocate device memory at the call site -- code under a
pooled or framework-owned allocator that forbids raw cudaMalloc, plugins that
must keep a fixed memory footprint -- use this entry point: it keeps its only
scratch (the per-stream coder states) in a static device array and writes into
buffers the caller owns.  Its streams must equal those of the regular
boa_rc_encode_cdf bit for bit, on consecutive calls (the static array keeps the
previous call's contents, so each call must reset what it uses).

This file is named to be collected last; it must also pass alone in a fresh
process.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import dirichlet_cdfs

pytestmark = pytest.mark.gpu


def test_noalloc_encoder_matches_allocating_encoder_twice(boa, weights):
    import torch
    m = boa.Model(weights("mamba", 64, 2, 3), "mamba", 64, 2)
    L = boa.lib()
    dev = torch.device("cuda", 0)
    for call, (ns, nt) in enumerate([(37, 400), (19, 250)]):  # second call: fewer streams, shorter
        rng = np.random.default_rng(100 + call)
        Q, syms = dirichlet_cdfs(rng, nt, ns)
        sizes_ref, pay_ref = m.rc_encode_cdf(Q, syms)
        pitch = boa.capacity_words(nt + 1)
        d_q = torch.from_numpy(Q.astype(np.int64).astype(np.uint32).view(np.int32)).to(dev)
        d_s = torch.from_numpy(syms).to(dev)
        d_w = torch.full((ns * pitch,), -1, dtype=torch.int32, device=dev)
        d_n = torch.zeros(ns, dtype=torch.int32, device=dev)
        rc = L.boa_rc_encode_cdf_noalloc(C.c_void_p(d_q.data_ptr()), C.c_void_p(d_s.data_ptr()), ns, nt,
                                         C.c_void_p(d_w.data_ptr()), pitch, C.c_void_p(d_n.data_ptr()), None)
        assert rc == 0, L.boa_last_error(None)
        torch.cuda.synchronize()
        sizes = d_n.cpu().numpy().view(np.uint32)
        words = d_w.cpu().numpy().view(np.uint32).reshape(ns, pitch)
        assert np.array_equal(sizes, sizes_ref)
        o = 0
        for i in range(ns):
            assert np.array_equal(words[i, :sizes[i]], pay_ref[o:o + sizes[i]])
            o += int(sizes[i])


def test_noalloc_encoder_rejects_oversize(boa):
    L = boa.lib()
    one = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.boa_rc_encode_cdf_noalloc(one, one, 65537, 10, one, boa.capacity_words(11), one, None)
    assert rc == boa.BOA_E_INVALID
    assert b"maximum" in L.boa_last_error(None)
