"""The allocation-free encoder entry point (boa_rc_encode_cdf_noalloc).

Callers that cannot allocate device memory at the call site -- code under a
pooled or framework-owned allocator that forbids raw cudaMalloc, plugins that
must keep a fixed memory footprint -- use this entry point: it keeps its only
scratch (the per-stream coder states) in a static device array and writes into
buffers the caller owns.  Its streams must equal those of the regular
boa_rc_encode_cdf bit for bit, on consecutive calls (the static array keeps the
previous call's contents, so each call must reset what it uses).  A stream
whose coding stops on the device is reported to this handle-free caller by its
size (BOA_STREAM_FAILED), never through a model handle's error state.

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


def _noalloc(boa, Q, syms, pitch, words=None, sizes=None):
    import torch
    dev = torch.device("cuda", 0)
    nt, ns = syms.shape
    d_q = torch.from_numpy(np.ascontiguousarray(Q, np.uint32).view(np.int32)).to(dev)
    d_s = torch.from_numpy(np.ascontiguousarray(syms)).to(dev)
    d_w = words if words is not None else torch.full((ns * pitch,), -1, dtype=torch.int32, device=dev)
    d_n = sizes if sizes is not None else torch.full((ns,), 7, dtype=torch.int32, device=dev)
    rc = boa.lib().boa_rc_encode_cdf_noalloc(C.c_void_p(d_q.data_ptr()), C.c_void_p(d_s.data_ptr()), ns, nt,
                                             C.c_void_p(d_w.data_ptr()), pitch, C.c_void_p(d_n.data_ptr()), None)
    torch.cuda.synchronize()
    return rc, d_w, d_n


def test_noalloc_failed_stream_is_marked_and_handles_stay_clean(boa, weights):
    """An empty interval in stream 1 marks that stream's size BOA_STREAM_FAILED;
    the other streams still equal the allocating encoder's, and a model handle
    on the same device syncs clean afterwards (the failure is not left in the
    device error word for it)."""
    m = boa.Model(weights("mamba", 64, 2, 3), "mamba", 64, 2)
    rng = np.random.default_rng(5)
    Q, syms = dirichlet_cdfs(rng, 120, 4)
    bad = Q.copy()
    s0 = int(syms[30, 1])
    bad[30, 1, s0 + 1] = bad[30, 1, s0]
    pitch = boa.capacity_words(121)
    rc, d_w, d_n = _noalloc(boa, bad, syms, pitch)
    assert rc == 0
    sizes = d_n.cpu().numpy().view(np.uint32)
    assert sizes[1] == boa.BOA_STREAM_FAILED
    ref_sizes, ref_pay = m.rc_encode_cdf(Q, syms)
    words = d_w.cpu().numpy().view(np.uint32).reshape(4, pitch)
    o = 0
    for i in range(4):
        if i != 1:
            assert sizes[i] == ref_sizes[i] and np.array_equal(words[i, :sizes[i]], ref_pay[o:o + sizes[i]])
        o += int(ref_sizes[i])
    m.sync()  # raises if the failure had been left in the device error word


def test_noalloc_edges_and_no_allocation(boa):
    """n_steps = 0 gives empty streams (size 0); a pitch one word below
    boa_stream_capacity_words(n_steps + 1) is rejected; repeated calls leave
    the device's free memory unchanged."""
    import torch
    Q, syms = dirichlet_cdfs(np.random.default_rng(8), 64, 300)
    pitch = boa.capacity_words(65)
    dev = torch.device("cuda", 0)
    q1 = torch.zeros(257, dtype=torch.int32, device=dev)  # valid pointers; nothing is read at n_steps = 0
    s1 = torch.zeros(1, dtype=torch.uint8, device=dev)
    w0 = torch.full((300 * pitch,), -1, dtype=torch.int32, device=dev)
    n0 = torch.full((300,), 7, dtype=torch.int32, device=dev)
    rc = boa.lib().boa_rc_encode_cdf_noalloc(C.c_void_p(q1.data_ptr()), C.c_void_p(s1.data_ptr()), 300, 0,
                                             C.c_void_p(w0.data_ptr()), pitch, C.c_void_p(n0.data_ptr()), None)
    torch.cuda.synchronize()
    assert rc == 0 and np.all(n0.cpu().numpy() == 0)
    rc = boa.lib().boa_rc_encode_cdf_noalloc(C.c_void_p(16), C.c_void_p(16), 300, 64, C.c_void_p(16), pitch - 1,
                                             C.c_void_p(16), None)
    assert rc == boa.BOA_E_INVALID and b"pitch" in boa.lib().boa_last_error(None)
    d_w = torch.empty(300 * pitch, dtype=torch.int32, device=dev)
    d_n = torch.empty(300, dtype=torch.int32, device=dev)
    _noalloc(boa, Q, syms, pitch, d_w, d_n)  # warm-up: module and symbol already resident after this
    d_q = torch.from_numpy(Q.view(np.int32)).to(dev)
    d_s = torch.from_numpy(syms).to(dev)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for _ in range(3):
        rc = boa.lib().boa_rc_encode_cdf_noalloc(C.c_void_p(d_q.data_ptr()), C.c_void_p(d_s.data_ptr()), 300, 64,
                                                 C.c_void_p(d_w.data_ptr()), pitch, C.c_void_p(d_n.data_ptr()), None)
        assert rc == 0
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(0)[0]
    assert free1 == free0, (free0, free1, free0 - free1)


def test_noalloc_encoder_rejects_oversize(boa):
    L = boa.lib()
    one = C.c_void_p(16)  # never dereferenced: the size check comes first
    rc = L.boa_rc_encode_cdf_noalloc(one, one, 65537, 10, one, boa.capacity_words(11), one, None)
    assert rc == boa.BOA_E_INVALID
    assert b"maximum" in L.boa_last_error(None)


def test_noalloc_rejects_a_stream_of_another_device(boa):
    """The coder states live on the current device; a stream created on
    another GPU is an argument error, not a launch failure.  Needs two GPUs."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two or more GPUs")
    other = torch.cuda.Stream(device=1)
    torch.cuda.set_device(0)
    one = C.c_void_p(16)  # never dereferenced: the stream check comes first
    rc = boa.lib().boa_rc_encode_cdf_noalloc(one, one, 4, 10, one, boa.capacity_words(11), one,
                                             C.c_void_p(other.cuda_stream))
    assert rc == boa.BOA_E_INVALID and b"another device" in boa.lib().boa_last_error(None)
