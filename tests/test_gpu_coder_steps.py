"""The step-wise, handle-free integer-CDF coder (boa_rc_encoder_init /
boa_rc_encode_cdf_steps / boa_rc_encoder_finish / boa_rc_decoder_init /
boa_rc_decode_cdf_steps), the shape of the reference's gpu_rc_init ->
per-position launches -> gpu_rc_finish_batch -> gpu_rc_init_decoder ->
per-position decode (range_coder_kernels.cu:46-60, :279-340, :479-490).

Streams coded in tiles of any length must equal, word for word, the CPU coder
(the oracle's restatement of the reference coder) on the same integer CDFs,
and decode back in tiles of other lengths."""
import ctypes as C

import numpy as np
import pytest

from conftest import dirichlet_cdfs

pytestmark = pytest.mark.gpu


def _vp(t):
    return C.c_void_p(t.data_ptr())


def _encode_tiles(boa, Q, syms, tiles, pitch):
    import torch
    L = boa.lib()
    dev = torch.device("cuda", 0)
    nt, ns = syms.shape
    es = torch.empty(ns * L.boa_rc_state_bytes(0), dtype=torch.uint8, device=dev)
    words = torch.full((ns * pitch,), -1, dtype=torch.int32, device=dev)
    sizes = torch.zeros(ns, dtype=torch.int32, device=dev)
    assert L.boa_rc_encoder_init(_vp(es), ns, None) == 0
    t0 = 0
    for n in tiles:
        q = torch.from_numpy(np.ascontiguousarray(Q[t0:t0 + n]).view(np.int32)).to(dev)
        s = torch.from_numpy(np.ascontiguousarray(syms[t0:t0 + n])).to(dev)
        assert L.boa_rc_encode_cdf_steps(_vp(es), _vp(q), _vp(s), ns, n, _vp(words), pitch, None) == 0
        torch.cuda.synchronize()  # q and s are released at the end of the iteration
        t0 += n
    assert t0 == nt
    assert L.boa_rc_encoder_finish(_vp(es), _vp(words), pitch, _vp(sizes), ns, None) == 0
    torch.cuda.synchronize()
    return words, sizes


def _decode_tiles(boa, Q, words, sizes, pitch, tiles):
    import torch
    L = boa.lib()
    dev = torch.device("cuda", 0)
    nt, ns = Q.shape[0], Q.shape[1]
    ds = torch.empty(ns * L.boa_rc_state_bytes(1), dtype=torch.uint8, device=dev)
    off = torch.arange(ns, dtype=torch.int64, device=dev) * pitch
    assert L.boa_rc_decoder_init(_vp(ds), _vp(words), _vp(off), _vp(sizes), ns, None) == 0
    out = []
    t0 = 0
    for n in tiles:
        q = torch.from_numpy(np.ascontiguousarray(Q[t0:t0 + n]).view(np.int32)).to(dev)
        got = torch.empty((n, ns), dtype=torch.uint8, device=dev)
        assert L.boa_rc_decode_cdf_steps(_vp(ds), _vp(q), ns, n, _vp(words), _vp(off), _vp(got), None) == 0
        out.append(got.cpu().numpy())
        t0 += n
    return np.concatenate(out)


@pytest.mark.parametrize("ns,enc_tiles,dec_tiles", [(33, [1, 7, 100, 92], [200]),
                                                    (1000, [64] * 5, [3, 61, 256])])
def test_step_coder_word_exact_and_round_trip(boa, oracle, ns, enc_tiles, dec_tiles):
    nt = sum(enc_tiles)
    Q, syms = dirichlet_cdfs(np.random.default_rng(ns + nt), nt, ns)
    pitch = boa.capacity_words(nt + 1)
    words, sizes = _encode_tiles(boa, Q, syms, enc_tiles, pitch)
    w = words.cpu().numpy().view(np.uint32).reshape(ns, pitch)
    n = sizes.cpu().numpy().view(np.uint32)
    for s in range(0, ns, max(1, ns // 40)):
        ref = oracle.rc_encode_cdf(Q[:, s], syms[:, s])
        assert n[s] == ref.size and np.array_equal(w[s, :n[s]], ref), s
    assert np.array_equal(_decode_tiles(boa, Q, words, sizes, pitch, dec_tiles), syms)


def test_step_coder_marks_failed_streams(boa, weights):
    """An empty interval stops only that stream; finish writes
    BOA_STREAM_FAILED as its size, the others round-trip, and a model handle
    on the device syncs clean afterwards."""
    m = boa.Model(weights("mamba", 64, 2, 3), "mamba", 64, 2)
    Q, syms = dirichlet_cdfs(np.random.default_rng(12), 90, 5)
    bad = Q.copy()
    s0 = int(syms[50, 3])
    bad[50, 3, s0 + 1] = bad[50, 3, s0]
    pitch = boa.capacity_words(91)
    words, sizes = _encode_tiles(boa, bad, syms, [40, 50], pitch)
    n = sizes.cpu().numpy().view(np.uint32)
    assert n[3] == boa.BOA_STREAM_FAILED and np.all(np.delete(n, 3) != boa.BOA_STREAM_FAILED)
    keep = [0, 1, 2, 4]
    ref_sizes, _ = m.rc_encode_cdf(Q[:, keep], syms[:, keep])
    assert np.array_equal(np.delete(n, 3), ref_sizes)
    # a pitch far too small: every stream overflows and is marked
    _, sizes = _encode_tiles(boa, Q, syms, [90], 3)
    assert np.all(sizes.cpu().numpy().view(np.uint32) == boa.BOA_STREAM_FAILED)
    m.sync()


def test_step_coder_rejects_bad_arguments(boa):
    L = boa.lib()
    one = C.c_void_p(16)
    assert L.boa_rc_encoder_init(None, 4, None) == boa.BOA_E_INVALID
    assert L.boa_rc_encode_cdf_steps(one, one, one, 4, 3, one, 1, None) == boa.BOA_E_INVALID
    assert L.boa_rc_encoder_finish(one, None, 100, one, 4, None) == boa.BOA_E_INVALID
    assert L.boa_rc_decoder_init(one, one, None, one, 4, None) == boa.BOA_E_INVALID
    assert L.boa_rc_decode_cdf_steps(one, one, 0, 3, one, one, one, None) == boa.BOA_E_INVALID
    assert L.boa_rc_state_bytes(0) == 32 and L.boa_rc_state_bytes(1) == 32
