"""The Python codec's batch coder (boa_b200.pycoder, the boa_pyrc_* entry
points) against the reference's own gpu_range_coder extension (golden
streams) and the CPU oracle."""
import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gr(boa):
    from boa_b200 import pycoder
    return pycoder


def _encode(torch, gr, probs, syms, mask, pitch_bytes=None):
    T, N, K = probs.shape
    b = gr.gpu.queue.RangeCoderBatch(N, K, T, pitch_bytes)
    P, S = torch.from_numpy(probs).cuda(), torch.from_numpy(syms).cuda()
    M = torch.from_numpy(mask).cuda()
    for t in range(T):
        b.encode_step(S[t], P[t], mask=M[t])
    b.finalize()
    return b.get_compressed_list(), b.get_sizes_list()


def _decode(torch, gr, probs, mask, streams):
    T, N, K = probs.shape
    b = gr.gpu.queue.RangeCoderBatch(N, K, T)
    b.load_compressed_list(streams)
    b.init_decoder()
    P, M = torch.from_numpy(probs).cuda(), torch.from_numpy(mask).cuda()
    out = torch.zeros(N, dtype=torch.int32, device="cuda")
    got = np.zeros((T, N), np.int32)
    for t in range(T):
        b.decode_step(P[t], out, mask=M[t])
        got[t] = out.cpu().numpy()
    return got


@pytest.mark.parametrize("case", ["k256", "k7", "k1000"])
def test_pycoder_matches_reference_streams(gr, manifest, golden_mod, case):
    import torch
    c = next(x for x in manifest["pyrc"] if x["name"] == case)
    probs, syms, mask = golden_mod.pyrc_inputs(c)
    streams, sizes = _encode(torch, gr, probs, syms, mask)
    z = np.load(f"{GOLDEN}/ref_pyrc.npz")
    assert sizes == z[case + "_sizes"].tolist()
    assert np.array_equal(np.concatenate(streams), z[case + "_words"])
    got = _decode(torch, gr, probs, mask, streams)
    assert np.array_equal(np.where(mask, got, 0), np.where(mask, syms, 0))


@pytest.mark.parametrize("K", [1, 2, 33, 255, 512, 1024])
def test_pycoder_matches_oracle(gr, oracle, K):
    import torch
    rng = np.random.default_rng(K)
    T, N = 50, 37
    probs = rng.dirichlet(np.full(K, 0.2), size=(T, N)).astype(np.float32)
    probs[rng.random((T, N, K)) < 0.05] = 0.0
    syms = rng.integers(0, K, (T, N)).astype(np.int32)
    mask = np.ones((T, N), bool)
    streams, _ = _encode(torch, gr, probs, syms, mask)
    for n in range(N):
        assert np.array_equal(streams[n], oracle.pyrc_encode(probs[:, n], syms[:, n])), n
    got = _decode(torch, gr, probs, mask, streams)
    assert np.array_equal(got, syms)


def test_pycoder_skips_out_of_range_symbols(gr, oracle):
    """encode_kernel returns early for symbols outside [0, K)."""
    import torch
    rng = np.random.default_rng(3)
    T, N, K = 40, 5, 256
    probs = rng.dirichlet(np.full(K, 0.3), size=(T, N)).astype(np.float32)
    syms = rng.integers(0, K, (T, N)).astype(np.int32)
    syms[rng.random((T, N)) < 0.2] = -1
    syms[3, 2] = K
    streams, _ = _encode(torch, gr, probs, syms, np.ones((T, N), bool))
    for n in range(N):
        assert np.array_equal(streams[n], oracle.pyrc_encode(probs[:, n], syms[:, n]))


def test_pycoder_pitch_overflow_is_reported(boa, gr):
    import torch
    rng = np.random.default_rng(4)
    T, N, K = 200, 3, 256
    probs = np.full((T, N, K), 1.0 / K, np.float32)
    syms = rng.integers(0, K, (T, N)).astype(np.int32)
    with pytest.raises(boa.BoaError) as e:
        _encode(torch, gr, probs, syms, np.ones((T, N), bool), pitch_bytes=64)
    assert e.value.code == boa.BOA_E_DEVICE
    b = gr.gpu.queue.RangeCoderBatch(N, K, T, 64)
    with pytest.raises(RuntimeError):
        b.load_compressed_list([np.zeros(17, np.uint32)] * N)
