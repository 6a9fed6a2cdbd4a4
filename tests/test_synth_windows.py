"""The bench's input generators (CPU): particle_windows must cut exactly the
bytes particle_stream produces, whatever the chunk geometry, shard offset and
window; markov_windows must be deterministic and follow its source's
transition tables."""
import numpy as np
import pytest


@pytest.mark.parametrize("chunk,first,n,window", [(16384, 0, 5, 100), (16384, 2040, 20, 16384),
                                                   (3000, 100, 13000, 1000), (1 << 20, 30, 10, 70000),
                                                   (1 << 20, 39, 2, 70000), (7, 0, 5000, 7)])
def test_particle_windows_equal_the_stream(boa, chunk, first, n, window):
    total = 40 * (1 << 20) + 5000  # two generator blocks of 2^20 records and a ragged end
    full = np.frombuffer(boa.synth.particle_stream(total, 7), np.uint8)
    got = boa.synth.particle_windows(total, 7, chunk, first, n, window)
    assert got.shape == (n, min(window, chunk))
    for i in range(n):
        exp = full[(first + i) * chunk:][:min(window, chunk)]
        assert np.array_equal(got[i, :exp.size], exp), i
        assert not got[i, exp.size:].any()


def test_markov_windows_deterministic_and_sparse(boa):
    a = boa.synth.markov_windows(3, 64, 200)
    b = boa.synth.markov_windows(3, 64, 200)
    assert a.shape == (64, 200) and a.dtype == np.uint8
    assert np.array_equal(a, b)
    assert not np.array_equal(a, boa.synth.markov_windows(4, 64, 200))
    # Dirichlet(0.05) rows put most mass on a few symbols: given a context, the
    # next byte is far more predictable than uniform
    ctx = {}
    for row in a:
        for t in range(2, row.size):
            ctx.setdefault((row[t - 2], row[t - 1]), []).append(row[t])
    repeats = [len(v) - len(set(v)) for v in ctx.values() if len(v) > 1]
    assert sum(repeats) > 0
