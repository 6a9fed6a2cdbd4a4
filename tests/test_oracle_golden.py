"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference binaries).  CPU only."""
import numpy as np
import pytest

from conftest import GOLDEN, dirichlet_cdfs


LOGIT_CFGS = ["d64L2", "d256L8", "d512L16", "mingru_d64L2", "lstm_d64L2", "gru_d64L2"]


def test_oracle_cdf_strictly_increasing_on_near_certain_rows(oracle):
    """The oracle's quantiser on the rows that give the reference's rule an
    empty interval: strictly increasing, total 2^24."""
    z = np.load(f"{GOLDEN}/cdf_edge_rows.npz")
    Q = oracle.cdf_rows(z["logits"]).astype(np.int64)
    assert (np.diff(Q, axis=1) > 0).all() and (Q[:, 256] == 1 << 24).all()


@pytest.mark.parametrize("name", ["mamba_d64L2", "mamba_d80L1", "mamba_d128L1", "mingru_d160L1"])
@pytest.mark.parametrize("mode", [0, 1])
def test_oracle_logits_match_reference_trained(oracle, boa, manifest, name, mode):
    """The CPU restatement on weights converted from the reference's trained
    checkpoints (non-uniform predictions, d_model 64 / 80 / 160) against the
    reference's own logits on the same bytes."""
    c = next(x for x in manifest["trained"] if x["name"] == name)
    z = np.load(f"{GOLDEN}/ref_logits_trained_{name}.npz")
    m = oracle.OracleModel(f"{GOLDEN}/trained_{name}.bin", boa.BACKBONES[c["backbone"]], c["d_model"],
                           c["n_layers"])
    ref = z["chunk" if mode == 0 else "step"]
    assert np.abs(m.logits(z["tokens"], mode) - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("cfg", LOGIT_CFGS)
@pytest.mark.parametrize("mode", [0, 1])
def test_oracle_logits_match_reference_gpu(oracle, boa, manifest, wdir, cfg, mode):
    c = next(x for x in manifest["logits"] if x["name"] == cfg)
    z = np.load(f"{GOLDEN}/ref_logits_{cfg}.npz")
    p = str(wdir / f"g_{cfg}.bin")
    bb = c.get("backbone", "mamba")
    boa.synth.write_random_weights(p, bb, c["d_model"], c["n_layers"], c["seed"], std=c.get("std", 0.02))
    m = oracle.OracleModel(p, boa.BACKBONES[bb], c["d_model"], c["n_layers"])
    lg = m.logits(z["tokens"], mode)
    ref = z["chunk" if mode == 0 else "step"]
    # the oracle uses libm exp/log, the reference CUDA's: agree to ~1e-6
    assert np.abs(lg - ref).max() <= 1e-5 * np.abs(ref).max()


def test_reference_chunk_and_step_logits_agree(manifest):
    for c in manifest["logits"]:
        z = np.load(f"{GOLDEN}/ref_logits_{c['name']}.npz")
        assert np.array_equal(z["chunk"], z["step"])


def test_oracle_reproduces_reference_container_bit_exact(oracle, boa, boa2, manifest, golden_mod, wdir):
    E = manifest["exact"]
    p = str(wdir / "exact.bin")
    boa.synth.write_weights(p, boa.synth.exact_logit_weights(E["d_model"], E["n_layers"], E["seed"], E["support"]))
    data = golden_mod.exact_input(E)
    m = oracle.OracleModel(p, 0, E["d_model"], E["n_layers"])
    fb, streams = m.compress(data, E["chunk"])
    blob = boa2.build(len(data), E["chunk"], fb, [s.tobytes() for s in streams])
    ref = open(f"{GOLDEN}/ref_exact.boa", "rb").read()
    assert blob == ref
    parsed = boa2.parse(ref)
    out = m.decompress(parsed["first_bytes"], [np.frombuffer(s, "<u4") for s in parsed["streams"]],
                       parsed["total_size"], parsed["chunk_len"])
    assert out == data


def test_reference_random_container_parses(boa2, manifest):
    blob = open(f"{GOLDEN}/ref_rand_d256L8.boa", "rb").read()
    p = boa2.parse(blob)
    R = manifest["rand"]
    assert p["total_size"] == R["n_bytes"] and p["chunk_len"] == R["chunk"]
    assert p["n_chunks"] == R["n_bytes"] // R["chunk"] and p["index_version"] == 2
    assert all(len(s) % 4 == 0 for s in p["streams"])


def test_oracle_coder_roundtrip_dirichlet(oracle):
    rng = np.random.default_rng(0)
    Q, syms = dirichlet_cdfs(rng, 3000, 1)
    w = oracle.rc_encode_cdf(Q[:, 0], syms[:, 0])
    assert np.array_equal(oracle.rc_decode_cdf(Q[:, 0], w, 3000), syms[:, 0])


def test_oracle_coder_frequency_one_symbols(oracle):
    # every symbol at frequency 1: longest renormalisation and carry runs
    Q = np.zeros((400, 257), np.uint32)
    Q[:, :256] = np.arange(256, dtype=np.uint32)
    Q[:, 256] = 1 << 24
    Q[:, 255] = 255
    Q[:, 1:256] += (1 << 24) - 256  # symbol 0 takes almost everything
    syms = np.random.default_rng(1).integers(1, 256, 400).astype(np.uint8)
    w = oracle.rc_encode_cdf(Q, syms)
    assert np.array_equal(oracle.rc_decode_cdf(Q, w, 400), syms)


def test_oracle_empty_stream_is_zero_words(oracle):
    Q = np.zeros((0, 257), np.uint32)
    assert oracle.rc_encode_cdf(Q, np.zeros(0, np.uint8)).size == 0


def test_oracle_codec_roundtrip_ragged(oracle, weights):
    m = oracle.OracleModel(weights("mamba", 64, 2, 3), 0, 64, 2)
    data = bytes(np.random.default_rng(2).integers(0, 256, 2301, dtype=np.uint8))
    fb, st = m.compress(data, 500)
    assert [len(s) for s in st][-1] > 0
    assert m.decompress(fb, st, len(data), 500) == data
    fb, st = m.compress(data[:2001], 500)  # last chunk of one byte -> zero words
    assert len(st[-1]) == 0
    assert m.decompress(fb, st, 2001, 500) == data[:2001]


def test_oracle_mingru_roundtrip(oracle, weights):
    m = oracle.OracleModel(weights("mingru", 64, 2, 2), 3, 64, 2)
    data = bytes(np.random.default_rng(4).integers(0, 256, 700, dtype=np.uint8))
    fb, st = m.compress(data, 300)
    assert m.decompress(fb, st, len(data), 300) == data
    a = m.logits(np.frombuffer(data[:64], np.uint8).reshape(2, 32), 0)
    b = m.logits(np.frombuffer(data[:64], np.uint8).reshape(2, 32), 1)
    assert np.array_equal(a, b)


def test_oracle_warm_start_roundtrip(oracle, boa, weights):
    m = oracle.OracleModel(weights("mamba", 64, 2, 3), 0, 64, 2)
    data = boa.synth.particle_stream(11 * 300 + 17, 7)
    fb, st = m.compress(data, 300, warm=4)
    assert m.decompress(fb, st, len(data), 300, warm=4) == data
    fb1, st1 = m.compress(data, 300, warm=12)  # one chunk per lane == plain
    fb0, st0 = m.compress(data, 300)
    assert all(np.array_equal(a, b) for a, b in zip(st0, st1))


@pytest.mark.parametrize("backbone", ["lstm", "gru"])
def test_oracle_rnn_roundtrip(oracle, boa, weights, backbone):
    m = oracle.OracleModel(weights(backbone, 64, 2, 4, 0.1), boa.BACKBONES[backbone], 64, 2)
    data = bytes(np.random.default_rng(6).integers(0, 256, 700, dtype=np.uint8))
    fb, st = m.compress(data, 300)
    assert m.decompress(fb, st, len(data), 300) == data
    tok = np.frombuffer(data[:64], np.uint8).reshape(2, 32)
    assert np.array_equal(m.logits(tok, 0), m.logits(tok, 1))


@pytest.mark.parametrize("case", ["k256", "k7", "k1000"])
def test_oracle_pyrc_matches_reference_streams(oracle, manifest, golden_mod, case):
    """The Python codec's coder (gpu_range_coder.py): the oracle's restatement
    of build_cdf_fast + the range coder reproduces the reference extension's
    streams word for word, and the reference decoded its own streams."""
    c = next(x for x in manifest["pyrc"] if x["name"] == case)
    res = manifest["pyrc_result"][case]
    assert res["ref_decoded"]
    probs, syms, mask = golden_mod.pyrc_inputs(c)
    import hashlib
    assert hashlib.sha256(probs.tobytes()).hexdigest() == res["probs_sha"]
    z = np.load(f"{GOLDEN}/ref_pyrc.npz")
    sizes, words = z[case + "_sizes"], z[case + "_words"]
    o = 0
    for n in range(c["N"]):
        act = mask[:, n]
        w = oracle.pyrc_encode(probs[act, n], syms[act, n])
        assert np.array_equal(w, words[o:o + sizes[n]]), n
        assert np.array_equal(oracle.pyrc_decode(probs[act, n], w), syms[act, n])
        o += int(sizes[n])
    assert o == words.size


def test_python_dialect_container(boa, boa2):
    """A container in the Python BoaFile dialect (16-byte blake2s fingerprint,
    flags 0) is written byte-identically to the restatement and parsed back."""
    import hashlib
    fp = hashlib.blake2s(b"BoaBytePredictor", digest_size=16).digest()
    assert boa.python_fingerprint() == fp
    rng = np.random.default_rng(9)
    sizes = [5, 0, 17, 3]
    words = rng.integers(0, 2**32, sum(sizes), dtype=np.uint64).astype(np.uint32)
    fb = [1, 2, 3, 4]
    streams, o = [], 0
    for s in sizes:
        streams.append(words[o:o + s].tobytes())
        o += s
    total = 3 * 100 + 41
    ours = boa.boa2_build(total, 100, fb, sizes, words, fingerprint=fp)
    assert ours == boa2.build(total, 100, fb, streams, fingerprint=fp)
    info = boa.boa2_parse(ours)
    assert info["fingerprint"] == fp and info["flags"] == 0 and info["interleave_batch"] == 0
    assert [bytes(s) for s in info["streams"]] == streams


def _peaked_logits(rng, rows):
    """Logits rows like the trained models' near-certain predictions: one byte
    20..60 nats above the others at a random position, the rest spread over
    ~80 nats (some probabilities underflow to zero)."""
    lg = rng.normal(0.0, 1.0, (rows, 256)).astype(np.float32) * rng.uniform(1, 25, (rows, 1)).astype(np.float32)
    top = rng.integers(0, 256, rows)
    lg[np.arange(rows), top] = lg.max(1) + rng.uniform(20, 60, rows).astype(np.float32)
    return lg


def test_oracle_cdf_strictly_increasing_on_peaked_rows(oracle):
    """Property behind the CDF repair: over many near-certain rows, every Q is
    strictly increasing with Q_256 = 2^24, so every symbol stays decodable.
    (Without the running maximum, about 2 % of these rows -- 370 of 20000 --
    leave some symbol an empty interval.)"""
    lg = _peaked_logits(np.random.default_rng(5), 20000)
    Q = oracle.cdf_rows(lg).astype(np.int64)
    assert (np.diff(Q, axis=1) > 0).all() and (Q[:, 256] == 1 << 24).all()


@pytest.mark.parametrize("name", ["mamba_d64L2", "mamba_d80L1", "mamba_d128L1", "mingru_d160L1"])
def test_oracle_bits_per_byte_trained_vs_reference(oracle, boa, boa2, manifest, name):
    """The CPU restatement's container for the trained models on the same
    64 KiB of particle records: byte-exact round trip, and within 0.5 % of the
    size of the reference CLI's container."""
    c = next(x for x in manifest["trained"] if x["name"] == name)
    td = manifest["trained_data"]
    data = boa.synth.particle_stream(td["n_bytes"], td["data_seed"])
    m = oracle.OracleModel(f"{GOLDEN}/trained_{name}.bin", boa.BACKBONES[c["backbone"]], c["d_model"],
                           c["n_layers"])
    fb, streams = m.compress(data, td["chunk"])
    assert m.decompress(fb, streams, len(data), td["chunk"]) == data
    blob = boa2.build(len(data), td["chunk"], fb, [s.tobytes() for s in streams])
    ref = manifest["trained_result"][name]["boa_bytes"]
    assert abs(len(blob) - ref) <= 0.005 * ref
