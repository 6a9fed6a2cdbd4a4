"""Seeded synthetic inputs for the BoaConstrictor hot path.

* ``write_random_weights`` writes a random-initialised model in the exact
  ``.bin`` layout produced by the reference exporter
  (portability_solved_cpp/convert_boa_weights.py:153-241, read back by
  boa_gpu.hpp:990-1029): ``"BOA\\0"`` magic, embedding, per block ln1,
  backbone, ln2, ff, then ``final_norm`` (non-Mamba backbones) and the head.
  Every tensor is drawn in file order from one ``numpy.random.default_rng(seed)``
  stream as N(0, 0.02), except LayerNorm/RMSNorm weights (= 1), LayerNorm
  biases (= 0), ``A_log[c][n] = log(n + 1)`` and ``D = 1``; those fixed tensors
  draw nothing from the stream.
* ``particle_stream`` produces little-endian float32 records of 8 fields
  (pT, eta, phi, mass, charge, three rounded N(0,1) covariates), drawn
  field-major per block of 2**20 records from ``default_rng(seed)``.

The reference ships no dataset for this path; these generators stand in for
the CMS particle data its experiments use.
"""
from __future__ import annotations

import math
import numpy as np

MAGIC_FP32 = b"BOA\x00"
MAGIC_FP16 = b"BOA\x01"

BACKBONES = {"mamba": 0, "mambav1": 0, "lstm": 1, "gru": 2, "mingru": 3}


def mamba_dims(d_model: int):
    """(d_inner, dt_rank, d_state) as MambaConfig computes them (gemm_gpu.hpp:57-65)."""
    return 2 * d_model, (d_model + 15) // 16, 16


def weight_tensors(backbone: str, d_model: int, n_layers: int):
    """Yield (name, shape, kind) in file order; kind in {'rand','one','zero','alog','D'}."""
    d = d_model
    yield ("embedding.weight", (256, d), "rand")
    for i in range(n_layers):
        p = f"blocks.{i}."
        yield (p + "ln1.weight", (d,), "one")
        yield (p + "ln1.bias", (d,), "zero")
        if BACKBONES[backbone] == 0:
            di, r, ds = mamba_dims(d)
            m = p + "mamba."
            yield (m + "in_proj.weight", (2 * di, d), "rand")
            yield (m + "in_proj.bias", (2 * di,), "rand")
            yield (m + "conv1d.weight", (di, 1, 4), "rand")
            yield (m + "conv1d.bias", (di,), "rand")
            yield (m + "x_proj.weight", (r + 2 * ds, di), "rand")
            yield (m + "dt_proj.weight", (di, r), "rand")
            yield (m + "dt_proj.bias", (di,), "rand")
            yield (m + "A_log", (di, ds), "alog")
            yield (m + "D", (di,), "D")
            yield (m + "out_proj.weight", (d, di), "rand")
            yield (m + "out_proj.bias", (d,), "rand")
        elif BACKBONES[backbone] == 3:
            m = p + "mingru."
            yield (m + "linear_z.weight", (d, d), "rand")
            yield (m + "linear_z.bias", (d,), "rand")
            yield (m + "linear_h.weight", (d, d), "rand")
            yield (m + "linear_h.bias", (d,), "rand")
        elif BACKBONES[backbone] in (1, 2):
            # convert_boa_weights.py export_lstm_block / export_gru_block order
            g = (4 if BACKBONES[backbone] == 1 else 3) * d
            m = p + ("lstm." if BACKBONES[backbone] == 1 else "gru.")
            yield (m + "weight_ih_l0", (g, d), "rand")
            yield (m + "bias_ih_l0", (g,), "rand")
            yield (m + "weight_hh_l0", (g, d), "rand")
            yield (m + "bias_hh_l0", (g,), "rand")
        else:
            raise ValueError(f"backbone {backbone!r} is not on this path")
        yield (p + "ln2.weight", (d,), "one")
        yield (p + "ln2.bias", (d,), "zero")
        yield (p + "ff.0.weight", (4 * d, d), "rand")
        yield (p + "ff.0.bias", (4 * d,), "rand")
        yield (p + "ff.2.weight", (d, 4 * d), "rand")
        yield (p + "ff.2.bias", (d,), "rand")
    if BACKBONES[backbone] != 0:
        yield ("final_norm.weight", (d,), "one")
    yield ("head.0.weight", (d, d), "rand")
    yield ("head.0.bias", (d,), "rand")
    yield ("head.2.weight", (256, d), "rand")
    yield ("head.2.bias", (256,), "rand")


def random_weights(backbone: str, d_model: int, n_layers: int, seed: int, std: float = 0.02):
    """Return an ordered list of (name, float32 array) for a random-init model."""
    rng = np.random.default_rng(seed)
    out = []
    for name, shape, kind in weight_tensors(backbone, d_model, n_layers):
        if kind == "rand":
            a = rng.normal(0.0, std, size=shape)
        elif kind == "one":
            a = np.ones(shape)
        elif kind == "zero":
            a = np.zeros(shape)
        elif kind == "alog":
            a = np.broadcast_to(np.log(np.arange(1, shape[1] + 1, dtype=np.float64)), shape)
        elif kind == "D":
            a = np.ones(shape)
        else:  # pragma: no cover
            raise AssertionError(kind)
        out.append((name, np.ascontiguousarray(a, dtype=np.float32)))
    return out


def write_weights(path: str, tensors, fp16: bool = False) -> int:
    """Write (name, array) pairs in order with the BOA header; returns bytes written."""
    with open(path, "wb") as f:
        f.write(MAGIC_FP16 if fp16 else MAGIC_FP32)
        for _, a in tensors:
            f.write((a.astype(np.float16) if fp16 else a.astype(np.float32)).tobytes())
        return f.tell()


def write_random_weights(path: str, backbone: str = "mamba", d_model: int = 256,
                         n_layers: int = 8, seed: int = 0, fp16: bool = False, std: float = 0.02) -> int:
    return write_weights(path, random_weights(backbone, d_model, n_layers, seed, std=std), fp16=fp16)


_BLOCK_RECORDS = 1 << 20


def _particle_blocks(n_bytes: int, seed: int):
    """Yield the stream's blocks of 2**20 records as little-endian f4 [nb, 8]."""
    rng = np.random.default_rng(seed)
    n_rec = (n_bytes + 31) // 32
    for start in range(0, n_rec, _BLOCK_RECORDS):
        nb = min(_BLOCK_RECORDS, n_rec - start)
        pt = rng.exponential(30.0, nb)
        eta = rng.uniform(-2.5, 2.5, nb)
        phi = rng.uniform(-math.pi, math.pi, nb)
        mass = np.abs(rng.normal(0.14, 0.05, nb))
        charge = rng.integers(0, 2, nb) * 2 - 1
        cov = np.round(rng.normal(0.0, 1.0, (3, nb)), 3)
        rec = np.stack([pt, eta, phi, mass, charge, cov[0], cov[1], cov[2]], axis=1)
        yield rec.astype("<f4")


def particle_stream(n_bytes: int, seed: int) -> bytes:
    """Little-endian float32 particle records (8 fields, 32 bytes each)."""
    blocks = list(_particle_blocks(n_bytes, seed))
    data = np.concatenate(blocks).tobytes() if blocks else b""
    return data[:n_bytes]


def particle_windows(total_bytes: int, seed: int, chunk_len: int, first_chunk: int, n_chunks: int,
                     window: int) -> np.ndarray:
    """The first ``window`` bytes of chunks [first_chunk, first_chunk + n_chunks)
    of ``particle_stream(total_bytes, seed)`` cut into ``chunk_len``-byte chunks, as a
    u8 array [n_chunks, window], without holding the whole stream: the
    generator walks the stream block by block (the same draws as
    ``particle_stream``) and keeps only the windows.  Row i equals
    ``particle_stream(...)[(first_chunk + i) * chunk_len:][:window]`` (zero-padded past the
    stream's end)."""
    window = min(window, chunk_len)
    out = np.zeros((n_chunks, window), np.uint8)
    c = 0                      # next chunk (relative) whose window is not complete
    pos = 0                    # stream offset of the start of `carry`
    carry = np.zeros(0, np.uint8)
    for blk in _particle_blocks(total_bytes, seed):  # block sizes depend on the total
        buf = np.concatenate([carry, blk.reshape(-1).view(np.uint8)])
        top = pos + buf.size
        while c < n_chunks:
            s = (first_chunk + c) * chunk_len
            need = max(0, min(window, total_bytes - s))  # the stream's last chunk may be short
            if s + need > top:
                break
            out[c, :need] = buf[s - pos: s - pos + need]
            c += 1
        if c >= n_chunks:
            break
        keep = min((first_chunk + c) * chunk_len - pos, buf.size)  # drop what no later window needs
        carry = buf[keep:]
        pos += keep
    return out


def exact_logit_weights(d_model: int, n_layers: int, seed: int, support, low: float = -1000.0):
    """Random-init Mamba model whose logits are exactly the head bias.

    ``head.2.weight`` is zero and ``head.2.bias`` is 0 on ``support`` and
    ``low`` elsewhere, so every position's logits are exact constants and the
    softmax exponentials are exactly 1 or 0 on any IEEE machine.  The integer
    CDF is then identical on CPU and GPU, which pins the quantiser, the range
    coder and the container bit for bit against the reference binary.
    """
    ts = random_weights("mamba", d_model, n_layers, seed)
    out = []
    for name, a in ts:
        if name == "head.2.weight":
            a = np.zeros_like(a)
        elif name == "head.2.bias":
            a = np.full_like(a, low)
            a[np.asarray(list(support), dtype=np.int64)] = 0.0
        out.append((name, a))
    return out


def markov_stream(n_bytes: int, seed: int, alpha: float = 0.05) -> bytes:
    """Order-2 Markov byte source: each of the 65536 contexts
    (previous two bytes) has its own next-byte distribution drawn from
    Dirichlet(alpha * 1_256) with ``numpy.random.default_rng(seed)``; the
    stream starts from context (0, 0) and draws each byte by inverse CDF from
    uniforms of the same generator (drawn after the tables)."""
    rng = np.random.default_rng(seed)
    g = rng.gamma(alpha, 1.0, size=(65536, 256))
    g /= g.sum(axis=1, keepdims=True)
    cdf = np.cumsum(g, axis=1)
    u = rng.random(n_bytes)
    out = np.empty(n_bytes, np.uint8)
    a = b = 0
    for i in range(n_bytes):
        row = cdf[(a << 8) | b]
        s = int(np.searchsorted(row, u[i] * row[-1], side="right"))
        s = 255 if s > 255 else s
        out[i] = s
        a, b = b, s
    return out.tobytes()


def markov_windows(seed: int, n_chunks: int, window: int, alpha: float = 0.05) -> np.ndarray:
    """configs[3]-scale input from the same order-2 Markov source as
    ``markov_stream``: the context tables are drawn first from
    ``default_rng(seed)`` exactly as there, then every chunk is its own run of
    the chain from context (0, 0), all chunks advanced together one position
    at a time (uniforms drawn [window, n_chunks]).  Returns u8 [n_chunks,
    window].  A single 256 MiB sequential stream would take hours in Python;
    the per-chunk runs have the same transition law."""
    rng = np.random.default_rng(seed)
    g = rng.gamma(alpha, 1.0, size=(65536, 256))
    g /= g.sum(axis=1, keepdims=True)
    cdf = np.cumsum(g, axis=1)
    # every row offset by its context index, so one sorted array serves all
    # rows: a draw in context r searches r + u * cdf[r][-1]
    ctx = np.arange(65536, dtype=np.float64)
    flat = (cdf + ctx[:, None]).reshape(-1)
    last = cdf[:, -1]
    out = np.empty((n_chunks, window), np.uint8)
    a = np.zeros(n_chunks, np.int64)
    b = np.zeros(n_chunks, np.int64)
    for t in range(window):
        u = rng.random(n_chunks)
        r = (a << 8) | b
        s = np.searchsorted(flat, r + u * last[r], side="right") - r * 256
        s = np.clip(s, 0, 255)
        out[:, t] = s
        a, b = b, s
    return out
