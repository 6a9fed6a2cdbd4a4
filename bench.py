"""Benchmark: BoaConstrictor chunk-parallel compress + decompress on B200.

Workload: the 256-d / 8-layer Mamba predictor,
random-init weights (seed 0), over a 256 MiB stream of seeded synthetic
float32 particle records (seed 1 + rank) split into 16,384 chunks of 16 KiB,
all chunks in one batch.  One step = one 64-position compress tile plus the 64
decode steps of the same positions, over every chunk: the K timed steps are
one compress call over the chunks' first 64K + 1 bytes and one decompress call
(256 steps are the whole chunks).  The round trip is verified after timing; a
mismatch exits with status 3.

  python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]
  python bench.py --workload coder     # configs[1]: the integer range coder alone
  python bench.py --workload configs3  # minGRU d256 L8 on the order-2 Markov source
  python bench.py --workload configs4  # Mamba d512 L16, 262,144 chunks split over the GPUs
  python bench.py --workload cms       # the reference's cms_experiment model (mambav1
                                       # d64 L2, its trained weights) on 16,384 chunks
                                       # of 4 KiB: the configuration of the reference's
                                       # published MB/s, so vs_baseline is set
  python bench.py --workload pyrc      # the Python codec's batch coder

Under torchrun each rank drives its own GPU.  configs[2]: every rank codes its
own 256 MiB stream (weak scaling); configs[4]: the workload's chunks are split
over the ranks (strong scaling).  Chunks are independent, so no collective
touches the data path; the only cross-rank traffic is the barrier and the
max-reduction of the timings.

value  = MB/s (2^20 B) of input round-tripped per second, whole job, inputs
         resident in HBM, device time (CUDA events) max over ranks.
e2e    = the same through the host-buffer C-ABI calls (boa_compress_chunks /
         boa_decompress_chunks) from pinned host memory, copies included.
--impl reference times the CPU restatement of the reference path on this
host's cores (the reference ships no CPU C++ path; its CUDA binary was timed
separately through its own CLI).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MiB = float(1 << 20)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--chunks", type=int, default=None,
                    help="chunks of the whole workload (weak scaling: per GPU); default from --workload")
    ap.add_argument("--chunk-len", type=int, default=None, help="bytes per chunk; default from --workload")
    ap.add_argument("--d-model", type=int, default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--e2e-steps", type=int, default=1, help="0 skips the host-buffer e2e measurement")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="roundtrip", choices=["roundtrip", "cms", "configs3", "configs4", "coder", "pyrc"],
                    help="roundtrip: configs[2] compress+decompress (the headline); cms: the same round trip "
                         "with the reference's cms_experiment model (trained mambav1 d64 L2) on 4 KiB chunks, "
                         "the configuration of the reference's published MB/s; configs3: minGRU d256 L8 on the "
                         "order-2 Markov source; configs4: Mamba d512 L16, 262,144 chunks sharded over the GPUs "
                         "(strong scaling); coder: configs[1], the integer range coder alone on Dirichlet(0.1) "
                         "CDFs; pyrc: the Python codec's batch range coder against the reference's own extension")
    ap.add_argument("--weights", default=None, help="weight file (.bin) instead of random-init weights")
    ap.add_argument("--streams", type=int, default=65536, help="pyrc: streams per batch")
    ap.add_argument("--positions", type=int, default=64, help="pyrc: coded positions per step")
    ap.add_argument("--coder-tile", type=int, default=16, help="coder: positions of every stream per step")
    return ap.parse_args()


def dist_info():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# --------------------------------------------------------------------------- roofline
def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(j["bf16_tflops_sustained"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def algorithmic_per_launch(cls, B, T, d, L):
    """Algorithmic work of one launch of kernel class `cls` over B chunks x T
    positions (M = B*T rows): ('hbm', bytes) or ('tensor', flops).  FLOPs
    count the three bf16 products of the split-precision GEMM."""
    M, di = B * T, 2 * d
    xp = ((d + 15) // 16 + 32 + 15) // 16 * 16
    gem = {"in_proj": (d, 4 * d), "x_proj": (di, xp), "out_proj_ln": (di, d), "ff2_res_ln": (4 * d, d),
           "head1": (d, d), "head2_coder": (d, 256)}
    if cls == "ffn":  # fused feed-forward (both GEMMs) for d 64 / 128 / 256, its first GEMM otherwise
        return "tensor", 2.0 * 3 * M * (4 * d * d) * (2 if d in (64, 128, 256) else 1)
    if cls in gem:
        K, N = gem[cls]
        return "tensor", 2.0 * 3 * M * N * K
    if cls == "scan":
        # state r+w (16 floats/channel) + u, z in + bf16 hi/lo y out (+ delta rows)
        return "hbm", B * di * 16 * 4 * 2 + M * di * (4 + 4 + 4) + M * xp * 4
    if cls == "conv":
        return "hbm", B * di * 3 * 4 * 2 + M * di * (4 + 4 + 4)
    if cls == "embed_ln":
        return "hbm", M * (d * 4 + d * 4)
    if cls == "encode_tile":
        return "hbm", M * 8 + M * 1
    return None, 0.0


def step_roofline(d, L, B, T, hbm_gbs, tf_sust):
    """Roofline of one compress tile (B chunks x T positions) and one decode
    step (B chunks x 1 position): the slower of the algorithmic GEMM FLOPs at
    the sustained bf16 tensor peak and the weight + recurrent-state bytes at
    the HBM copy peak.  FLOPs are the fp32 model's (the three bf16 products of
    the split-precision GEMMs are not counted); state is conv [3][di] + ssm
    [16][di] fp32 per layer, read and written once per tile or step."""
    di = 2 * d
    r = (d + 15) // 16
    xp = ((r + 32 + 15) // 16) * 16
    gemm_kn = [(d, 2 * di), (di, xp), (r, di), (di, d), (d, 4 * d), (4 * d, d)]
    flops_per_byte = L * sum(2 * k * n for k, n in gemm_kn) + 2 * (d * d + d * 256)
    weight_bytes = 4 * (L * sum(k * n for k, n in gemm_kn) + d * d + d * 256 + 256 * d)
    state_per_chunk = L * (16 + 3) * di * 4

    def one(tokens_per_chunk):
        byts = 2 * state_per_chunk * B + weight_bytes + 2 * B * tokens_per_chunk
        t_mem = byts / (hbm_gbs * 1e9)
        t_flop = flops_per_byte * B * tokens_per_chunk / (tf_sust * 1e12)
        return max(t_mem, t_flop), ("hbm" if t_mem >= t_flop else "tensor")

    tc, bc = one(T)
    td, bd = one(1)
    return {"compress_bound_MBps": B * T / MiB / tc, "compress_bound": bc,
            "decompress_bound_MBps": B / MiB / td, "decompress_bound": bd,
            "flops_per_byte": flops_per_byte, "state_bytes_per_chunk": state_per_chunk,
            "weight_bytes": weight_bytes}


# DRAM bytes (read + write) of one launch from `ncu --set full` (the capture
# summarised in profiles/ncu_configs2_step_kernels.md), per chunk of the batch
# (the kernel's traffic scales with the number of chunks): decompress-step scan.
NCU_TRAFFIC_PER_CHUNK = {("scan", "decode"): (607.283e6 + 512.869e6) / 16384}


# --------------------------------------------------------------------------- clocks
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        under = [s for s in sm if s > 0.5 * mx] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(under), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- CPU legs
def cpu_sample(weights, d, L, chunk_len, seed, budget_s, threads, backbone="mamba", kind="particle"):
    """Round trip of the CPU restatement on `threads` chunks, each a prefix of
    one of the workload's chunks, sized so one pass takes about budget_s seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    boa = __import__("__graft_entry__").load_package()
    m = O.OracleModel(weights, boa.BACKBONES[backbone], d, L)
    if kind == "markov":
        data = boa.synth.markov_windows(seed, threads, chunk_len).tobytes()
    else:
        data = boa.synth.particle_stream(threads * chunk_len, seed)
    # calibrate: 64-byte prefixes
    probe = 64
    sub = b"".join(data[i * chunk_len: i * chunk_len + probe] for i in range(threads))
    t = time.perf_counter()
    fb, st = m.compress(sub, probe, threads=threads)
    m.decompress(fb, st, len(sub), probe, threads=threads)
    rate = len(sub) / (time.perf_counter() - t)
    plen = int(max(probe, min(chunk_len, rate * budget_s / threads)))
    sub = b"".join(data[i * chunk_len: i * chunk_len + plen] for i in range(threads))
    t = time.perf_counter()
    fb, st = m.compress(sub, plen, threads=threads)
    out = m.decompress(fb, st, len(sub), plen, threads=threads)
    dt = time.perf_counter() - t
    assert out == sub
    return len(sub) / MiB / dt, f"{threads} chunks x {plen}-byte prefixes of the workload's chunks, round trip", dt


# The reference's published throughput (portability_solved_cpp/README.md:122-126): the cms_experiment
# model (experiments/cms_experiment/cms_experiment.yaml: mambav1, d_model 64, 2 layers) on an RTX 5090.
CMS_PUBLISHED = {"compress_MBps": 7.0, "decompress_MBps": 5.0, "hardware": "RTX 5090",
                 "source": "portability_solved_cpp/README.md:122-126"}
CMS_WEIGHTS = os.path.join(ROOT, "tests", "golden", "trained_mamba_d64L2.bin")


def apply_workload(a):
    """Fill the model geometry from the workload table unless given.  --workload cms: the
    cms_experiment model with its trained weights (converted from the reference's checkpoint by
    tests/golden/convert_trained.py), 4 KiB chunks."""
    if a.workload in WORKLOADS:
        _, d, L, _, chunks, S, _, _, _ = WORKLOADS[a.workload]
        a.d_model = a.d_model or d
        a.layers = a.layers or L
        a.chunks = a.chunks or chunks
        a.chunk_len = a.chunk_len or S
    if a.workload == "cms":
        a.weights = a.weights or CMS_WEIGHTS
    return a


def workload_name(a, C, S):
    """The workload string both arms report for this geometry (C = the whole workload's chunks)."""
    n = C * S
    if a.workload == "cms":
        return (f"cms_experiment model (mambav1 d64 L2, trained weights), {C} chunks x {S} B = "
                f"{n / MiB:g} MiB per GPU")
    bb = WORKLOADS.get(a.workload, WORKLOADS["roundtrip"])[0]
    tags = {("roundtrip", 256, 8, 16384, 16384): "configs[2]: ", ("configs3", 256, 8, 16384, 16384): "configs[3]: ",
            ("configs4", 512, 16, 262144, 16384): "configs[4]: "}
    tag = tags.get((a.workload, a.d_model, a.layers, C, S), "")
    per = "sharded over the GPUs" if a.workload == "configs4" else "per GPU"
    return f"{tag}{bb} d{a.d_model} L{a.layers}, {C} chunks x {S} B = {n / MiB:g} MiB {per}"


def published_baseline(a):
    """value / published round trip for the cms workload (null otherwise: no published number exists
    for configs[2])."""
    if a.workload != "cms":
        return None, None
    rt = 1.0 / (1.0 / CMS_PUBLISHED["compress_MBps"] + 1.0 / CMS_PUBLISHED["decompress_MBps"])
    return rt, dict(CMS_PUBLISHED, roundtrip_MBps=rt)


def run_reference_coder(a):
    """configs[1] reference arm: the CPU coder (the oracle's restatement of the
    reference's integer range coder) on all host threads, each thread coding
    its own streams of Dirichlet(0.1) CDFs (numpy, seeded); a step is a bounded
    sample of streams x the bench's positions."""
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build()
    threads = os.cpu_count() or 1
    P = 16384          # symbols per stream per step
    per_thread = 4     # streams per host thread
    rng = np.random.default_rng(11)

    def gen(n_streams, n_steps):
        p = rng.dirichlet(np.full(256, 0.1), size=(n_steps, n_streams))
        c = np.concatenate([np.zeros(p.shape[:2] + (1,)), np.cumsum(p, -1)[..., :-1]], -1)
        Q = np.empty(p.shape[:2] + (257,), np.uint32)
        Q[..., :256] = (c * float((1 << 24) - 256)).astype(np.uint32) + np.arange(256, dtype=np.uint32)
        Q[..., 256] = 1 << 24
        u = rng.random(p.shape[:2] + (1,))
        return Q, np.minimum((np.cumsum(p, -1) < u).sum(-1), 255).astype(np.uint8)

    def code(args):
        Q, S = args
        w = O.rc_encode_cdf(Q, S)
        return np.array_equal(O.rc_decode_cdf(Q, w, S.size), S)

    Q, S = gen(threads * per_thread, P)
    jobs = [(np.ascontiguousarray(Q[:, j]), np.ascontiguousarray(S[:, j])) for j in range(threads * per_thread)]
    vals, secs = [], []
    with ThreadPoolExecutor(threads) as ex:
        for i in range(a.warmup + a.steps):
            t0 = time.perf_counter()
            ok = all(ex.map(code, jobs))
            dt = time.perf_counter() - t0
            if i >= a.warmup:
                vals.append(2 * len(jobs) * P / dt)
                secs.append(dt)
    v = statistics.median(vals)
    line = {"metric": "range-coder symbols/s (encode + decode)", "value": v, "unit": "symbols/s", "n_gpus": 1,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": statistics.median(secs) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32 CDF, u64 coder",
            "data": "synthetic: Dirichlet(0.1) CDFs (numpy, seed 11)", "impl": "reference",
            "config": {"workload": f"configs[1]: {a.streams} streams x 65536 symbols, range coder alone",
                       "step": f"{len(jobs)} streams x {P} symbols, encode + decode, {threads} host threads"},
            "cpu_baseline": {"value": v, "unit": "symbols/s", "cores": threads, "kind": "port",
                             "sample": f"{len(jobs)} streams x {P} symbols per step", "round_trip_ok": bool(ok)},
            "e2e": {"value": v, "unit": "symbols/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference(a):
    ws, rank, _ = dist_info()
    if rank != 0:
        return
    if a.workload == "coder":
        return run_reference_coder(a)
    sys.path.insert(0, ROOT)
    boa = __import__("__graft_entry__").load_package()
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as td:
        w = os.path.join(td, "w.bin")
        backbone, _, _, wseed, _, _, kind, dseed, _ = WORKLOADS[a.workload]
        if a.weights:
            w = a.weights
        else:
            boa.synth.write_random_weights(w, backbone, a.d_model, a.layers, wseed)
        for _ in range(a.warmup):
            cpu_sample(w, a.d_model, a.layers, a.chunk_len, dseed, 0.2, threads, backbone, kind)
        vals, secs = [], []
        per_step = min(a.cpu_seconds, 60.0 / max(1, a.steps))  # the whole run stays near a minute
        for _ in range(a.steps):
            v, sample, dt = cpu_sample(w, a.d_model, a.layers, a.chunk_len, dseed, per_step, threads,
                                       backbone, kind)
            vals.append(v)
            secs.append(dt)
    v = statistics.median(vals)
    line = {"metric": "compress+decompress round-trip MB/s", "value": v, "unit": "MB/s", "n_gpus": ws,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": statistics.median(secs) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": workload_name(a, a.chunks, a.chunk_len),
                       "step": "a bounded sample of the workload per step (cpu_baseline.sample); ms_per_step is its "
                               "duration"},
            "cpu_baseline": {"value": v, "unit": "MB/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "MB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- pyrc leg
def load_ref_pyrc():
    """The reference's gpu_range_coder extension, built by oracle/build_ref.sh
    (None when it was not built)."""
    import glob
    import importlib.machinery
    import importlib.util
    so = glob.glob(os.path.join(ROOT, "oracle", "_ref", "_gpu_range_cuda_ext*.so"))
    if not so:
        return None
    loader = importlib.machinery.ExtensionFileLoader("_gpu_range_cuda_ext", so[0])
    mod = importlib.util.module_from_spec(importlib.util.spec_from_loader("_gpu_range_cuda_ext", loader))
    loader.exec_module(mod)
    return mod


def run_pyrc(a):
    """One step = encode `positions` symbols in each of `streams` streams from
    fp32 probability rows already in HBM (plus finalize), then decode them
    again.  Rows are softmax(3 * N(0,1)) over K = 256, one distinct 64 MiB
    buffer per position (4 GiB in all, far above L2)."""
    import torch
    boa = __import__("__graft_entry__").load_package()
    from boa_b200 import pycoder
    hbm_peak, _, _, peak_kind = load_peaks()
    N, T, K = a.streams, a.positions, 256
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    probs = torch.empty((T, N, K), dtype=torch.float32, device=dev)
    syms = torch.empty((T, N), dtype=torch.int32, device=dev)
    for t in range(T):
        probs[t] = torch.softmax(3.0 * torch.randn((N, K), device=dev, generator=g), dim=-1)
        syms[t] = torch.multinomial(probs[t], 1, generator=g)[:, 0].to(torch.int32)
    out = torch.empty(N, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    clocks = Clocks(0)

    def ours():
        # each loop is captured in a CUDA graph, so the timed region holds the
        # kernels alone (the per-call Python overhead of the class is larger
        # than one launch); capture and host copies stay outside it
        enc = pycoder.gpu.queue.RangeCoderBatch(N, K, T)
        g_enc = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_enc, stream=stream):
            for t in range(T):
                enc.encode_step(syms[t], probs[t])
            enc.finalize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize()
        ev[0].record(stream)
        g_enc.replay()
        ev[1].record(stream)
        streams = enc.get_compressed_list()
        dec = pycoder.gpu.queue.RangeCoderBatch(N, K, T)
        dec.load_compressed_list(streams)
        got = torch.empty((T, N), dtype=torch.int32, device=dev)
        g_dec = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_dec, stream=stream):
            dec.init_decoder()
            for t in range(T):
                dec.decode_step(probs[t], got[t])
        torch.cuda.synchronize()
        ev[2].record(stream)
        g_dec.replay()
        ev[3].record(stream)
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3]), streams, bool(torch.equal(got, syms))

    def reference(ext):
        pitch = (max(256, T * 8) + 3) // 4
        ds = torch.cuda.default_stream(dev)
        torch.cuda.synchronize()
        enc = ext.RangeCoderBatch(N, K, pitch)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ds)
        for t in range(T):
            enc.encode_step_from_device(syms[t].data_ptr(), probs[t].data_ptr(), 0)
        enc.finalize()
        e1.record(ds)
        torch.cuda.synchronize()
        streams = [np.asarray(x, np.uint32) for x in enc.get_compressed_host()]
        dec = ext.RangeCoderBatch(N, K, pitch)
        dec.load_compressed_from_host(streams)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e2.record(ds)
        dec.init_decoder_from_current_bytes()
        for t in range(T):
            dec.decode_step_to_device(probs[t].data_ptr(), out.data_ptr(), 0)
        e3.record(ds)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1), e2.elapsed_time(e3), streams

    for _ in range(a.warmup):
        ours()
    clocks.start()
    runs = [ours() for _ in range(a.steps)]
    clk = clocks.stop()
    enc_ms = max(r[0] for r in runs)
    dec_ms = max(r[1] for r in runs)
    streams, ok = runs[-1][2], all(r[3] for r in runs)
    words = sum(len(x) for x in streams)
    ext = load_ref_pyrc()
    ref = None
    if ext is not None:
        for _ in range(min(a.warmup, 1)):
            reference(ext)
        r_enc, r_dec, r_streams = reference(ext)
        same = len(r_streams) == len(streams) and all(np.array_equal(x, y) for x, y in zip(r_streams, streams))
        ref = {"encode_symbols_per_s": N * T / (r_enc * 1e-3), "decode_symbols_per_s": N * T / (r_dec * 1e-3),
               "encode_ms": r_enc, "decode_ms": r_dec, "streams_identical": bool(same),
               "source": "gpu_range_coder.py's extension built from the reference source (oracle/build_ref.sh)"}
    # algorithmic bytes of one launch: probability rows + symbol/out + coder state r/w + words
    per_enc = N * (K * 4 + 4 + 64) + words * 4 / T
    per_dec = N * (K * 4 + 4 + 64) + words * 4 / T
    enc_launch_ms, dec_launch_ms = enc_ms / (T + 1), dec_ms / (T + 1)
    achieved = per_dec / (dec_launch_ms * 1e-3) / 1e9
    line = {"metric": "Python-codec batch coder symbols/s (encode+decode)", "value": 2 * N * T / ((enc_ms + dec_ms) * 1e-3),
            "unit": "symbols/s", "n_gpus": 1, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": enc_ms + dec_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 rows, f64 prefix sums, u64 coder", "data": "synthetic: softmax(3 N(0,1)) rows, seed 5",
            "config": {"workload": f"pyrc: {N} streams x {T} positions, K = {K}", "l2": "one distinct 64 MiB row "
                       "buffer per position, 4 GiB in all; no flush needed"},
            "encode_symbols_per_s": N * T / (enc_ms * 1e-3), "decode_symbols_per_s": N * T / (dec_ms * 1e-3),
            "bits_per_symbol": 32.0 * words / (N * T), "roundtrip_ok": ok,
            "roofline": {"kernel": "pyrc_decode", "bound": "hbm", "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": None,
                         "peak_source": f"{peak_kind} (HBM copy)",
                         "encode_achieved": per_enc / (enc_launch_ms * 1e-3) / 1e9},
            "reference_extension": ref, "gpu_launches": 2 * (T + 1) + 1, "clocks": clk}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- coder leg
def coder_tile(dev, seed, tile, P, N, alpha=0.1):
    """Step tile `tile` of the configs[1] workload, generated on the device:
    for P positions x N streams a Dirichlet(alpha) distribution over 256
    symbols (normalised Gamma(alpha) draws), quantised to the reference's
    integer CDF Q_k = floor(C_k * (2^24 - 256)) + k with C_k the fp64
    exclusive prefix sum (Q_256 = 2^24), and a symbol drawn from it by
    inverse CDF.  The PRNG is torch's CUDA generator (Philox4x32-10,
    counter-based) seeded with seed * 1,000,003 + tile, so any tile can be
    regenerated on its own.  Returns (Q int32 view [P, N, 257], syms u8 [P, N])."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed * 1000003 + tile)
    Q = torch.empty((P, N, 257), dtype=torch.int32, device=dev)
    syms = torch.empty((P, N), dtype=torch.uint8, device=dev)
    ar = torch.arange(256, dtype=torch.int64, device=dev)
    for p in range(P):  # one position at a time keeps the fp64 temporaries at 128 MiB
        gam = torch._standard_gamma(torch.full((N, 256), alpha, device=dev), generator=g).double()
        c = torch.cumsum(gam, -1)
        c = c / c[:, -1:]
        excl = torch.cat([torch.zeros((N, 1), dtype=torch.float64, device=dev), c[:, :-1]], -1)
        q = torch.floor(excl * float((1 << 24) - 256)).to(torch.int64) + ar
        Q[p, :, :256] = q.to(torch.int32)
        Q[p, :, 256] = 1 << 24
        u = torch.rand((N, 1), dtype=torch.float64, device=dev, generator=g)
        syms[p] = torch.clamp((c < u).sum(-1), max=255).to(torch.uint8)
    return Q, syms


def run_coder(a):
    """65,536 independent streams x 65,536 symbols; one step = P
    positions of every stream (CDF tile generated on the device before the
    step, outside its timing), encoded with boa_rc_encode_cdf_steps; after
    the K encode steps and the finish, the same K tiles (regenerated) are
    decoded with boa_rc_decode_cdf_steps and compared with the drawn symbols.
    K steps cover positions 0..P*K-1 of every stream (65,536 / P steps are
    the whole streams)."""
    import torch
    import ctypes as Ct
    boa = __import__("__graft_entry__").load_package()
    L = boa.lib()
    ws, rank, local = dist_info()
    if rank != 0:
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(local)
    hbm_peak, _, _, peak_kind = load_peaks()
    N, P, K = a.streams, a.coder_tile, a.steps
    total_steps = 65536
    K = max(1, min(K, total_steps // P))
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = Ct.c_void_p(stream.cuda_stream)
    vp = lambda t: Ct.c_void_p(t.data_ptr())  # noqa: E731
    pitch = boa.capacity_words(P * max(K, a.warmup, 1) + 1)
    es = torch.empty(N * L.boa_rc_state_bytes(0), dtype=torch.uint8, device=dev)
    ds = torch.empty(N * L.boa_rc_state_bytes(1), dtype=torch.uint8, device=dev)
    words = torch.empty(N * pitch, dtype=torch.int32, device=dev)
    sizes = torch.zeros(N, dtype=torch.int32, device=dev)
    offs = torch.arange(N, dtype=torch.int64, device=dev) * pitch
    got = torch.empty((P, N), dtype=torch.uint8, device=dev)
    seed = 11

    def ck(rc):
        if rc != 0:
            raise RuntimeError(L.boa_last_error(None).decode())

    def run(tiles, timed):
        """Encode tiles [0, tiles), finish, decode them; per-tile event times."""
        enc_ms, dec_ms, ok = [], [], True
        ck(L.boa_rc_encoder_init(vp(es), N, sp))
        for t in range(tiles):
            Q, sy = coder_tile(dev, seed, t, P, N)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ck(L.boa_rc_encode_cdf_steps(vp(es), vp(Q), vp(sy), N, P, vp(words), pitch, sp))
            e1.record(stream)
            e1.synchronize()
            enc_ms.append(e0.elapsed_time(e1))
        ck(L.boa_rc_encoder_finish(vp(es), vp(words), pitch, vp(sizes), N, sp))
        ck(L.boa_rc_decoder_init(vp(ds), vp(words), vp(offs), vp(sizes), N, sp))
        for t in range(tiles):
            Q, sy = coder_tile(dev, seed, t, P, N)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            ck(L.boa_rc_decode_cdf_steps(vp(ds), vp(Q), N, P, vp(words), vp(offs), vp(got), sp))
            e1.record(stream)
            e1.synchronize()
            dec_ms.append(e0.elapsed_time(e1))
            ok = ok and bool(torch.equal(got, sy))
        return enc_ms, dec_ms, ok

    run(max(1, a.warmup), False)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    enc_ms, dec_ms, ok = run(K, True)
    clk = clocks.stop()
    n_words = sizes.cpu().numpy().view(np.uint32)
    failed = int((n_words == boa.BOA_STREAM_FAILED).sum())
    ok = ok and failed == 0
    t_enc, t_dec = sum(enc_ms), sum(dec_ms)
    syms_total = N * P * K
    bits_per_symbol = 32.0 * float(n_words.astype(np.float64).sum()) / syms_total

    # e2e: the same K steps from pinned host buffers, H2D copy of every tile
    # and D2H of the streams / symbols inside the timed region
    hQ = torch.empty((P, N, 257), dtype=torch.int32).pin_memory()
    hS = torch.empty((P, N), dtype=torch.uint8).pin_memory()
    dQ = torch.empty((P, N, 257), dtype=torch.int32, device=dev)
    dS = torch.empty((P, N), dtype=torch.uint8, device=dev)
    hW = torch.empty(N * pitch, dtype=torch.int32).pin_memory()
    hG = torch.empty((P, N), dtype=torch.uint8).pin_memory()
    e2e_ms, e2e_ok = 0.0, True
    ck(L.boa_rc_encoder_init(vp(es), N, sp))
    for t in range(K):
        Q, sy = coder_tile(dev, seed, t, P, N)
        hQ.copy_(Q)
        hS.copy_(sy)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dQ.copy_(hQ, non_blocking=True)
        dS.copy_(hS, non_blocking=True)
        ck(L.boa_rc_encode_cdf_steps(vp(es), vp(dQ), vp(dS), N, P, vp(words), pitch, sp))
        if t == K - 1:
            ck(L.boa_rc_encoder_finish(vp(es), vp(words), pitch, vp(sizes), N, sp))
            hW.copy_(words, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        e2e_ms += e0.elapsed_time(e1)
    words.copy_(hW)  # the decoder reads the streams the host received
    ck(L.boa_rc_decoder_init(vp(ds), vp(words), vp(offs), vp(sizes), N, sp))
    for t in range(K):
        Q, sy = coder_tile(dev, seed, t, P, N)
        hQ.copy_(Q)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dQ.copy_(hQ, non_blocking=True)
        ck(L.boa_rc_decode_cdf_steps(vp(ds), vp(dQ), N, P, vp(words), vp(offs), vp(got), sp))
        hG.copy_(got, non_blocking=True)
        e1.record(stream)
        e1.synchronize()
        e2e_ms += e0.elapsed_time(e1)
        e2e_ok = e2e_ok and bool(torch.equal(hG, sy.cpu()))

    # CPU baseline + checker: the CPU coder (oracle restatement of the
    # reference coder) on a subset of streams, word-exact against the GPU
    cpu = None
    if not a.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        O.build()
        sub = np.arange(0, N, max(1, N // 64))[:64]
        idx = torch.from_numpy(sub).to(dev)
        Qs = np.concatenate([coder_tile(dev, seed, t, P, N)[0][:, idx].cpu().numpy() for t in range(K)])
        Ss = np.concatenate([coder_tile(dev, seed, t, P, N)[1][:, idx].cpu().numpy() for t in range(K)])
        W = words.view(N, pitch)[idx].cpu().numpy().view(np.uint32)
        t0 = time.perf_counter()
        exact = True
        for j, s_ in enumerate(sub):
            ref = O.rc_encode_cdf(Qs[:, j].view(np.uint32), Ss[:, j])
            back = O.rc_decode_cdf(Qs[:, j].view(np.uint32), ref, Ss.shape[0])
            exact = exact and ref.size == n_words[s_] and np.array_equal(ref, W[j, :ref.size]) \
                and np.array_equal(back, Ss[:, j])
        dt = time.perf_counter() - t0
        cpu = {"value": 2 * len(sub) * Ss.shape[0] / dt, "unit": "symbols/s", "cores": 1, "kind": "port",
               "sample": f"{len(sub)} of the {N} streams x {Ss.shape[0]} symbols, encode + decode, one thread",
               "streams_word_exact_vs_cpu_coder": bool(exact)}
        ok = ok and exact

    # roofline of the dominant kernel: the decoder reads each symbol's whole
    # 257-entry CDF row (1,028 B) plus the symbol byte it writes
    dec_launch_ms = t_dec / K
    per_launch = N * P * (257 * 4 + 1)
    achieved = per_launch / (dec_launch_ms * 1e-3) / 1e9
    enc_bytes = N * P * (2 * 4 + 1)
    line = {"metric": "range-coder symbols/s (encode + decode)", "value": 2 * syms_total / ((t_enc + t_dec) * 1e-3),
            "unit": "symbols/s", "n_gpus": 1, "steps": K, "warmup": a.warmup, "ms_per_step": (t_enc + t_dec) / K,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32 CDF, u64 coder",
            "data": "synthetic: Dirichlet(0.1) distributions over 256 symbols drawn on the device (torch Philox)",
            "config": {"workload": f"configs[1]: {N} streams x 65536 symbols, range coder alone",
                       "step": f"{P} positions of all {N} streams; the {K} timed steps are positions 0..{P * K - 1} "
                               f"(encode steps, finish, then decode steps); {total_steps // P} steps are the whole "
                               "streams",
                       "l2": f"each step's CDF tile is {N * P * 1028 / 2**30:.2f} GiB, above L2; no flush needed",
                       "cdf_generation": "outside the timed region, before each step"},
            "encode_symbols_per_s": syms_total / (t_enc * 1e-3), "decode_symbols_per_s": syms_total / (t_dec * 1e-3),
            "roofline": {"kernel": "rc_decode_cdf_kernel", "bound": "hbm", "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": None,
                         "peak_source": f"{peak_kind} (HBM copy)",
                         "algorithmic_bytes_per_launch": per_launch,
                         "encode_kernel": {"name": "rc_encode_cdf_kernel", "algorithmic_bytes_per_launch": enc_bytes,
                                           "achieved_GBps": enc_bytes / (t_enc / K * 1e-3) / 1e9}},
            "cpu_baseline": cpu,
            "e2e": {"value": 2 * syms_total / (e2e_ms * 1e-3), "unit": "symbols/s",
                    "h2d_bytes_per_step": 2 * N * P * 257 * 4 + N * P + N * pitch * 4 / K,
                    "d2h_bytes_per_step": N * pitch * 4 / K + N * P,
                    "how": "per step: pinned-host CDF tile copied in, coded, symbols / streams copied out"},
            "gpu_launches": 2,
            "clocks": clk,
            "bits_per_symbol": bits_per_symbol, "failed_streams": failed,
            "roundtrip_ok": bool(ok and e2e_ok)}
    print(json.dumps(line), flush=True)
    if not (ok and e2e_ok):
        print("coder round trip NOT exact", file=sys.stderr, flush=True)
        sys.exit(3)


# --------------------------------------------------------------------------- GPU leg
WORKLOADS = {
    # name: (backbone, d_model, layers, weight seed, chunks (whole job), chunk_len, data, data seed, sharding)
    "roundtrip": ("mamba", 256, 8, 0, 16384, 16384, "particle", 1, "weak"),
    "cms": ("mamba", 64, 2, 0, 16384, 4096, "particle", 1, "weak"),
    "configs3": ("mingru", 256, 8, 2, 16384, 16384, "markov", 3, "weak"),
    "configs4": ("mamba", 512, 16, 3, 262144, 16384, "particle", 4, "strong"),
}


def shard_range(n_chunks, ws, rank, mode):
    """Chunks [c0, c0 + n) of this rank: weak scaling gives every rank the
    whole workload's chunk count (its own stream, seed + rank); strong
    scaling splits the workload's chunks evenly in contiguous ranges."""
    if mode == "weak":
        return 0, n_chunks
    per = -(-n_chunks // ws)
    c0 = min(n_chunks, rank * per)
    return c0, min(n_chunks, c0 + per) - c0


def workload_data(a, kind, seed, total_chunks, S, c0, C, window, rank, weak):
    """u8 [C, window]: the first `window` bytes of this rank's chunks."""
    boa = __import__("__graft_entry__").load_package()
    if kind == "markov":
        return boa.synth.markov_windows(seed + (rank if weak else 0), C, window)
    return boa.synth.particle_windows(total_chunks * S, seed + (rank if weak else 0), S, c0, C, window)


def main():
    a = apply_workload(parse())
    if a.workload == "pyrc":
        return run_pyrc(a)
    if a.impl == "reference":
        return run_reference(a)  # a already carries the workload's model and weights
    if a.workload == "coder":
        return run_coder(a)
    import torch
    ws, rank, local = dist_info()
    dist = None
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                device_id=torch.device("cuda", local) if torch.cuda.is_available() else None)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    boa = __import__("__graft_entry__").load_package()
    boa.lib()
    hbm_peak, tf_burst, tf_sust, peak_kind = load_peaks()
    backbone, _, _, wseed, _, _, kind, dseed, scaling = WORKLOADS[a.workload]

    td = tempfile.mkdtemp()
    wpath = os.path.join(td, f"w{rank}.bin")
    if a.weights:
        wpath = a.weights
    else:
        boa.synth.write_random_weights(wpath, backbone, a.d_model, a.layers, wseed)
    m = boa.Model(wpath, backbone, a.d_model, a.layers, device=local)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    m.set_stream(stream.cuda_stream)

    # ---- the step: one T-position compress tile plus the T decode steps of the
    # same positions, over every chunk of this rank.  K steps cover positions
    # 1..T*K of each chunk (position 0 is the raw first byte); K = (S-1)/T steps
    # are the whole chunks.  The timed region runs the K steps as one compress
    # call over the chunks' first T*K+1 bytes, then one decompress call.
    S = a.chunk_len
    T = min(64, S - 1)
    K = max(1, min(a.steps, -(-(S - 1) // T)))
    Lp = min(S, T * K + 1)
    Lw = min(Lp, T * max(1, a.warmup) + 1)  # the warm-up data is a prefix of the timed data
    c0, C = shard_range(a.chunks, ws, rank, scaling)
    weak = scaling == "weak"
    t_gen = time.perf_counter()
    host = np.ascontiguousarray(workload_data(a, kind, dseed, a.chunks, S, c0, C, Lp, rank, weak))
    t_gen = time.perf_counter() - t_gen
    n = C * Lp
    data = torch.from_numpy(host.reshape(-1)).to(dev)
    cap = C * boa.capacity_words(max(Lp, Lw))
    payload = torch.empty(cap, dtype=torch.int32, device=dev)
    sizes = torch.empty(C, dtype=torch.int32, device=dev)
    offsets = torch.empty(C + 1, dtype=torch.int64, device=dev)
    first = torch.empty(C, dtype=torch.uint8, device=dev)
    out = torch.empty(n, dtype=torch.uint8, device=dev)

    def compress(src, ln):
        m.compress_device(src.data_ptr(), C * ln, ln, C, first.data_ptr(), payload.data_ptr(), cap,
                          sizes.data_ptr(), offsets.data_ptr())

    def decompress(ln):
        m.decompress_device(payload.data_ptr(), offsets.data_ptr(), sizes.data_ptr(), first.data_ptr(), C * ln,
                            ln, C, out.data_ptr())

    # buffers for the timed geometry are allocated here, outside every timed region
    m.reserve(C, Lp)
    # warm-up: W steps (the chunks' first T*W+1 bytes), untimed
    wdata = data.view(C, Lp)[:, :Lw].contiguous().view(-1)
    for _ in range(1 if a.warmup > 0 else 0):
        compress(wdata, Lw)
        decompress(Lw)
    m.sync()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    l0 = m.launch_count()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record(stream)
    compress(data, Lp)
    e1.record(stream)
    decompress(Lp)
    e2.record(stream)
    e2.synchronize()
    m.sync()
    launches = (m.launch_count() - l0) / K
    clk = clocks.stop()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    comp_ms, dec_ms = e0.elapsed_time(e1), e1.elapsed_time(e2)
    ok = bool(torch.equal(out, data))
    total_words = int(offsets[C].item())
    t = torch.tensor([comp_ms, dec_ms, comp_ms + dec_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    comp_ms, dec_ms, job_ms = t.tolist()
    step_ms = job_ms / K
    # BOA2 file size of this rank's coded prefix (header 33 B, payload, index, CRC)
    sz = sizes.cpu().numpy().astype(np.int64) * 4
    varint = np.ones_like(sz) + (sz >= 1 << 7) + (sz >= 1 << 14) + (sz >= 1 << 21) + (sz >= 1 << 28)
    boa_bytes = 33 + total_words * 4 + 4 + C + int(varint.sum()) + 4
    bpb = 8.0 * boa_bytes / n

    # ---- e2e: the same K steps through the host-buffer C ABI from pinned host
    # memory (boa_compress_chunks / boa_decompress_chunks), copies included
    h_in = torch.from_numpy(host.reshape(-1)).pin_memory()
    h_pay = torch.empty(cap, dtype=torch.int32).pin_memory()
    h_sizes = np.zeros(C, np.uint32)
    h_first = np.zeros(C, np.uint8)
    h_out = torch.empty(n, dtype=torch.uint8).pin_memory()
    lens = np.full(C, Lp, np.uint32)
    import ctypes as Ct
    L = boa.lib()
    e2e_ms, e2e_words = float("nan"), 0
    if a.e2e_steps > 0:
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        used = Ct.c_uint64()
        rc = L.boa_compress_chunks(m.h, Ct.cast(h_in.data_ptr(), boa._u8p), n, Lp, 0, C,
                                   h_first.ctypes.data_as(boa._u8p), Ct.cast(h_pay.data_ptr(), boa._u32p), cap,
                                   h_sizes.ctypes.data_as(boa._u32p), Ct.byref(used))
        boa._check(rc, m.h)
        rc = L.boa_decompress_chunks(m.h, Ct.cast(h_pay.data_ptr(), boa._u32p), h_sizes.ctypes.data_as(boa._u32p),
                                     h_first.ctypes.data_as(boa._u8p), lens.ctypes.data_as(boa._u32p), Lp, C,
                                     Ct.cast(h_out.data_ptr(), boa._u8p))
        boa._check(rc, m.h)
        s1.record(stream)
        s1.synchronize()
        e2e_ms = s0.elapsed_time(s1)
        e2e_words = used.value
    e2e_ok = bool(torch.equal(h_out, h_in)) if a.e2e_steps > 0 else True
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_job_ms = te.item()

    # ---- per-kernel timing: instrumented pass (events around every launch)
    # over one compress tile and T decode steps of the same chunks
    m.set_profiling(True)
    m.profile()
    tl = T + 1
    tdata = data.view(C, Lp)[:, :tl].contiguous().view(-1)
    compress(tdata, tl)
    prof_c = m.profile()
    decompress(tl)
    prof_d = m.profile()
    m.set_profiling(False)
    kern = {}
    for name in prof_c:
        cms, cn = prof_c[name]
        dms, dn = prof_d[name]
        kern[name] = {"compress_ms_per_launch": cms / cn if cn else 0.0, "compress_launches": cn,
                      "decode_ms_per_launch": dms / dn if dn else 0.0, "decode_launches": dn,
                      "ms_per_step": cms + dms}
    dom = max(kern, key=lambda k: kern[k]["ms_per_step"])
    kd = kern[dom]
    Bc = m.batch_geometry(C, S, True)[0]
    in_decode = kd["decode_ms_per_launch"] * kd["decode_launches"] >= kd["compress_ms_per_launch"] * kd["compress_launches"]
    if in_decode:
        bound, work = algorithmic_per_launch(dom, Bc, 1, a.d_model, a.layers)
        dur = kd["decode_ms_per_launch"]
        phase = f"decompress step (M = {Bc} chunks)"
    else:
        bound, work = algorithmic_per_launch(dom, Bc, T, a.d_model, a.layers)
        dur = kd["compress_ms_per_launch"]
        phase = f"compress tile (M = {Bc} x {T})"
    if bound == "tensor":
        achieved = work / (dur * 1e-3) / 1e12
        peak, unit = tf_sust, "TFLOP/s"
    else:
        achieved = work / (dur * 1e-3) / 1e9
        peak, unit = hbm_peak, "GB/s"

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and ws == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample, _ = cpu_sample(wpath, a.d_model, a.layers, S, dseed, a.cpu_seconds, threads, backbone, kind)
        cpu = {"value": v, "unit": "MB/s", "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        total = n * ws if weak else a.chunks * Lp
        pub_rt, pub = published_baseline(a)
        step_rl = step_roofline(a.d_model, a.layers, Bc, T, hbm_peak, tf_sust) if backbone == "mamba" else {}
        if step_rl:
            # batches run one after another, so the bound of one batch is the rank's bound
            step_rl["compress_frac"] = (n / MiB / (comp_ms * 1e-3)) / step_rl["compress_bound_MBps"]
            step_rl["decompress_frac"] = (n / MiB / (dec_ms * 1e-3)) / step_rl["decompress_bound_MBps"]
            step_rl["peaks"] = f"{peak_kind}: HBM copy {hbm_peak} GB/s, bf16 sustained {tf_sust} TFLOP/s"
        value = total / MiB / (job_ms * 1e-3)
        state_b = C * a.layers * (19 * 2 * a.d_model if backbone == "mamba" else a.d_model) * 4
        line = {
            "metric": "compress+decompress round-trip MB/s",
            "value": value,
            "unit": "MB/s", "n_gpus": ws, "steps": K, "warmup": a.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": scaling,
            "vs_baseline": value / pub_rt if pub_rt else None,
            "dtype": "bf16x3 (fp32-accurate)",
            "data": (f"synthetic: seeded {'order-2 Markov bytes' if kind == 'markov' else 'float32 particle records'}"
                     + (f", weights {os.path.basename(a.weights)}" if a.weights else ", random-init weights")),
            "config": {"workload": workload_name(a, C, S),
                       "backbone": backbone, "d_model": a.d_model, "n_layers": a.layers,
                       "chunks_total": a.chunks, "chunks_per_gpu": C, "chunk_len": S,
                       "batch_chunks": Bc, "compress_tile": T, "parallelism": f"chunk-sharded x{ws} ({scaling})",
                       "step": (f"one {T}-position compress tile + the {T} decode steps of the same positions over "
                                f"all {C} chunks of the GPU; the {K} timed steps are positions 1..{Lp - 1} of every "
                                f"{S}-byte chunk (one compress call over the chunks' first {Lp} bytes, then one "
                                f"decompress call); {-(-(S - 1) // T)} steps are the whole chunks"),
                       "l2": (f"recurrent state {state_b / MiB / 1024:.2f} GiB per GPU "
                              + ("exceeds L2 (126 MB): every step streams it from HBM; no flush needed"
                                 if state_b > 126e6 else "fits in L2 (126 MB): warm-cache timing")),
                       "warmup": f"one untimed round trip of the same chunks' first {Lw} bytes ({a.warmup} steps)",
                       "input_gen_s": round(t_gen, 2)},
            "compress_MBps": total / MiB / (comp_ms * 1e-3),
            "decompress_MBps": total / MiB / (dec_ms * 1e-3),
            "roofline": {"kernel": dom, "phase": phase, "bound": bound, "achieved": achieved, "peak": peak,
                         "unit": unit, "frac": achieved / peak,
                         "traffic": (NCU_TRAFFIC_PER_CHUNK[(dom, "decode")] * Bc
                                     if in_decode and (dom, "decode") in NCU_TRAFFIC_PER_CHUNK
                                     and a.workload == "roundtrip" else None),
                         "peak_source": f"{peak_kind} ({'bf16 sustained' if bound == 'tensor' else 'HBM copy'})"},
            "step_roofline": step_rl,
            "published_baseline": pub,
            "kernels": kern,
            "cpu_baseline": cpu,
            "e2e": {"value": total / MiB / (e2e_job_ms * 1e-3), "unit": "MB/s",
                    "h2d_bytes_per_step": (n + e2e_words * 4 + C * 9) / K,
                    "d2h_bytes_per_step": (e2e_words * 4 + C * 5 + 8 + n) / K,
                    "how": "the K steps as one boa_compress_chunks + boa_decompress_chunks call from pinned host "
                           "buffers, CUDA events around both, max over ranks"},
            "gpu_launches": int(round(launches)),
            "clocks": clk,
            "bits_per_byte": bpb,
            "roundtrip_ok": ok and e2e_ok,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if not (ok and e2e_ok):
        print(f"rank {rank}: round trip NOT byte-exact (device {ok}, e2e {e2e_ok})", file=sys.stderr, flush=True)
        sys.exit(3)


if __name__ == "__main__":
    main()
