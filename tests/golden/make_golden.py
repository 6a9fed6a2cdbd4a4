"""Generates the golden fixtures in tests/golden/ from the REFERENCE itself.

Run on a GPU box (the reference is CUDA-only) after oracle/build_ref.sh has
built oracle/_ref/{boa_constrictor,ref_logits} from the reference sources:

    python tests/golden/make_golden.py <out_dir>

Fixtures written (all inputs regenerate from the seeds recorded in
manifest.json, so only reference OUTPUTS are stored):
  ref_logits_<cfg>.npz   tokens + logits from BoaPredictorGPU::forward_chunk
                         and ::step_batch (boa_gpu.hpp:1034, :1081)
  ref_exact.boa          reference CLI compress of a seeded byte stream under
                         an exact-logit model (synth.exact_logit_weights):
                         pins quantiser + range coder + BOA2 container bit-exact
  ref_exact_warm.boa     the same with --warm-start --gpu-batch 3: pins the
                         warm-start container fields (flags bit0, batch)
  ref_pyrc.npz           streams of the Python codec's batch coder
                         (gpu_range_coder.py RangeCoderBatch, built by
                         oracle/build_ref.sh) over seeded probability rows
  ref_rand_d256L8.boa    reference CLI compress of 64 KiB of particle records
                         under the configs[0] model: container layout and the
                         reference's bits/byte
  manifest.json          parameters, sizes, sha256, reference round-trip flags

With --configs4 it writes only ref_logits_d512L16.npz (the configs[4] model,
Mamba d512 / 16 layers, seed 3, both forms) and the reference CLI's container
size for 32 KiB of particle records under it, merged into manifest.json.

With --trained it writes only the trained-checkpoint fixtures (weights
converted by convert_trained.py) and merges them into manifest.json:
  ref_logits_trained_<name>.npz  tokens (bytes of the particle stream) and
                                 the reference's logits in both forms
  manifest "trained_result"      size, sha256 and round-trip flag of the
                                 reference CLI's container of 64 KiB of
                                 particle records under each model
"""
import hashlib
import importlib.util
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.path.join(ROOT, "oracle", "_ref")
spec = importlib.util.spec_from_file_location(
    "synth", os.path.join(ROOT, "boa-constrictor_b200", "synth.py"))
synth = importlib.util.module_from_spec(spec)
spec.loader.exec_module(synth)

EXACT = dict(d_model=64, n_layers=1, seed=7, support=list(range(0, 256, 5)) + [255],
             n_bytes=4001, data_seed=11, chunk=1000, batch=8, p_out=0.05)
# "backbone" defaults to mamba and "std" (weight init) to 0.02; the RNN
# backbones use std 0.1 so that their gates leave the linear region.
LOGIT_CFGS = [dict(name="d64L2", d_model=64, n_layers=2, seed=3, B=3, T=40, tok_seed=5),
              dict(name="d256L8", d_model=256, n_layers=8, seed=0, B=2, T=48, tok_seed=6),
              dict(name="mingru_d64L2", backbone="mingru", std=0.1, d_model=64, n_layers=2, seed=3, B=3, T=40,
                   tok_seed=5),
              dict(name="lstm_d64L2", backbone="lstm", std=0.1, d_model=64, n_layers=2, seed=3, B=3, T=40,
                   tok_seed=5),
              dict(name="gru_d64L2", backbone="gru", std=0.1, d_model=64, n_layers=2, seed=3, B=3, T=40,
                   tok_seed=5)]
RAND = dict(d_model=256, n_layers=8, seed=0, n_bytes=65536, data_seed=1, chunk=4096, batch=16)
# Python-codec coder cases: N streams x T steps over K symbols
PYRC = [dict(name="k256", seed=21, N=48, T=160, K=256, alpha=0.1),
        dict(name="k7", seed=22, N=33, T=90, K=7, alpha=0.5),
        dict(name="k1000", seed=23, N=9, T=40, K=1000, alpha=0.05)]


# trained checkpoints (tests/golden/trained_<name>.bin, see convert_trained.py)
TRAINED = [dict(name="mamba_d64L2", backbone="mamba", d_model=64, n_layers=2),
           dict(name="mamba_d80L1", backbone="mamba", d_model=80, n_layers=1),
           dict(name="mamba_d128L1", backbone="mamba", d_model=128, n_layers=1),
           dict(name="mingru_d160L1", backbone="mingru", d_model=160, n_layers=1)]
TRAINED_DATA = dict(n_bytes=65536, data_seed=41, chunk=4096, batch=16, B=3, T=64)


def trained_tokens():
    """B rows of T consecutive bytes of the particle stream (the models' own
    kind of input), row b starting at byte b * chunk."""
    data = np.frombuffer(synth.particle_stream(TRAINED_DATA["n_bytes"], TRAINED_DATA["data_seed"]), np.uint8)
    B, T, S = TRAINED_DATA["B"], TRAINED_DATA["T"], TRAINED_DATA["chunk"]
    return np.stack([data[b * S: b * S + T] for b in range(B)])


def main_trained(out_dir):
    tmp = os.path.join(out_dir, "_tmp")
    os.makedirs(tmp, exist_ok=True)
    man = json.load(open(os.path.join(out_dir, "manifest.json")))
    man["trained"] = TRAINED
    man["trained_data"] = TRAINED_DATA
    man["trained_result"] = {}
    tok = trained_tokens()
    tf = os.path.join(tmp, "tok.u8")
    tok.tofile(tf)
    data = synth.particle_stream(TRAINED_DATA["n_bytes"], TRAINED_DATA["data_seed"])
    fin = os.path.join(tmp, "trained.in"); open(fin, "wb").write(data)
    for c in TRAINED:
        w = os.path.join(out_dir, f"trained_{c['name']}.bin")
        B, T = tok.shape
        res = {}
        for mode in ("chunk", "step"):
            of = os.path.join(tmp, f"lg_{mode}.f32")
            run([os.path.join(REF, "ref_logits"), w, c["backbone"], str(c["d_model"]), str(c["n_layers"]),
                 tf, str(B), str(T), mode, of])
            res[mode] = np.fromfile(of, np.float32).reshape(B, T, 256)
        np.savez_compressed(os.path.join(out_dir, f"ref_logits_trained_{c['name']}.npz"),
                            tokens=tok, chunk=res["chunk"], step=res["step"])
        boa = os.path.join(tmp, "t.boa")
        args = [str(c["d_model"]), str(c["n_layers"]), "--backbone", c["backbone"]]
        run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa] + args +
            ["--gpu-batch", str(TRAINED_DATA["batch"]), "--chunk-size", str(TRAINED_DATA["chunk"])])
        back = os.path.join(tmp, "t.out")
        run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa, back] + args +
            ["--gpu-batch", str(TRAINED_DATA["batch"])])
        man["trained_result"][c["name"]] = dict(
            weights_sha=sha(open(w, "rb").read()), input_sha=sha(data), boa_bytes=os.path.getsize(boa),
            boa_sha=sha(open(boa, "rb").read()), bits_per_byte=8.0 * os.path.getsize(boa) / len(data),
            ref_roundtrip=open(back, "rb").read() == data)
    for f in os.listdir(tmp):
        os.remove(os.path.join(tmp, f))
    os.rmdir(tmp)
    json.dump(man, open(os.path.join(out_dir, "manifest.json"), "w"), indent=1)
    print(json.dumps(man["trained_result"], indent=1))


def pyrc_inputs(cfg):
    """probs [T][N][K] float32 (Dirichlet rows with some exact zeros and a few
    all-zero rows, which take the equal-split branch), symbols [T][N] int32
    drawn from each row, and a ragged activity mask [T][N] (stream n is active
    for t < len_n), as codec.compress_GPU masks finished chunks."""
    rng = np.random.default_rng(cfg["seed"])
    T, N, K = cfg["T"], cfg["N"], cfg["K"]
    probs = rng.dirichlet(np.full(K, cfg["alpha"]), size=(T, N)).astype(np.float32)
    probs[rng.random((T, N, K)) < 0.02] = 0.0
    probs[rng.random((T, N)) < 0.01] = 0.0
    syms = np.empty((T, N), np.int32)
    u = rng.random((T, N))
    for t in range(T):
        for n in range(N):
            p = probs[t, n].astype(np.float64)
            c = np.cumsum(p / p.sum()) if p.sum() > 0 else np.arange(1, K + 1) / K
            syms[t, n] = min(int(np.searchsorted(c, u[t, n], side="right")), K - 1)
    lens = rng.integers(1, T + 1, N)
    lens[0] = T
    mask = np.arange(T)[:, None] < lens[None, :]
    return probs, syms, mask


def run_ref_pyrc(ext, cfg):
    """Encode then decode one case through the reference extension."""
    import torch
    probs, syms, mask = pyrc_inputs(cfg)
    T, N, K = cfg["T"], cfg["N"], cfg["K"]
    pitch = (max(256, T * 8) + 3) // 4  # the gpu.queue.RangeCoderBatch default
    P = torch.from_numpy(probs).cuda()
    S = torch.from_numpy(syms).cuda()
    Mk = torch.from_numpy(mask.astype(np.uint8)).cuda()
    enc = ext.RangeCoderBatch(N, K, pitch)
    for t in range(T):
        enc.encode_step_from_device(S[t].data_ptr(), P[t].data_ptr(), Mk[t].data_ptr())
    enc.finalize()
    streams = [np.asarray(a, np.uint32) for a in enc.get_compressed_host()]
    dec = ext.RangeCoderBatch(N, K, pitch)
    dec.load_compressed_from_host(streams)
    dec.init_decoder_from_current_bytes()
    out = torch.zeros(N, dtype=torch.int32, device="cuda")
    got = np.zeros((T, N), np.int32)
    for t in range(T):
        dec.decode_step_to_device(P[t].data_ptr(), out.data_ptr(), Mk[t].data_ptr())
        got[t] = out.cpu().numpy()
    decoded_ok = bool(np.array_equal(np.where(mask, got, 0), np.where(mask, syms, 0)))
    return streams, decoded_ok, hashlib.sha256(probs.tobytes()).hexdigest()


def exact_input(cfg):
    """Bytes mostly from the support (exercise normal coding) and sometimes
    outside it (frequency-1 symbols: long carry runs)."""
    rng = np.random.default_rng(cfg["data_seed"])
    sup = np.array(cfg["support"], np.uint8)
    data = sup[rng.integers(0, len(sup), cfg["n_bytes"])]
    out = rng.random(cfg["n_bytes"]) < cfg["p_out"]
    data[out] = rng.integers(0, 256, int(out.sum()), dtype=np.uint8)
    return data.tobytes()


def sha(b):
    return hashlib.sha256(b).hexdigest()


def run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{cmd} failed: {r.stdout[-2000:]} {r.stderr[-2000:]}")
    return r.stdout


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    tmp = os.path.join(out_dir, "_tmp")
    os.makedirs(tmp, exist_ok=True)
    man = {"exact": EXACT, "logits": LOGIT_CFGS, "rand": RAND}

    for c in LOGIT_CFGS:
        w = os.path.join(tmp, f"w_{c['name']}.bin")
        bb = c.get("backbone", "mamba")
        synth.write_random_weights(w, bb, c["d_model"], c["n_layers"], c["seed"], std=c.get("std", 0.02))
        tok = np.random.default_rng(c["tok_seed"]).integers(0, 256, (c["B"], c["T"]), dtype=np.uint8)
        tf = os.path.join(tmp, "tok.u8")
        tok.tofile(tf)
        res = {}
        for mode in ("chunk", "step"):
            of = os.path.join(tmp, f"lg_{mode}.f32")
            run([os.path.join(REF, "ref_logits"), w, bb, str(c["d_model"]), str(c["n_layers"]),
                 tf, str(c["B"]), str(c["T"]), mode, of])
            res[mode] = np.fromfile(of, np.float32).reshape(c["B"], c["T"], 256)
        np.savez_compressed(os.path.join(out_dir, f"ref_logits_{c['name']}.npz"),
                            tokens=tok, chunk=res["chunk"], step=res["step"])

    # exact-logit container
    w = os.path.join(tmp, "w_exact.bin")
    synth.write_weights(w, synth.exact_logit_weights(EXACT["d_model"], EXACT["n_layers"],
                                                     EXACT["seed"], EXACT["support"]))
    data = exact_input(EXACT)
    fin = os.path.join(tmp, "exact.in"); open(fin, "wb").write(data)
    boa = os.path.join(out_dir, "ref_exact.boa")
    run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa, str(EXACT["d_model"]),
         str(EXACT["n_layers"]), "--gpu-batch", str(EXACT["batch"]), "--chunk-size", str(EXACT["chunk"])])
    back = os.path.join(tmp, "exact.out")
    run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa, back, str(EXACT["d_model"]),
         str(EXACT["n_layers"]), "--gpu-batch", str(EXACT["batch"])])
    man["exact_result"] = dict(input_sha=sha(data), boa_bytes=os.path.getsize(boa),
                               boa_sha=sha(open(boa, "rb").read()),
                               ref_roundtrip=open(back, "rb").read() == data)

    boa_w = os.path.join(out_dir, "ref_exact_warm.boa")
    run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa_w, str(EXACT["d_model"]),
         str(EXACT["n_layers"]), "--gpu-batch", "3", "--chunk-size", str(EXACT["chunk"]), "--warm-start"])
    back_w = os.path.join(tmp, "exact_warm.out")
    run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa_w, back_w, str(EXACT["d_model"]),
         str(EXACT["n_layers"])])
    man["exact_warm_result"] = dict(boa_bytes=os.path.getsize(boa_w), ref_roundtrip=open(back_w, "rb").read() == data)

    # random-init configs[0] model on particle records
    w = os.path.join(tmp, "w_rand.bin")
    synth.write_random_weights(w, "mamba", RAND["d_model"], RAND["n_layers"], RAND["seed"])
    data = synth.particle_stream(RAND["n_bytes"], RAND["data_seed"])
    fin = os.path.join(tmp, "rand.in"); open(fin, "wb").write(data)
    boa = os.path.join(out_dir, "ref_rand_d256L8.boa")
    run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa, str(RAND["d_model"]),
         str(RAND["n_layers"]), "--gpu-batch", str(RAND["batch"]), "--chunk-size", str(RAND["chunk"])])
    back = os.path.join(tmp, "rand.out")
    run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa, back, str(RAND["d_model"]),
         str(RAND["n_layers"]), "--gpu-batch", str(RAND["batch"])])
    man["rand_result"] = dict(input_sha=sha(data), boa_bytes=os.path.getsize(boa),
                              boa_sha=sha(open(boa, "rb").read()),
                              bits_per_byte=8.0 * os.path.getsize(boa) / len(data),
                              ref_roundtrip=open(back, "rb").read() == data)
    # the reference's own warm-start round trip on the same model and data
    boa_rw = os.path.join(tmp, "rand_warm.boa")
    run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa_rw, str(RAND["d_model"]),
         str(RAND["n_layers"]), "--gpu-batch", "4", "--chunk-size", str(RAND["chunk"]), "--warm-start"])
    back_rw = os.path.join(tmp, "rand_warm.out")
    run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa_rw, back_rw, str(RAND["d_model"]),
         str(RAND["n_layers"])])
    man["rand_warm_result"] = dict(ref_roundtrip=open(back_rw, "rb").read() == data)
    # the Python codec's batch coder, built from gpu_range_coder.py
    import glob
    import importlib.machinery
    so = glob.glob(os.path.join(REF, "_gpu_range_cuda_ext*.so"))[0]
    loader = importlib.machinery.ExtensionFileLoader("_gpu_range_cuda_ext", so)
    ext = importlib.util.module_from_spec(importlib.util.spec_from_loader("_gpu_range_cuda_ext", loader))
    loader.exec_module(ext)
    man["pyrc"] = PYRC
    man["pyrc_result"] = {}
    arrays = {}
    for c in PYRC:
        streams, ok, probs_sha = run_ref_pyrc(ext, c)
        arrays[c["name"] + "_sizes"] = np.array([len(x) for x in streams], np.int32)
        arrays[c["name"] + "_words"] = np.concatenate(streams).astype(np.uint32)
        man["pyrc_result"][c["name"]] = dict(ref_decoded=ok, probs_sha=probs_sha)
    np.savez_compressed(os.path.join(out_dir, "ref_pyrc.npz"), **arrays)
    for f in os.listdir(tmp):
        os.remove(os.path.join(tmp, f))
    os.rmdir(tmp)
    json.dump(man, open(os.path.join(out_dir, "manifest.json"), "w"), indent=1)
    print(json.dumps(man, indent=1))


# configs[4] model (Mamba d512 / 16 layers, seed 3) at full depth
CONFIGS4_LOGITS = dict(name="d512L16", d_model=512, n_layers=16, seed=3, B=2, T=32, tok_seed=9)
CONFIGS4_DATA = dict(n_bytes=32768, data_seed=4, chunk=4096, batch=8)


def main_configs4(out_dir):
    """--configs4: the reference's logits of the configs[4] model in both forms
    (ref_logits_d512L16.npz, appended to manifest "logits") and the size of the
    reference CLI's container of 32 KiB of particle records under it
    (manifest "configs4_result")."""
    tmp = os.path.join(out_dir, "_tmp")
    os.makedirs(tmp, exist_ok=True)
    man = json.load(open(os.path.join(out_dir, "manifest.json")))
    c = CONFIGS4_LOGITS
    w = os.path.join(tmp, "w_c4.bin")
    synth.write_random_weights(w, "mamba", c["d_model"], c["n_layers"], c["seed"])
    tok = np.random.default_rng(c["tok_seed"]).integers(0, 256, (c["B"], c["T"]), dtype=np.uint8)
    tf = os.path.join(tmp, "tok.u8")
    tok.tofile(tf)
    res = {}
    for mode in ("chunk", "step"):
        of = os.path.join(tmp, f"lg_{mode}.f32")
        run([os.path.join(REF, "ref_logits"), w, "mamba", str(c["d_model"]), str(c["n_layers"]),
             tf, str(c["B"]), str(c["T"]), mode, of])
        res[mode] = np.fromfile(of, np.float32).reshape(c["B"], c["T"], 256)
    np.savez_compressed(os.path.join(out_dir, f"ref_logits_{c['name']}.npz"),
                        tokens=tok, chunk=res["chunk"], step=res["step"])
    man["logits"] = [x for x in man["logits"] if x["name"] != c["name"]] + [c]
    D = CONFIGS4_DATA
    data = synth.particle_stream(D["n_bytes"], D["data_seed"])
    fin = os.path.join(tmp, "c4.in"); open(fin, "wb").write(data)
    boa = os.path.join(tmp, "c4.boa")
    args = [str(c["d_model"]), str(c["n_layers"])]
    run([os.path.join(REF, "boa_constrictor"), "compress", w, fin, boa] + args +
        ["--gpu-batch", str(D["batch"]), "--chunk-size", str(D["chunk"])])
    back = os.path.join(tmp, "c4.out")
    run([os.path.join(REF, "boa_constrictor"), "decompress", w, boa, back] + args + ["--gpu-batch", str(D["batch"])])
    man["configs4_data"] = D
    man["configs4_result"] = dict(input_sha=sha(data), boa_bytes=os.path.getsize(boa),
                                  bits_per_byte=8.0 * os.path.getsize(boa) / len(data),
                                  ref_roundtrip=open(back, "rb").read() == data)
    for f in os.listdir(tmp):
        os.remove(os.path.join(tmp, f))
    os.rmdir(tmp)
    json.dump(man, open(os.path.join(out_dir, "manifest.json"), "w"), indent=1)
    print(json.dumps(man["configs4_result"], indent=1))


if __name__ == "__main__":
    flags = {"--trained", "--configs4"}
    args = [a for a in sys.argv[1:] if a not in flags]
    out = args[0] if args else os.path.join(ROOT, "tests", "golden")
    if "--trained" in sys.argv:
        main_trained(out)
    elif "--configs4" in sys.argv:
        main_configs4(out)
    else:
        main(out)
