"""Converts trained checkpoints of the reference into .bin weight fixtures.

Runs in a container that has the reference checkout (the converter and the
checkpoints are read from it, nothing is written there):

    python tests/golden/convert_trained.py <reference root>

It calls the reference's own converter (portability_solved_cpp/
convert_boa_weights.py) on three of the C++-compatible checkpoints in
experiments/cms_experiment/ and writes tests/golden/trained_<name>.bin.
Unlike random-init weights these predict sharply non-uniform byte
distributions, so logits and bits/byte comparisons against the reference
are strict.  The widths cover d_model 64, 80 and 128 (Mamba, dt_rank 4, 5 and 8) and
160 (minGRU).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# name -> (checkpoint file, backbone, d_model, n_layers)
TRAINED = {
    "mamba_d64L2": ("cms_experiment_final_model_fp32_mambav1_64_2_20ep.pt", "mamba", 64, 2),
    "mamba_d80L1": ("cms_experiment_final_model_fp32_mambav1_80_1_20.pt", "mamba", 80, 1),
    "mamba_d128L1": ("cms_experiment_final_model_fp32_128dm_mambav1.pt", "mamba", 128, 1),
    "mingru_d160L1": ("cms_experiment_final_model_fp32_160MinGRU.pt", "mingru", 160, 1),
}


def main(ref_root):
    conv = os.path.join(ref_root, "portability_solved_cpp", "convert_boa_weights.py")
    for name, (ckpt, _, _, _) in TRAINED.items():
        src = os.path.join(ref_root, "experiments", "cms_experiment", ckpt)
        out = os.path.join(HERE, f"trained_{name}.bin")
        subprocess.run([sys.executable, conv, "--model", src, "--output", out], check=True,
                       stdout=subprocess.DEVNULL)
        print(out, os.path.getsize(out))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/convert_trained.py <reference root>")
    main(sys.argv[1])
