"""Writes tests/golden/cdf_edge_rows.npz: logits rows on which the reference's
integer-CDF rule (Q_k = k + floor(C_k * (2^24 - 256)) after its lane-boundary
fix-up) is not strictly increasing, i.e. gives a symbol an empty interval.

They are rows 54 and 698 of the logits of the trained mambav1 d64 L2 model
(tests/golden/trained_mamba_d64L2.bin) on bytes 0..1023 of chunk 1543 (4 KiB
chunks) of particle_stream(16384 * 4096, seed 1): near-certain predictions
(top probability 0.99995) after which the running CDF reaches 1.0 before the
last lanes.  Generated on a GPU with this repository's library (the rows are
test INPUTS; the expected behaviour -- a strictly increasing Q -- needs no
stored output):

    python tests/golden/make_cdf_edge.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main():
    import __graft_entry__ as g
    boa = g.load_package()
    m = boa.Model(os.path.join(ROOT, "tests", "golden", "trained_mamba_d64L2.bin"), "mamba", 64, 2)
    S = 4096
    data = boa.synth.particle_stream(1544 * S, 1)
    tok = np.frombuffer(data[1543 * S:1543 * S + 1024], np.uint8).reshape(1, 1024)
    lg = m.logits(tok, 0)[0]
    rows = np.stack([lg[54], lg[698]])
    np.savez_compressed(os.path.join(ROOT, "tests", "golden", "cdf_edge_rows.npz"), logits=rows,
                        tokens=tok[0, :1024], next_bytes=np.array([tok[0, 55], tok[0, 699]], np.uint8))
    print(rows.shape)


if __name__ == "__main__":
    main()
