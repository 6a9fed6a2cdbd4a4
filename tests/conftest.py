"""Shared fixtures.  GPU tests carry @pytest.mark.gpu and run only on a B200
box; everything else runs on CPU (the oracle, the container and the C ABI's
host-side checks)."""
import importlib.util
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_package():
    if "boa_b200" in sys.modules:
        return sys.modules["boa_b200"]
    pkg = os.path.join(ROOT, "boa-constrictor_b200")
    spec = importlib.util.spec_from_file_location("boa_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["boa_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def boa():
    mod = load_package()
    if not os.path.exists(mod.LIB_PATH):
        mod.build()
    return mod


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def boa2():
    import boa2 as B2
    return B2


@pytest.fixture(scope="session")
def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def golden_mod():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="session")
def wdir(tmp_path_factory):
    return tmp_path_factory.mktemp("weights")


@pytest.fixture(scope="session")
def weights(boa, wdir):
    """Factory: path of a random-init weight file (cached per config)."""
    cache = {}

    def make(backbone="mamba", d=256, L=8, seed=0, std=0.02):
        key = (backbone, d, L, seed, std)
        if key not in cache:
            p = str(wdir / f"w_{backbone}_{d}_{L}_{seed}_{std}.bin")
            boa.synth.write_random_weights(p, backbone, d, L, seed, std=std)
            cache[key] = p
        return cache[key]
    return make


def dirichlet_cdfs(rng, n_steps, n_streams, alpha=0.1):
    """configs[1]-style integer CDFs: Dirichlet(alpha) over 256 symbols,
    quantised with the reference rule Q_k = floor(C_k * (2^24 - 256)) + k,
    and a symbol sampled from each distribution."""
    p = rng.dirichlet(np.full(256, alpha), size=(n_steps, n_streams))
    c = np.concatenate([np.zeros(p.shape[:2] + (1,)), np.cumsum(p, -1)[..., :-1]], -1)
    Q = np.empty(p.shape[:2] + (257,), np.uint32)
    Q[..., :256] = (c * float((1 << 24) - 256)).astype(np.uint32) + np.arange(256, dtype=np.uint32)
    Q[..., 256] = 1 << 24
    u = rng.random(p.shape[:2] + (1,))
    syms = np.minimum((np.cumsum(p, -1) < u).sum(-1), 255).astype(np.uint8)
    return Q, syms


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
