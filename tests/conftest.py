import hashlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "needle-rs_b200"))

CACHE = os.environ.get("NEEDLE_TEST_CACHE", "/tmp/needle_b200_test_cache")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _cached_archive(name, **shape):
    """A synthetic archive written by the oracle's writer (the engine's own
    writer is checked against it byte for byte in test_archive_writer.py),
    cached on disk per process host (the writer is deterministic)."""
    from oracle import oracle as orc

    key = hashlib.sha1(repr(sorted((k, repr(v)) for k, v in shape.items())).encode()).hexdigest()[:12]
    path = os.path.join(CACHE, f"{name}-{key}-oracle.cact")
    if not os.path.exists(path):
        os.makedirs(CACHE, exist_ok=True)
        data = orc.synth_cact(**shape)
        tmp = path + f".{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    with open(path, "rb") as f:
        return f.read()


# A three-layer model with a global layer, two engram sites, a short sliding
# window (so windowing is exercised at test lengths) and a small vocab.
SMALL = dict(num_layers=3, vocab=1024, engram_slots=96, sliding_window=24, global_layers=(1,), engram_sites=(0, 2),
             seed=7)
FULL = dict(seed=0)


# Mixed code widths (record bits per CQ role; 5 = ternary): fused parts
# share a width, ternary and 2-bit parts mix within q|k|v|gate, and every
# width appears in a matmul, a dequantized row (embedding, engram table)
# and the mHC rows.
MIXED_BITS = dict(embedding=2, q=5, k=2, v=5, gate=2, out=3, phi_pre=5, phi_post=3, phi_res=2, table=5, key=3,
                  value=3)


@pytest.fixture(scope="session")
def small_archive():
    return _cached_archive("small", **SMALL)


@pytest.fixture(scope="session")
def mixed_archive():
    return _cached_archive("small-mixed", bits=MIXED_BITS, **SMALL)


@pytest.fixture(scope="session")
def full_archive():
    return _cached_archive("needle3", **FULL)


def gpu_available():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda_device():
    if not gpu_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    return 0
