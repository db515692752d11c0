"""The fused row ops alone on the GPU (BASELINE's fused-ops sweep, through the
C ABI: nd_op_zcn, nd_op_rope, nd_op_silu, nd_op_gather) against the
oracle's restatements of the reference, bit for bit, at the sweep's token
counts T in 1, 64, 1024, 8192 with its input distributions: rows N(0, 1),
RMSNorm weights N(1, 0.1) rounded to f16 (the archive stores f16), RoPE at
positions 0..T-1 with the config's theta, SiLU over the MLP's [T, 1024],
and the gather of uniform-random ids from the Needle 3 embedding. Extreme
rows (tiny, huge, zero) and SiLU's saturating tails are added."""

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu

TS = [1, 64, 1024, 8192]


def _dev(a, device):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{device}")


@pytest.mark.parametrize("T", TS + [7])
def test_zcn_matches_oracle(cuda_device, T):
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(T)
    x = rng.standard_normal((T, 768)).astype(np.float32)
    if T > 4:
        x[1] *= 1e-20
        x[2] *= 1e15
        x[3] = 0.0
    s = (1.0 + 0.1 * rng.standard_normal(768)).astype(np.float16).astype(np.float32)
    got = nb.op_zcn(_dev(x, cuda_device), _dev(s, cuda_device)).cpu().numpy()
    want = orc.op_zcn(x, s)
    assert bits_equal(got, want), describe_diff(f"zcn T={T}", got, want)


@pytest.mark.parametrize("T", TS + [4097])
def test_rope_matches_oracle(cuda_device, T):
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(100 + T)
    x = rng.standard_normal((T, 672)).astype(np.float32)
    got = nb.op_rope(_dev(x, cuda_device), 100000.0).cpu().numpy()
    want = orc.op_rope(x, 100000.0)
    assert bits_equal(got, want), describe_diff(f"rope T={T}", got, want)


@pytest.mark.parametrize("T", TS)
def test_silu_matches_oracle(cuda_device, T):
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(200 + T)
    x = rng.standard_normal((T, 1024)).astype(np.float32)
    if T > 1:
        x[0, :8] = [0.0, -0.0, 88.0, -88.0, 200.0, -200.0, 1e-30, -1e-30]
    got = nb.op_silu(_dev(x, cuda_device)).cpu().numpy()
    want = orc.op_silu(x)
    assert bits_equal(got, want), describe_diff(f"silu T={T}", got, want)


def test_silu_ragged_length(cuda_device):
    """A length that is not a multiple of four (the scalar tail)."""
    import needle_b200 as nb
    from oracle import oracle as orc

    x = np.random.default_rng(7).standard_normal(1027).astype(np.float32) * 5
    got = nb.op_silu(_dev(x, cuda_device)).cpu().numpy()
    assert bits_equal(got, orc.op_silu(x)), describe_diff("silu 1027", got, orc.op_silu(x))


@pytest.fixture(scope="module")
def models(full_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(full_archive, cuda_device), orc.Model(full_archive)


@pytest.mark.parametrize("T", TS)
def test_gather_matches_oracle(models, cuda_device, T):
    import needle_b200 as nb

    g, o = models
    rng = np.random.default_rng(300 + T)
    ids = rng.integers(0, g.vocab, T).astype(np.int32)
    if T > 2:
        ids[:2] = [0, g.vocab - 1]
    got = nb.op_gather(g, _dev(ids, cuda_device)).cpu().numpy()
    want = o.gather(ids.astype(np.uint32))
    assert bits_equal(got, want), describe_diff(f"gather T={T}", got, want)


def test_ops_refuse_bad_arguments(models, cuda_device):
    import torch

    import needle_b200 as nb

    g, _ = models
    x = torch.zeros((4, 768), device=f"cuda:{cuda_device}")
    lib = nb.lib()
    assert lib.nd_op_zcn(nb._p(x), nb._p(x), 0, nb._p(x), None) == -1
    assert lib.nd_op_zcn(x.data_ptr() + 4, nb._p(x), 1, nb._p(x), None) == -1
    assert b"16-byte aligned" in lib.nd_last_error()
    assert lib.nd_op_rope(nb._p(x), 1, -1.0, nb._p(x), None) == -1
    assert lib.nd_op_silu(nb._p(x), 0, nb._p(x), None) == -1
    # an id past the vocabulary reads as a row of zeros
    ids = torch.tensor([g.vocab, -1], dtype=torch.int32, device=f"cuda:{cuda_device}")
    out = nb.op_gather(g, ids).cpu().numpy()
    assert not out.any()
