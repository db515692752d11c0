"""The CQ/A8 matmul alone on the GPU (nd_cqmat_apply) against the oracle's
restatement of qlinear.rs, bit for bit: the decode combine (T = 1) through
the one-warp GEMV (1-4 rows) and the tensor-core tiles (5+ rows), and the
prefill combine with its block/remainder rule for the token counts the
reference's own kernel test uses (qlinear.rs:977-1029: T in 2, 3, 5, 9, 13,
17) plus full chunks and several sequences at once. Output widths include a
ragged one (100) so the last column tile is partial. Codes of 2 bits
(their own decode lane rule), 3 bits and ternary records run the same
cases as 4-bit ones (qlinear.rs:1009-1029)."""

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu


def _matrix(rng, out):
    codes = rng.integers(0, 256, (out, 6, 64), dtype=np.uint8)
    norms = np.abs(rng.standard_normal((out, 6)) * 0.02).astype(np.float16).view(np.uint16)
    return codes, norms


@pytest.fixture(scope="module")
def mats(cuda_device):
    import needle_b200 as nb

    rng = np.random.default_rng(77)
    out = {}
    for n in (100, 768):
        codes, norms = _matrix(rng, n)
        out[n] = (codes, norms, nb.CQMat(codes, norms, cuda_device))
    return out


CASES = [(1, 1), (3, 1), (4, 1), (5, 1), (64, 1), (200, 1),
         (2, 2), (3, 3), (5, 5), (9, 9), (13, 13), (17, 17), (32, 32), (64, 32), (96, 3)]


@pytest.mark.parametrize("n", [100, 768])
@pytest.mark.parametrize("M,T", CASES)
def test_cq_matmul_matches_oracle(mats, n, M, T):
    from oracle import oracle as orc

    codes, norms, mat = mats[n]
    rng = np.random.default_rng(1000 * M + T + n)
    x = rng.standard_normal((M, 768)).astype(np.float32)
    x[0] *= 1e-3  # one row far smaller, one far larger
    x[-1] *= 50.0
    got = mat(x, T=T)
    want = np.concatenate([orc.cq_matmul(codes.reshape(n, -1), norms, 768, x[s:s + T]) for s in range(0, M, T)])
    assert bits_equal(got, want), describe_diff(f"cq matmul M={M} T={T} n={n}", got, want)


@pytest.fixture(scope="module")
def width_mats(cuda_device):
    import needle_b200 as nb

    rng = np.random.default_rng(78)
    out = {}
    for bits in (2, 3, 5):
        width = nb.code_width(bits)
        for n in (100, 768):
            codes = rng.integers(0, 256, (n, 6 * 16 * width), dtype=np.uint8)
            norms = np.abs(rng.standard_normal((n, 6)) * 0.02).astype(np.float16).view(np.uint16)
            out[bits, n] = (codes, norms, nb.CQMat(codes, norms, cuda_device, bits=bits))
    return out


WIDTH_CASES = [(1, 1), (2, 1), (4, 1), (5, 1), (200, 1), (3, 3), (5, 5), (17, 17), (64, 32)]


@pytest.mark.parametrize("bits", [2, 3, 5])
@pytest.mark.parametrize("n", [100, 768])
@pytest.mark.parametrize("M,T", WIDTH_CASES)
def test_cq_matmul_widths_match_oracle(width_mats, bits, n, M, T):
    from oracle import oracle as orc

    codes, norms, mat = width_mats[bits, n]
    rng = np.random.default_rng(2000 * M + T + n + bits)
    x = rng.standard_normal((M, 768)).astype(np.float32)
    x[-1] *= 30.0
    got = mat(x, T=T)
    want = np.concatenate([orc.cq_matmul(codes, norms, 768, x[s:s + T], bits=bits) for s in range(0, M, T)])
    assert bits_equal(got, want), describe_diff(f"cq matmul bits={bits} M={M} T={T} n={n}", got, want)


@pytest.fixture(scope="module")
def model_shapes(cuda_device):
    """The model's matrix shapes: q|k|v|gate (1568), engram key|value (1536)
    and the tied lm_head (16384), 768 inputs each."""
    import needle_b200 as nb

    rng = np.random.default_rng(79)
    out = {}
    for n in (1568, 1536, 16384):
        codes, norms = _matrix(rng, n)
        out[n] = (codes, norms, nb.CQMat(codes, norms, cuda_device))
    return out


@pytest.mark.parametrize("n", [1568, 1536, 16384])
@pytest.mark.parametrize("M,T", [(2048, 1), (2048, 32), (2046, 31), (1, 1), (16, 1), (128, 32)])
def test_cq_matmul_model_shapes(model_shapes, n, M, T):
    """The matmul sweep's sizes (M in 1, 16, 128, 2048)
    at the model's real output widths, both combines: M = 2048 as 2048
    decode rows, as 64 prefill chunks of 32, and as 66 chunks of 31 (three
    remainder rows each). The oracle checks a sample of whole sequences
    (rows are independent across sequences): the first, the last and three
    between."""
    from oracle import oracle as orc

    codes, norms, mat = model_shapes[n]
    rng = np.random.default_rng(3000 + M + T + n)
    x = rng.standard_normal((M, 768)).astype(np.float32)
    x[0] *= 1e-3
    x[-1] *= 50.0
    got = mat(x, T=T)
    nseq = M // T
    picks = sorted({0, nseq - 1, *rng.choice(nseq, min(3, nseq), replace=False).tolist()})
    if T == 1:
        picks = sorted(set(picks) | set(range(min(8, M))))
    for s in picks:
        rows = slice(s * T, (s + 1) * T)
        want = orc.cq_matmul(codes.reshape(n, -1), norms, 768, x[rows])
        assert bits_equal(got[rows], want), describe_diff(f"cq matmul n={n} M={M} T={T} seq {s}", got[rows], want)
