"""The call sampler's start (crates/needle-engine/src/agent.rs:295-343,
1130-1252) in the oracle against the pure-Python restatement: the engine's
f32 exp bit for bit, softmax_stats' four f32 lanes and f64 tail, and the
candidate order (logit descending, lowest id first on ties, masked logits
out). CPU only."""

import numpy as np
import pytest

import pyref

f32 = np.float32


def test_engine_expf_matches_restatement():
    from oracle import oracle as orc

    xs = np.concatenate([np.linspace(-100, 100, 2001, dtype=np.float32),
                         np.array([0.0, -0.0, -88.37626, 88.37626, -1e30, 1e-8, -1e-8], np.float32)])
    for x in xs:
        got = f32(orc.engine_expf(float(x)))
        want = pyref.engine_expf(x)
        assert got.view(np.uint32) == want.view(np.uint32), (x, got, want)
    assert abs(orc.engine_expf(1.0) / np.exp(1.0) - 1) < 1e-6


@pytest.mark.parametrize("n", [8, 13, 64, 101])
def test_softmax_stats_matches_restatement(n):
    from oracle import oracle as orc

    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    x[rng.random(n) < 0.2] = f32(-1e30)  # masked, inside the lanes and in the f64 tail
    m, z = orc.softmax_stats(x)
    wm, wz = pyref.softmax_stats(x)
    assert m == wm and z == wz, (m, z, wm, wz)


def test_candidate_order_ties_and_masks():
    from oracle import oracle as orc

    x = np.array([1.0, 3.0, 3.0, -1e30, 2.0, 0.0, -0.0, 3.0, -5.0, -1e30, 0.0], np.float32)
    for k in (1, 3, 5, 9, 20):
        got, live = orc.candidate_order(x, k)
        want, wlive = pyref.candidate_order(x, k)
        assert list(got) == want and live == wlive == 9
    got, _ = orc.candidate_order(x, 9)
    assert list(got) == [1, 2, 7, 4, 0, 5, 6, 10, 8]  # -0.0 and 0.0 tie: lower id first


def test_candidate_order_random():
    from oracle import oracle as orc

    rng = np.random.default_rng(3)
    x = np.round(rng.standard_normal(4000) * 3, 1).astype(np.float32)  # many exact ties
    x[rng.random(4000) < 0.3] = f32(-1e30)
    got, live = orc.candidate_order(x, 128)
    want, wlive = pyref.candidate_order(x, 128)
    assert list(got) == want and live == wlive


def test_max_keeps_positive_zero():
    """f32::max on the reference's platform (aarch64 FMAXNM) orders -0 below
    +0, so the max of signed zeros is +0 whatever their order."""
    from oracle import oracle as orc

    for x in ([-0.0, 0.0, -0.0, -0.0], [0.0, -0.0, -0.0, -0.0], [-0.0] * 4):
        m, _ = orc.softmax_stats(np.array(x, np.float32))
        wm, _ = pyref.softmax_stats(np.array(x, np.float32))
        assert np.signbit(m) == np.signbit(wm) == bool(np.all(np.signbit(x)))
