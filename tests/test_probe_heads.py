"""Probe-pooling heads (crates/needle-engine/src/heads.rs, linalg.rs) in
the oracle against the pure-Python restatement, and probe-head archives
(cact.rs:354-392, weights.rs:422-469) through the oracle. CPU only."""

import numpy as np
import pytest

import pyref
from conftest import SMALL

f32 = np.float32


def test_fast_exp_matches_restatement():
    from oracle import oracle as orc

    for x in np.concatenate([np.linspace(-90, 90, 1801, dtype=np.float32), np.array([0.0, -0.0, 0.5, -0.5, 2.5], np.float32)]):
        got = f32(orc.fast_exp(float(x)))
        want = pyref.fast_exp(x)
        assert got.view(np.uint32) == want.view(np.uint32), (x, got, want)


@pytest.mark.parametrize("n", [8, 13, 768])
def test_dot8_matches_restatement(n):
    from oracle import oracle as orc

    rng = np.random.default_rng(n)
    a = rng.standard_normal(n).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    assert orc.dot8(a, b).view(np.uint32) == pyref.dot8(a, b).view(np.uint32)


def test_probe_pool_matches_restatement():
    from oracle import oracle as orc

    rng = np.random.default_rng(4)
    t, l1, d, k, q = 5, 3, 24, 2, 2
    cells = rng.standard_normal((t, l1, d)).astype(np.float32)
    probes = rng.standard_normal((l1, k, d)).astype(np.float32)
    gain = (1 + 0.1 * rng.standard_normal((l1, k))).astype(np.float32)
    query = rng.standard_normal((q, d)).astype(np.float32)
    row_bias = rng.standard_normal((q, l1 * k)).astype(np.float32)
    got = orc.probe_pool(cells, probes, gain, query, row_bias)
    want = pyref.probe_pool(cells, probes, gain, query, row_bias)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_head_archives_load_and_embed():
    import needle_b200 as nb
    from oracle import oracle as orc

    ids = (np.arange(11) * 37 % 1000).astype(np.uint32)
    both = orc.Model(nb.synth_cact(heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE), **SMALL))
    e = both.embed(ids)
    assert e.shape == (128,) and abs(float(np.linalg.norm(e)) - 1) < 1e-5
    assert np.isfinite(both.confidence(ids))
    # without an embedding head the confidence head's pool is the embedding
    conf = orc.Model(nb.synth_cact(heads=(nb.HEAD_CONFIDENCE, nb.HEAD_ROUTER), **SMALL))
    assert conf.embed(ids).shape == (4 * 768,)
    plain = orc.Model(nb.synth_cact(**SMALL))
    with pytest.raises(RuntimeError, match="no probe head"):
        plain.embed(ids)
    # the cells: depth 0 is the embedding row's lane mean, every lane equal
    c = both.cells(ids)
    assert c.shape == (11, SMALL["num_layers"] + 1, 768)
