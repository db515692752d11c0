"""Probe heads on the GPU (nd_batch_embed, nd_batch_confidence) against
the oracle (crates/needle-engine/src/heads.rs): the cells of every position
and depth recorded during the forward, the probe pool, the projection and
the unit norm, bit for bit, for several sequences of one batch."""

import numpy as np
import pytest

from conftest import SMALL, _cached_archive

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def heads(cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    data = _cached_archive("small-heads", heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE), **SMALL)
    return nb.Model(data, cuda_device), orc.Model(data)


@pytest.mark.parametrize("T", [1, 7, 40])
def test_embedding(heads, T):
    g, o = heads
    rng = np.random.default_rng(T)
    S = 4
    ids = rng.integers(0, g.vocab, (S, T)).astype(np.int32)
    got = g.batch(S, T + 2).embed(ids)
    assert got.shape == (S, 128)
    for s in range(S):
        want = o.embed(ids[s].astype(np.uint32))
        assert np.array_equal(got[s].view(np.uint32), want.view(np.uint32)), (s, np.abs(got[s] - want).max())


@pytest.mark.parametrize("T", [3, 33])
def test_confidence(heads, T):
    g, o = heads
    rng = np.random.default_rng(100 + T)
    S = 3
    ids = rng.integers(0, g.vocab, (S, T)).astype(np.int32)
    got = g.batch(S, T).confidence(ids)
    for s in range(S):
        want = o.confidence(ids[s].astype(np.uint32))
        assert got[s].view(np.uint32) == np.float32(want).view(np.uint32), (s, got[s], want)


def test_embedding_from_the_confidence_pool(cuda_device):
    """Without an embedding head the confidence head's pool, unit norm."""
    import needle_b200 as nb
    from oracle import oracle as orc

    data = _cached_archive("small-conf", heads=(nb.HEAD_CONFIDENCE,), **SMALL)
    g, o = nb.Model(data, cuda_device), orc.Model(data)
    ids = (np.arange(2 * 9).reshape(2, 9) * 53 % g.vocab).astype(np.int32)
    got = g.batch(2, 9).embed(ids)
    assert got.shape == (2, 4 * 768)
    for s in range(2):
        want = o.embed(ids[s].astype(np.uint32))
        assert np.array_equal(got[s].view(np.uint32), want.view(np.uint32))


def test_errors(heads, small_archive, cuda_device):
    import needle_b200 as nb

    g, _ = heads
    b = g.batch(2, 16)
    b.forward(np.zeros((2, 3), np.int32))
    with pytest.raises(RuntimeError, match="fresh batch"):
        b.embed(np.zeros((2, 3), np.int32))
    plain = nb.Model(small_archive, cuda_device)
    with pytest.raises(RuntimeError, match="no probe head"):
        plain.batch(1, 8).embed(np.zeros((1, 3), np.int32))


def test_full_geometry_embedding_and_confidence(cuda_device):
    """Needle 3 geometry (20 layers, 21 depths): two texts of 45 tokens."""
    import needle_b200 as nb
    from oracle import oracle as orc

    data = _cached_archive("needle3-heads", seed=0, heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE))
    g, o = nb.Model(data, cuda_device), orc.Model(data)
    ids = np.random.default_rng(45).integers(0, g.vocab, (2, 45)).astype(np.int32)
    emb = g.batch(2, 45).embed(ids)
    conf = g.batch(2, 45).confidence(ids)
    for s in range(2):
        want = o.embed(ids[s].astype(np.uint32))
        assert np.array_equal(emb[s].view(np.uint32), want.view(np.uint32))
        assert conf[s].view(np.uint32) == np.float32(o.confidence(ids[s].astype(np.uint32))).view(np.uint32)
