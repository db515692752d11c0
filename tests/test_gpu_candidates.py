"""The call sampler's start on the GPU (nd_batch_candidates) against the
oracle (agent.rs:295-343, 1130-1252): per sequence the softmax max and sum
bit for bit (f32 lanes, f64 total), the live count, and the first k
candidates in the reference's order (logit descending, lowest id first on
ties), over the engine's own logits and over crafted rows with ties, signed
zeros, masked logits, rows with fewer than k live, and a vocabulary that is
not a multiple of four (the f64 tail)."""

import numpy as np
import pytest

from conftest import SMALL

pytestmark = pytest.mark.gpu
f32 = np.float32


def expect(logits, allow, allow_order, k):
    from oracle import oracle as orc

    x = np.array(logits, np.float32, copy=True)
    V = len(x)
    if allow is not None:
        x[~np.unpackbits(allow, bitorder="little")[:V].astype(bool)] = f32(-1e30)
    m, z = orc.softmax_stats(x)
    if allow_order is not None:
        x[~np.unpackbits(allow_order, bitorder="little")[:V].astype(bool)] = f32(-1e30)
    ids, live = orc.candidate_order(x, k)
    return m, z, ids, live


def check(got, logits, allow, allow_order, k):
    ids, m, z, live = got
    for s in range(len(logits)):
        wm, wz, wids, wlive = expect(logits[s], None if allow is None else allow[s],
                                     None if allow_order is None else allow_order[s], k)
        assert m[s].view(np.uint32) == f32(wm).view(np.uint32), (s, m[s], wm)
        assert z[s] == wz, (s, z[s], wz)
        assert live[s] == wlive, (s, live[s], wlive)
        n = min(k, wlive)
        assert list(ids[s][:n]) == list(wids), s
        assert (ids[s][n:] == -1).all(), s


def random_masks(rng, S, V, p):
    return np.stack([np.packbits(rng.random(V) >= p, bitorder="little") for _ in range(S)])


@pytest.fixture(scope="module")
def small(small_archive, cuda_device):
    import needle_b200 as nb

    return nb.Model(small_archive, cuda_device)


def test_engine_logits(small):
    """After a prefill of eight sequences: the batch's own last logits."""
    import needle_b200 as nb

    rng = np.random.default_rng(5)
    S = 8
    b = small.batch(S, 64)
    logits = b.forward(rng.integers(0, small.vocab, (S, 21)).astype(np.int32), nb.OUT_LAST_LOGITS)[:, 0]
    V = small.out_rows
    allow = random_masks(rng, S, V, 0.1)
    order = random_masks(rng, S, V, 0.2)
    for k in (128, 1, 37):
        check(b.candidates(allow, order, k), logits, allow, order, k)
    check(b.candidates(None, None, 128), logits, None, None, 128)


def test_crafted_rows(small):
    rng = np.random.default_rng(6)
    S, V = 6, small.out_rows
    b = small.batch(S, 64)
    x = np.round(rng.standard_normal((S, V)) * 2, 1).astype(np.float32)  # many exact ties
    x[1, :] = 0.0
    x[1, ::3] = -0.0  # signed zeros tie
    x[2, 100:] = f32(-1e30)  # fewer than k live
    x[3, :] = f32(-1e30)  # nothing live
    x[4, 7] = f32(30.0)
    allow = random_masks(rng, S, V, 0.05)
    allow[5] = 0  # every entry banned
    check(b.candidates(allow, None, 128, logits=x), x, allow, None, 128)
    check(b.candidates(None, allow, 128, logits=x), x, None, allow, 128)


def test_ragged_vocab_tail(cuda_device):
    """out_rows = 1021: the last group of one is the f64 tail."""
    import needle_b200 as nb

    shape = dict(SMALL)
    shape.update(vocab=1021, num_layers=1, engram_sites=(0,), global_layers=())
    m = nb.Model(nb.synth_cact(**shape), cuda_device)
    assert m.out_rows == 1021
    rng = np.random.default_rng(7)
    S = 3
    b = m.batch(S, 32)
    x = (rng.standard_normal((S, 1021)) * 3).astype(np.float32)
    x[1, 1020] = f32(-1e30)
    allow = random_masks(rng, S, 1021, 0.3)
    check(b.candidates(allow, None, 128, logits=x), x, allow, None, 128)


def test_full_vocab_many_rows(cuda_device, full_archive):
    """1024 rows of the Needle 3 vocabulary (16384 logits each)."""
    import needle_b200 as nb

    m = nb.Model(full_archive, cuda_device)
    rng = np.random.default_rng(8)
    S, V = 1024, m.out_rows
    b = m.batch(S, 8)
    x = (rng.standard_normal((S, V)) * 3).astype(np.float32)
    allow = random_masks(rng, S, V, 0.5)
    got = b.candidates(allow, None, 128, logits=x)
    pick = list(range(0, S, 97)) + [S - 1]
    check(tuple(a[pick] for a in got), x[pick], allow[pick], None, 128)
