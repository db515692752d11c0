"""A mixed-width archive (2-bit, 3-bit, ternary and 4-bit CQ records, fused
parts of 2-bit and ternary codes side by side) through the CUDA engine
against the CPU oracle: logits and hidden states bit for bit, greedy token
streams exactly (qlinear.rs:220-265, 500-518)."""

import numpy as np
import pytest

from conftest import SMALL
from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mixed(mixed_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(mixed_archive, cuda_device), orc.Model(mixed_archive)


@pytest.mark.parametrize("rows", [1, 3, 5, 130])
def test_head_logits(mixed, rows):
    """The tied lm_head at 2 bits: the GEMV's 2-bit lanes (1-4 rows) and the
    tensor-core tiles' (5+ rows)."""
    g, o = mixed
    rng = np.random.default_rng(rows)
    b = g.batch(8, 64)
    h = (rng.standard_normal((rows, g.d_model)) * 2.0).astype(np.float32)
    got = b.head_logits(h)
    for r in range(rows):
        want = o.head_logits(h[r])
        assert bits_equal(got[r], want), f"row {r}: " + describe_diff("head_logits", got[r], want)


def test_head_logits_sparse(mixed):
    g, o = mixed
    rng = np.random.default_rng(9)
    b = g.batch(1, 64)
    h = rng.standard_normal(g.d_model).astype(np.float32)
    ids = rng.choice(g.out_rows, 29, replace=False).astype(np.int32)
    got = b.head_logits_sparse(h, ids)
    want = o.head_logits_sparse(h, ids.astype(np.uint32))
    assert bits_equal(got, want), describe_diff("sparse", got, want)


@pytest.mark.parametrize("t", [1, 6, 32])
def test_single_chunk(mixed, t):
    g, o = mixed
    rng = np.random.default_rng(20 + t)
    ids = rng.integers(0, g.vocab, t).astype(np.int32)
    b = g.batch(1, 64)
    got = b.forward(ids.reshape(1, t))[0, 0]
    want = o.session().forward(ids.astype(np.uint32))[0]
    assert bits_equal(got, want), describe_diff("logits", got, want)


def test_chunks_then_decode(mixed):
    g, o = mixed
    from oracle import oracle as orc
    import needle_b200 as nb

    rng = np.random.default_rng(31)
    ids = rng.integers(0, g.vocab, 45).astype(np.int32)
    b = g.batch(1, 96)
    s = o.session()
    got = b.forward(ids.reshape(1, -1))[0, 0]
    want = s.forward(ids.astype(np.uint32))[0]
    assert bits_equal(got, want), describe_diff("prefill logits", got, want)
    for k in range(10):
        nxt = int(np.argmax(want))
        got = b.forward(np.array([[nxt]], np.int32))[0, 0]
        want = s.forward(np.array([nxt], np.uint32))[0]
        assert bits_equal(got, want), f"step {k}: " + describe_diff("decode logits", got, want)
    got = b.forward(ids[:7].reshape(1, -1), nb.OUT_HIDDEN)[0]
    want = s.forward(ids[:7].astype(np.uint32), orc.OUT_HIDDEN)
    assert bits_equal(got, want), describe_diff("hidden", got, want)


def test_batched_decode(mixed):
    """72 sequences in lockstep (tensor-core tiles for every projection,
    2-bit decode lanes among them) through a 13-token prefill and 5 masked
    greedy steps."""
    g, o = mixed
    rng = np.random.default_rng(32)
    S, n, steps = 72, 13, 5
    prompts = rng.integers(0, g.vocab, (S, n)).astype(np.int32)
    mb = (g.out_rows + 7) // 8
    masks = np.zeros((S, steps, mb), np.uint8)
    for s_ in range(S):
        for k in range(steps):
            allow = rng.random(g.out_rows) < rng.uniform(0.05, 0.5)
            allow[rng.integers(0, g.out_rows)] = True
            masks[s_, k] = np.packbits(allow, bitorder="little")
    b = g.batch(S, n + steps + 1)
    b.forward(prompts)
    got = np.zeros((S, steps), np.int64)
    for k in range(steps):
        got[:, k] = b.step(masks[:, k])
    for s_ in range(S):
        want = o.generate(prompts[s_].astype(np.uint32), steps, masks=masks[s_])
        assert list(got[s_]) == list(want), f"sequence {s_}: {got[s_]} vs {want}"


def test_engine_refuses_mixed_widths_in_a_fused_projection(cuda_device):
    import needle_b200 as nb

    with pytest.raises(RuntimeError, match="code width"):
        nb.Model(nb.synth_cact(bits=dict(key=2, value=4), **SMALL), cuda_device)


def test_full_geometry_low_width_stream(cuda_device):
    """Needle 3 geometry with ternary attention projections, 2-bit out and
    engram projections and 3-bit engram tables: a 70-token prompt (chunks
    32, 32, 6) and 20 greedy steps, token-identical to the oracle; first
    logits bit-exact."""
    import needle_b200 as nb
    from oracle import oracle as orc
    from conftest import _cached_archive

    data = _cached_archive("needle3-low-width", seed=0, bits=dict(q=5, k=5, v=5, gate=5, out=2, key=2, value=2, table=3))
    g, o = nb.Model(data, cuda_device), orc.Model(data)
    rng = np.random.default_rng(70)
    S, n, steps = 2, 70, 20
    prompts = rng.integers(0, g.vocab, (S, n)).astype(np.int32)
    b = g.batch(S, n + steps + 1)
    first = b.forward(prompts)[:, 0]
    got = np.zeros((S, steps), np.int64)
    for k in range(steps):
        got[:, k] = b.step()
    for s_ in range(S):
        want, logits = o.generate(prompts[s_].astype(np.uint32), steps, want_logits=True)
        assert bits_equal(first[s_], logits), describe_diff("first logits", first[s_], logits)
        assert list(got[s_]) == list(want), f"sequence {s_}: {got[s_]} vs {want}"
