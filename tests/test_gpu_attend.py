"""The agent's attention span (Session::attend, crates/needle-engine/src/
model.rs:63-66, infer.rs:1749-1825) on the GPU against the oracle: with
(sink, ring) set, each query sees the sink within its layer's band and the
ring as of its chunk's end, which the band does not cut. Logits bit for bit
through prefill chunks and graph-replayed decode steps, on the small
archive whose 24-position band makes both runs matter."""

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(small_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(small_archive, cuda_device), orc.Model(small_archive)


@pytest.mark.parametrize("sink,ring,n", [(5, 20, 70), (9, 40, 70), (0, 16, 70), (50, 30, 70), (40, 260, 320)])
def test_span_prefill_and_decode(small, sink, ring, n):
    """The last case passes 256 keys in the global layer: key chunks that
    hold the end of the sink run and the start of the ring run together."""
    g, o = small
    rng = np.random.default_rng(sink * 100 + ring)
    S, steps = 3, 10
    prompts = rng.integers(0, g.vocab, (S, n)).astype(np.int32)
    b = g.batch(S, n + steps + 1)
    b.set_attend(sink, ring)
    sessions = []
    for s_ in range(S):
        ss = o.session()
        ss.set_attend(sink, ring)
        sessions.append(ss)
    got = b.forward(prompts)[:, 0]
    want = [sessions[s_].forward(prompts[s_].astype(np.uint32))[0] for s_ in range(S)]
    for s_ in range(S):
        assert bits_equal(got[s_], want[s_]), describe_diff(f"prefill seq {s_}", got[s_], want[s_])
    for k in range(steps):
        nxt = b.step()
        for s_ in range(S):
            assert int(nxt[s_]) == int(np.argmax(want[s_])), (k, s_)
        want = [sessions[s_].forward(np.array([nxt[s_]], np.uint32))[0] for s_ in range(S)]
    # the logits after the last step
    last = b.head_logits(b.last_hidden())
    for s_ in range(S):
        assert bits_equal(last[s_], want[s_]), describe_diff(f"decode seq {s_}", last[s_], want[s_])


def test_span_off_again_matches_plain(small):
    """ring 0 restores plain attention: the same stream as a batch that never
    set a span."""
    g, _ = small
    ids = (np.arange(2 * 40).reshape(2, 40) * 37 % g.vocab).astype(np.int32)
    a = g.batch(2, 48)
    a.set_attend(4, 10)
    a.set_attend(0, 0)
    b = g.batch(2, 48)
    assert bits_equal(a.forward(ids)[:, 0], b.forward(ids)[:, 0])
