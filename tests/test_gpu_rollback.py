"""Session::rollback, rewind_zeroed and truncate on the GPU (crates/
needle-engine/src/model.rs:81-145, infer.rs:1039-1077) against the oracle
doing the same operations: logits bit for bit after each, through prefill
chunks, one-token feeds and graph-replayed decode steps, with and without
an attention span; and the refusal when a rollback would leave a kept
position's ring slot to a dropped one."""

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(small_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(small_archive, cuda_device), orc.Model(small_archive)


class Pair:
    """A GPU batch of S sequences and S oracle sessions driven alike."""

    def __init__(self, g, o, S, cap, attend=None):
        self.b = g.batch(S, cap)
        self.ss = [o.session() for _ in range(S)]
        if attend:
            self.b.set_attend(*attend)
            for s in self.ss:
                s.set_attend(*attend)

    def feed(self, ids, what):
        got = self.b.forward(ids)[:, 0]
        for k, s in enumerate(self.ss):
            want = s.forward(ids[k].astype(np.uint32))[0]
            assert bits_equal(got[k], want), describe_diff(f"{what} seq {k}", got[k], want)
        return got

    def steps(self, n, what):
        """Greedy steps (graph replays) checked against the oracle."""
        want = [None] * len(self.ss)
        for i in range(n):
            nxt = self.b.step()
            for k, s in enumerate(self.ss):
                want[k] = s.forward(np.array([nxt[k]], np.uint32))[0]
        got = self.b.head_logits(self.b.last_hidden())
        for k in range(len(self.ss)):
            assert bits_equal(got[k], want[k]), describe_diff(f"{what} seq {k}", got[k], want[k])

    def op(self, name, arg):
        getattr(self.b, name)(arg)
        for s in self.ss:
            getattr(s, name)(arg)
        assert len(self.b) == len(self.ss[0])


@pytest.mark.parametrize("attend", [None, (5, 60)])
def test_rollback_then_feed_and_step(small, attend):
    g, o = small
    rng = np.random.default_rng(11)
    S = 2
    ids = rng.integers(0, g.vocab, (S, 60)).astype(np.int32)
    p = Pair(g, o, S, 96, attend)
    p.feed(ids[:, :33], "prefill")
    p.feed(ids[:, 33:40], "chunk")
    p.steps(6, "steps")
    p.op("rollback", 6)
    p.feed(ids[:, 50:51], "one token after rollback")
    p.steps(3, "steps after rollback")
    p.op("rollback", 20)
    p.feed(ids[:, 40:47], "chunk after rollback")
    p.feed(ids[:, 47:48], "one token")
    p.steps(2, "steps")


def test_rewind_zeroed_and_truncate(small):
    g, o = small
    rng = np.random.default_rng(12)
    S = 2
    ids = rng.integers(0, g.vocab, (S, 80)).astype(np.int32)
    p = Pair(g, o, S, 96)
    p.feed(ids[:, :50], "prefill")
    p.op("rewind_zeroed", 30)
    p.feed(ids[:, 30:40], "after rewind")
    p.steps(3, "steps after rewind")
    p.op("rollback", 5)
    p.feed(ids[:, 40:45], "after rollback below the rewind")
    p.op("truncate", 12)
    p.feed(ids[:, 12:15], "after truncate")
    p.steps(2, "steps after truncate")


def test_rollback_across_the_ring_is_refused(small):
    """Positions 40-45 of a (5, 40) span take the ring slots of 0-5's
    successors 5 on: dropping them would leave position 5's slot to 45."""
    g, _ = small
    b = g.batch(1, 64)
    b.set_attend(5, 40)
    b.forward((np.arange(41) * 7 % g.vocab).astype(np.int32).reshape(1, -1))
    for _ in range(5):
        b.step()  # graph replays mark their slots too
    with pytest.raises(RuntimeError, match="ring slots"):
        b.rollback(6)
    assert len(b) == 46
    b.rollback(0)
    b.rollback(0)
    with pytest.raises(RuntimeError, match="exceeds 32"):
        b.rollback(33)
