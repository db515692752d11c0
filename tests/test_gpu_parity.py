"""GPU parity: the CUDA engine (through the C ABI) against the CPU oracle on
the same archive and ids. Logits and hidden states must agree bit for bit,
and greedy token streams exactly."""

import os

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff, first_divergence

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small(small_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(small_archive, cuda_device), orc.Model(small_archive)


@pytest.fixture(scope="module")
def full(full_archive, cuda_device):
    import needle_b200 as nb
    from oracle import oracle as orc

    return nb.Model(full_archive, cuda_device), orc.Model(full_archive)


def test_head_logits_decode_combine(small):
    g, o = small
    rng = np.random.default_rng(1)
    b = g.batch(1, 64)
    for scale in (1.0, 1e-3, 40.0):
        h = (rng.standard_normal((3, g.d_model)) * scale).astype(np.float32)
        got = b.head_logits(h)
        for r in range(3):
            want = o.head_logits(h[r])
            assert bits_equal(got[r], want), describe_diff("head_logits", got[r], want)


@pytest.mark.parametrize("rows", [5, 128, 200])
def test_head_logits_many_rows(small, rows):
    """The decode combine at batch sizes past the one-warp GEMV (tensor-core
    tiles, the last one partial)."""
    g, o = small
    rng = np.random.default_rng(100 + rows)
    b = g.batch(8, 64)
    h = (rng.standard_normal((rows, g.d_model)) * 3.0).astype(np.float32)
    got = b.head_logits(h)
    for r in range(rows):
        want = o.head_logits(h[r])
        assert bits_equal(got[r], want), f"row {r}: " + describe_diff("head_logits", got[r], want)


def test_head_logits_sparse_single_row(small):
    g, o = small
    rng = np.random.default_rng(2)
    b = g.batch(1, 64)
    h = rng.standard_normal(g.d_model).astype(np.float32)
    ids = rng.choice(g.out_rows, 37, replace=False).astype(np.int32)
    got = b.head_logits_sparse(h, ids)
    want = o.head_logits_sparse(h, ids.astype(np.uint32))
    assert bits_equal(got, want), describe_diff("sparse", got, want)


@pytest.mark.parametrize("t", [1, 2, 5, 13, 32])
def test_single_chunk(small, t):
    g, o = small
    rng = np.random.default_rng(10 + t)
    ids = rng.integers(0, g.vocab, t).astype(np.int32)
    b = g.batch(1, 64)
    got = b.forward(ids.reshape(1, t))[0, 0]
    want = o.session().forward(ids.astype(np.uint32))[0]
    if not bits_equal(got, want):
        pytest.fail(describe_diff("logits", got, want) + "\n" + first_divergence(g, o, ids))


def test_chunks_then_decode(small):
    """A 70-token feed (chunks 32, 32, 6: the last uses the remainder rule),
    then 12 decode steps with the RoPE recurrence, the sliding window
    (24 positions) and the engram history across chunk boundaries."""
    g, o = small
    rng = np.random.default_rng(3)
    ids = rng.integers(0, g.vocab, 70).astype(np.int32)
    b = g.batch(1, 128)
    s = o.session()
    got = b.forward(ids.reshape(1, -1))[0, 0]
    want = s.forward(ids.astype(np.uint32))[0]
    assert bits_equal(got, want), describe_diff("prefill logits", got, want)
    for k in range(12):
        nxt = int(np.argmax(want))
        got = b.forward(np.array([[nxt]], np.int32))[0, 0]
        want = s.forward(np.array([nxt], np.uint32))[0]
        assert bits_equal(got, want), f"step {k}: " + describe_diff("decode logits", got, want)


def test_long_context_key_chunks(small):
    """A 300-token feed in two sequences, then 6 decode steps: the global
    layer's rows pass 256 keys, so prefill rows split their keys into two
    chunks and decode rows into four (key_chunks' rule for one-token steps),
    and the per-chunk parts are merged; logits bit for bit every step."""
    g, o = small
    rng = np.random.default_rng(11)
    S, n, steps = 2, 300, 6
    ids = rng.integers(0, g.vocab, (S, n)).astype(np.int32)
    b = g.batch(S, n + steps + 1)
    sess = [o.session() for _ in range(S)]
    got = b.forward(ids)[:, 0]
    want = [sess[s_].forward(ids[s_].astype(np.uint32))[0] for s_ in range(S)]
    for s_ in range(S):
        assert bits_equal(got[s_], want[s_]), describe_diff(f"prefill seq {s_}", got[s_], want[s_])
    for k in range(steps):
        nxt = np.array([[int(np.argmax(want[s_]))] for s_ in range(S)], np.int32)
        got = b.forward(nxt)[:, 0]
        want = [sess[s_].forward(nxt[s_].astype(np.uint32))[0] for s_ in range(S)]
        for s_ in range(S):
            assert bits_equal(got[s_], want[s_]), f"step {k}: " + describe_diff(f"decode seq {s_}", got[s_], want[s_])


def test_all_logits_and_hidden(small):
    g, o = small
    from oracle import oracle as orc
    import needle_b200 as nb

    rng = np.random.default_rng(4)
    ids = rng.integers(0, g.vocab, 11).astype(np.int32)
    b = g.batch(1, 64)
    s = o.session()
    got = b.forward(ids[:6].reshape(1, -1), nb.OUT_ALL_LOGITS)[0]
    want = s.forward(ids[:6].astype(np.uint32), orc.OUT_ALL_LOGITS)
    assert bits_equal(got, want), describe_diff("all logits", got, want)
    got = b.forward(ids[6:].reshape(1, -1), nb.OUT_HIDDEN)[0]
    want = s.forward(ids[6:].astype(np.uint32), orc.OUT_HIDDEN)
    assert bits_equal(got, want), describe_diff("hidden", got, want)
    assert bits_equal(b.last_hidden()[0], s.last_hidden())


def test_batched_sequences_match_single(small):
    """Eight sequences fed in one batch equal eight separate oracle sessions,
    through a 37-token prefill and 6 masked greedy steps."""
    g, o = small
    rng = np.random.default_rng(5)
    S, n, steps = 8, 37, 6
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


@pytest.mark.parametrize("S", [144, 201, 301, 600])
def test_batched_decode_many_sequences(small, S):
    """S sequences in one batch (matmul tiles of 64 rows, the last partial)
    equal S separate oracle sessions through a 9-token prefill and 4 masked
    greedy steps. At 144 the decode steps take the one-row post block and
    the one-unit-a-warp conv; at 201 the two-row post block and at 301 the
    four-row one (each with a last CTA of one row); at 600 the seven-row
    post block and the two-units-a-warp conv, as the bench's 1024 do."""
    g, o = small
    rng = np.random.default_rng(6)
    n, steps = 9, 4
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


def test_committed_streams(small):
    """The GPU reproduces the committed oracle streams (tests/golden)."""
    import hashlib
    import json
    import os

    g, _ = small
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "small_model_streams.json")
    gold = json.load(open(path))
    for case in gold["cases"]:
        prompt = np.array(case["prompt"], np.int32).reshape(1, -1)
        b = g.batch(1, prompt.shape[1] + len(case["tokens"]) + 1)
        first = b.forward(prompt)[0, 0]
        assert hashlib.sha256(first.view(np.uint32).tobytes()).hexdigest() == case["first_logits_sha256"]
        toks = [int(b.step()[0]) for _ in case["tokens"]]
        assert toks == case["tokens"]


def test_full_model_greedy_stream(full):
    """Needle 3 geometry: a 118-token prompt (chunks 32, 32, 32, 22) and 45
    greedy decode steps, token-identical to the oracle; first logits bit-exact."""
    g, o = full
    rng = np.random.default_rng(118)
    S, n, steps = 2, 118, 45
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


def _oracle_streams(o, prompts, steps, masks=None):
    """Greedy (optionally masked) streams and first logits of the oracle for
    each prompt, one host thread per sequence."""
    from concurrent.futures import ThreadPoolExecutor

    def one(s_):
        m = masks[:, s_] if masks is not None else None
        return o.generate(prompts[s_].astype(np.uint32), steps, masks=m, want_logits=True)

    with ThreadPoolExecutor(max_workers=min(len(prompts), os.cpu_count() or 1)) as ex:
        return list(ex.map(one, range(len(prompts))))


def test_full_model_prefill_700(full):
    """BASELINE configs[3]'s sequences at the Needle 3 geometry: three
    sequences of 700 tokens fed as 22 chunks (the last 28 tokens, all block
    rows), so the late prefill rows split their keys into three chunks
    (key_chunks, infer.rs:2093-2101: ceil(700 / 256) = 3, 240 keys each);
    last-position logits bit for bit, then four greedy decode steps whose
    rows take four key chunks of up to 704 keys (every layer global or
    windowed, the band of 1024 not cutting), tokens and logits exact."""
    g, o = full
    rng = np.random.default_rng(700)
    S, n, steps = 3, 700, 4
    prompts = rng.integers(0, g.vocab, (S, n)).astype(np.int32)
    b = g.batch(S, n + steps + 1)
    first = b.forward(prompts)[:, 0]
    got = np.zeros((S, steps), np.int64)
    for k in range(steps):
        got[:, k] = b.step()
    for s_, (want, logits) in enumerate(_oracle_streams(o, prompts, steps)):
        assert bits_equal(first[s_], logits), describe_diff(f"seq {s_} logits after 700 tokens", first[s_], logits)
        assert list(got[s_]) == list(want), f"sequence {s_}: {got[s_]} vs {want}"


def test_headline_batch_sampled_streams(full):
    """BASELINE configs[4] as the bench runs it: 1024 sequences in one batch
    at the Needle 3 geometry, the bench's own 118-token prompts and seeded
    masks (bench.make_inputs), 45 masked greedy steps (graph-replayed). A
    sample of 24 sequences spread over the batch (both ends, every matmul
    row tile) must give the oracle's token streams exactly."""
    import bench

    g, o = full
    S, steps = 1024, 45
    prompts, masks = bench.make_inputs(0, S, steps, g.out_rows)
    b = g.batch(S, bench.PROMPT + steps + 1)
    first = b.forward(prompts)[:, 0]
    got = np.zeros((S, steps), np.int64)
    for k in range(steps):
        got[:, k] = b.step(masks[k])
    sample = np.unique(np.concatenate([[0, 1, 63, 64, 511, 512, 1022, 1023],
                                       np.random.default_rng(45).choice(S, 16, replace=False)]))
    want = _oracle_streams(o, prompts[sample], steps, masks=masks[:, sample])
    for i, s_ in enumerate(sample):
        toks, logits = want[i]
        assert bits_equal(first[s_], logits), describe_diff(f"seq {s_} prompt logits", first[s_], logits)
        assert list(got[s_]) == list(toks), f"sequence {s_}: {got[s_]} vs {toks}"
