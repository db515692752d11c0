"""The GPU reproduces the committed records of the widened rows
(tests/golden/next_rows.json, written by the oracle): mixed-width greedy
streams and first-logit digests, the call sampler on fixed rows, and the
probe heads' embedding digests and confidence logits."""

import json
import os
import sys

import numpy as np
import pytest

from conftest import MIXED_BITS, SMALL, _cached_archive

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def gold():
    sys.path.insert(0, os.path.join(HERE, "golden"))
    return json.load(open(os.path.join(HERE, "golden", "next_rows.json")))


def digest(a):
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


def test_mixed_width_streams(gold, cuda_device):
    import needle_b200 as nb

    g = nb.Model(_cached_archive("small-mixed", bits=MIXED_BITS, **SMALL), cuda_device)
    for case in gold["mixed_width"]["cases"]:
        prompt = np.array(case["prompt"], np.int32).reshape(1, -1)
        b = g.batch(1, prompt.shape[1] + len(case["tokens"]) + 1)
        first = b.forward(prompt)[0, 0]
        assert digest(first) == case["first_logits_sha256"]
        assert [int(b.step()[0]) for _ in case["tokens"]] == case["tokens"]


def test_call_sampler_rows(gold, cuda_device):
    import needle_b200 as nb
    from make_golden import call_sampler_logits

    x = call_sampler_logits()
    assert digest(x) == gold["call_sampler"]["logits_sha256"]
    shape = dict(SMALL)
    shape.update(vocab=x.shape[1], num_layers=1, engram_sites=(0,), global_layers=())
    m = nb.Model(nb.synth_cact(**shape), cuda_device)
    ids, mo, z, live = m.batch(len(x), 8).candidates(logits=x)
    for r, row in enumerate(gold["call_sampler"]["rows"]):
        assert float(mo[r]) == row["m"] and float(z[r]) == row["z"] and int(live[r]) == row["live"]
        assert [int(v) for v in ids[r][:len(row["ids"])]] == row["ids"]


def test_probe_heads(gold, cuda_device):
    import needle_b200 as nb

    g = nb.Model(_cached_archive("small-heads", heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE), **SMALL), cuda_device)
    for t in gold["probe_heads"]["texts"]:
        ids = np.array(t["ids"], np.int32).reshape(1, -1)
        assert digest(g.batch(1, ids.shape[1]).embed(ids)[0]) == t["embedding_sha256"]
        assert float(g.batch(1, ids.shape[1]).confidence(ids)[0]) == t["confidence"]
