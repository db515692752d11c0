"""Writes the committed fixtures under tests/golden/.

reference_kat.json: known answers transcribed from the reference's own unit
tests (file:line in needle-rs given per entry).

small_model_streams.json: the oracle's greedy token streams and a digest of
its first logits on the small synthetic archive the tests build
(tests/conftest.py SMALL), so a later change to the oracle, the archive
writer or the engine shows up against a fixed record.

next_rows.json: the same kind of record for the widened rows: greedy
streams on the mixed-width small archive (conftest MIXED_BITS), the call
sampler's statistics and candidate order on fixed logits, and the probe
heads' embedding and confidence digests on the small archive with heads.

Run: python tests/golden/make_golden.py
"""

import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "needle-rs_b200"))
sys.path.insert(0, os.path.dirname(HERE))

import numpy as np  # noqa: E402

REFERENCE_KAT = {
    "mt19937_permutation": {
        "source": "crates/needle-core/src/rng.rs:94-98",
        "seed": 11, "n": 16, "expect": [8, 3, 6, 10, 15, 4, 5, 14, 2, 13, 12, 7, 1, 11, 0, 9],
    },
    "hada_blocks": {"source": "crates/needle-core/src/config.rs:495-499", "n": 1024, "expect": [32, 32]},
    "nearest_ties_low": {
        "source": "crates/needle-core/src/quant.rs:314-321",
        "codebook": [-1.0, 0.0, 1.0],
        "cases": [[0.5, 1], [-0.5, 0], [5.0, 2], [-5.0, 0]],
    },
    "nexp_tolerance": {"source": "crates/needle-engine/src/infer.rs:3078-3084", "rel": 2e-7, "x": "i * 0.37, i in -200..200"},
    "kernels_match_reference": {
        "source": "crates/needle-engine/src/qlinear.rs:976-1006",
        "out": 37, "in": 384, "tolerance": "0.02 * (1 + |want|)", "prefill_rows": [2, 3, 5, 9, 13, 17],
    },
    "kv_window_default": {"source": "crates/needle-core/src/config.rs:448-482", "expect": 3456},
    "two_bit_kernels_match_reference": {
        "source": "crates/needle-engine/src/qlinear.rs:1008-1033",
        "out": 9, "in": 256, "code_byte": "(i * 37) % 251 over out * in / 4 bytes",
        "norm": "f16(0.5 + 0.01 * i) over out * groups", "x": "cos(0.21 * i) over 5 * in", "block_rows": 4,
    },
}


def streams():
    from conftest import SMALL, _cached_archive
    from oracle import oracle as orc

    data = _cached_archive("small", **SMALL)
    m = orc.Model(data)
    out = {"archive_sha256": hashlib.sha256(data).hexdigest(), "shape": {k: list(v) if isinstance(v, tuple) else v
                                                                        for k, v in SMALL.items()}, "cases": []}
    rng = np.random.default_rng(2024)
    for n in (5, 33, 70):
        prompt = rng.integers(0, m.vocab, n).astype(np.uint32)
        toks, logits = m.generate(prompt, 12, want_logits=True)
        out["cases"].append({
            "prompt": [int(v) for v in prompt],
            "tokens": [int(v) for v in toks],
            "first_logits_sha256": hashlib.sha256(logits.view(np.uint32).tobytes()).hexdigest(),
        })
    return out


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


def call_sampler_logits():
    """Four rows of 1000 logits rounded to 0.1 (many exact ties), every
    seventh of row 1 banned (-1e30)."""
    x = np.round(np.random.default_rng(7070).standard_normal((4, 1000)) * 3, 1).astype(np.float32)
    x[1, ::7] = np.float32(-1e30)
    return x


def next_rows():
    import needle_b200 as nb
    from conftest import MIXED_BITS, SMALL, _cached_archive
    from oracle import oracle as orc

    out = {}
    mixed = _cached_archive("small-mixed", bits=MIXED_BITS, **SMALL)
    m = orc.Model(mixed)
    rng = np.random.default_rng(2025)
    cases = []
    for n in (7, 40):
        prompt = rng.integers(0, m.vocab, n).astype(np.uint32)
        toks, logits = m.generate(prompt, 10, want_logits=True)
        cases.append({"prompt": [int(v) for v in prompt], "tokens": [int(v) for v in toks],
                      "first_logits_sha256": digest(logits)})
    out["mixed_width"] = {"archive_sha256": hashlib.sha256(mixed).hexdigest(), "bits": MIXED_BITS, "cases": cases}
    # the call sampler on fixed rows: logits rounded to 0.1 (many ties)
    x = call_sampler_logits()
    rows = []
    for r in range(4):
        mx, z = orc.softmax_stats(x[r])
        ids, live = orc.candidate_order(x[r], 128)
        rows.append({"m": float(mx), "z": float(z), "live": int(live), "ids": [int(v) for v in ids]})
    out["call_sampler"] = {"logits_sha256": digest(x), "rows": rows}
    heads = _cached_archive("small-heads", heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE), **SMALL)
    m = orc.Model(heads)
    texts = []
    for n in (3, 21):
        ids = rng.integers(0, m.vocab, n).astype(np.uint32)
        texts.append({"ids": [int(v) for v in ids], "embedding_sha256": digest(m.embed(ids)),
                      "confidence": float(m.confidence(ids))})
    out["probe_heads"] = {"archive_sha256": hashlib.sha256(heads).hexdigest(), "texts": texts}
    return out


def main():
    with open(os.path.join(HERE, "reference_kat.json"), "w") as f:
        json.dump(REFERENCE_KAT, f, indent=1)
    with open(os.path.join(HERE, "small_model_streams.json"), "w") as f:
        json.dump(streams(), f, indent=1)
    with open(os.path.join(HERE, "next_rows.json"), "w") as f:
        json.dump(next_rows(), f, indent=1)


if __name__ == "__main__":
    main()
