"""The C-ABI library loads and exports every entry point include/*.h
declares; host-only entry points (archive writer, CQ packer, archive
validation) behave without a GPU. No compute runs on a device here."""

import ctypes
import glob
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\([^;{]*\)\s*;", src, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    import needle_b200 as nb

    names = declared_functions()
    assert "needle_load" in names and "nd_batch_step" in names and len(names) >= 20
    lib = ctypes.CDLL(nb.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_cq_pack_matches_oracle():
    """Two restatements of quant.rs:233-256 (engine and oracle) agree bit for bit."""
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(5)
    w = (rng.standard_normal((64, 3072)) * 0.02).astype(np.float32)
    c1, n1 = nb.cq_pack(w)
    c2, n2 = orc.cq_pack(w)
    assert np.array_equal(c1, c2) and np.array_equal(n1, n2)


def test_synth_archive_is_deterministic_and_valid(small_archive):
    import needle_b200 as nb
    from conftest import SMALL

    again = nb.synth_cact(**SMALL)
    assert again == small_archive
    hdr = np.frombuffer(small_archive[:196], np.uint32)
    assert hdr[0] == 0x05E12A84 and hdr[10] == 3 and hdr[5] == 1024
    full_hdr = np.frombuffer(nb.synth_cact(seed=0, num_layers=1, engram_sites=(0,), global_layers=())[:196], np.uint32)
    assert full_hdr[7] == 768 and full_hdr[14] == 1024


def test_default_kv_window_matches_config_rs():
    """config.rs:448-482 at the Needle 3 defaults gives 3456 (header word 3)."""
    import needle_b200 as nb

    kat = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_kat.json")))["kv_window_default"]["expect"]
    data = nb.synth_cact(seed=1, vocab=256, engram_slots=8)
    assert np.frombuffer(data[:196], np.uint32)[3] == kat


def test_engine_rejects_corrupt_archives(small_archive):
    """Archive validation runs before any device work (cact.rs:122-135,
    580-606), so it is testable here."""
    import needle_b200 as nb

    bad = bytearray(small_archive)
    bad[0:4] = (0x05E12A83).to_bytes(4, "little")
    with pytest.raises(RuntimeError, match="Needle 2"):
        nb.Model(bytes(bad))
    with pytest.raises(RuntimeError, match="past the end|truncated"):
        nb.Model(small_archive[: len(small_archive) // 2])
    with pytest.raises(RuntimeError, match="not a complete"):
        nb.Model(small_archive[:10])


def test_needle_h_errors_without_a_model():
    import needle_b200 as nb

    L = nb.lib()
    assert L.needle_init(b"", b"[]", None) == -1
    assert b"needle_load" in L.needle_last_error()
    buf = ctypes.create_string_buffer(256)
    assert L.needle_complete(b"hi", 8, buf, 256) == -1
    assert b"needle_init" in buf.value
    assert L.needle_load(None, 0) == -1


def test_oracle_reproduces_committed_streams(small_archive):
    """The oracle still produces the committed greedy streams on the small
    archive (tests/golden/make_golden.py wrote them)."""
    import hashlib

    from oracle import oracle as orc

    g = json.load(open(os.path.join(ROOT, "tests", "golden", "small_model_streams.json")))
    assert hashlib.sha256(small_archive).hexdigest() == g["archive_sha256"]
    m = orc.Model(small_archive)
    for case in g["cases"]:
        toks, logits = m.generate(np.array(case["prompt"], np.uint32), len(case["tokens"]), want_logits=True)
        assert [int(t) for t in toks] == case["tokens"]
        assert hashlib.sha256(logits.view(np.uint32).tobytes()).hexdigest() == case["first_logits_sha256"]


def test_oracle_reproduces_committed_next_rows():
    """The oracle still produces the committed records of the widened rows
    (tests/golden/make_golden.py wrote them): mixed-width streams, the call
    sampler on fixed rows, the probe heads."""
    import hashlib
    import sys

    import needle_b200 as nb
    from conftest import MIXED_BITS, SMALL, _cached_archive
    from oracle import oracle as orc

    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    from make_golden import call_sampler_logits, digest

    g = json.load(open(os.path.join(ROOT, "tests", "golden", "next_rows.json")))
    mixed = _cached_archive("small-mixed", bits=MIXED_BITS, **SMALL)
    assert hashlib.sha256(mixed).hexdigest() == g["mixed_width"]["archive_sha256"]
    m = orc.Model(mixed)
    for case in g["mixed_width"]["cases"]:
        toks, logits = m.generate(np.array(case["prompt"], np.uint32), len(case["tokens"]), want_logits=True)
        assert [int(t) for t in toks] == case["tokens"]
        assert digest(logits) == case["first_logits_sha256"]
    x = call_sampler_logits()
    assert digest(x) == g["call_sampler"]["logits_sha256"]
    for r, row in enumerate(g["call_sampler"]["rows"]):
        mx, z = orc.softmax_stats(x[r])
        ids, live = orc.candidate_order(x[r], 128)
        assert float(mx) == row["m"] and float(z) == row["z"] and live == row["live"]
        assert [int(v) for v in ids] == row["ids"]
    heads = _cached_archive("small-heads", heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE), **SMALL)
    assert hashlib.sha256(heads).hexdigest() == g["probe_heads"]["archive_sha256"]
    m = orc.Model(heads)
    for t in g["probe_heads"]["texts"]:
        ids = np.array(t["ids"], np.uint32)
        assert digest(m.embed(ids)) == t["embedding_sha256"]
        assert float(m.confidence(ids)) == t["confidence"]
