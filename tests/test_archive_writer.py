"""The engine's synthetic archive writer (nd_synth_cact) against the
oracle's, written separately from the reference's exporter
(crates/needle-core/src/cact.rs:279-475, quant.rs:184-256,
config.rs:448-482): the two archives must be identical byte for byte, so
the archive every test and the bench load does not rest on the product's
own packer. Covers the small test geometry, a mixed-width plan (2-bit,
3-bit and ternary records), probe heads, and the full Needle 3 archive the
bench runs."""

import numpy as np
import pytest

SMALL = dict(num_layers=3, vocab=1024, engram_slots=96, sliding_window=24, global_layers=(1,), engram_sites=(0, 2),
             seed=7)
MIXED = dict(embedding=2, q=5, k=2, v=5, gate=2, out=3, phi_pre=5, phi_post=3, phi_res=2, table=5, key=3, value=3)


def _same(a, b):
    if a == b:
        return ""
    x, y = np.frombuffer(a, np.uint8), np.frombuffer(b, np.uint8)
    n = min(len(x), len(y))
    d = np.nonzero(x[:n] != y[:n])[0]
    return f"sizes {len(x)} / {len(y)}, first differing byte {d[0] if len(d) else n}"


@pytest.mark.parametrize("case", ["small", "mixed", "heads", "no_window", "needle3"])
def test_engine_writer_matches_oracle_writer(case):
    import needle_b200 as nb
    from oracle import oracle as orc

    kw = {"small": dict(SMALL), "mixed": dict(SMALL, bits=MIXED),
          "heads": dict(num_layers=2, vocab=512, engram_slots=64, sliding_window=16, global_layers=(1,),
                        engram_sites=(0,), seed=3, heads=(1, 2, 3)),
          "no_window": dict(num_layers=2, vocab=256, engram_slots=32, sliding_window=0, global_layers=(),
                            engram_sites=(1,), seed=5, std=0.05),
          "needle3": dict(seed=0)}[case]
    a, b = nb.synth_cact(**kw), orc.synth_cact(**kw)
    assert a == b, _same(a, b)


def test_oracle_archive_loads_with_needle3_geometry():
    """The oracle reads back its own Needle 3 archive with the config's
    dims (config.rs:60-103) and the budget kv_window (3456, the reference's
    effective_kv_window for this geometry)."""
    from oracle import oracle as orc

    data = orc.synth_cact(num_layers=20)
    m = orc.Model(data)
    assert (m.vocab, m.d_model, m.num_layers, m.num_heads, m.num_kv_heads, m.qk_head_dim, m.v_head_dim,
            m.max_seq_len) == (16384, 768, 20, 12, 2, 48, 64, 4096)
    assert int(np.frombuffer(data[12:16], np.uint32)[0]) == 3456
