"""CQ records of 2, 3 and ternary bits next to the 4-bit ones
(crates/needle-engine/src/qlinear.rs:220-265, crates/needle-core/src/quant.rs
:11-12, 259-287), on the CPU: the oracle's matmul against the literal
pure-Python restatement (activations stored at act_pos, the width's decode
lane rule), the engine's packer against the nearest-centroid rule, and
mixed-width archives through the oracle."""

import numpy as np
import pytest

import pyref
from conftest import MIXED_BITS, SMALL

WIDTHS = [2, 3, 4, 5]
f32 = np.float32


def hand_matrix(out, din, bits):
    """qlinear.rs:1010-1015's hand-built matrix at any width: code bytes
    cycle through (i * 37) % 251, norms 0.5 + 0.01 i."""
    width = pyref.code_width(bits)
    groups = din // 128
    codes = np.array([(i * 37) % 251 for i in range(out * din * width // 8)], np.uint8).reshape(out, -1)
    norms = np.array([f32(0.5) + f32(i) * f32(0.01) for i in range(out * groups)], np.float32)
    return codes, norms.astype(np.float16).view(np.uint16).reshape(out, groups)


def hand_inputs(rows, din):
    return np.cos(np.arange(rows * din, dtype=np.float32) * f32(0.21)).astype(np.float32).reshape(rows, din)


@pytest.mark.parametrize("bits", WIDTHS)
def test_decode_combine_matches_literal_restatement(bits):
    from oracle import oracle as orc

    codes, norms = hand_matrix(9, 256, bits)
    x = hand_inputs(1, 256)
    y = orc.cq_matmul(codes, norms, 256, x, bits=bits)[0]
    cb = orc.codebook(bits)
    for r in range(9):
        want = pyref.decode_row(codes[r], norms[r], x[0], cb, bits)
        assert y[r].view(np.uint32) == f32(want).view(np.uint32), (bits, r, y[r], want)


@pytest.mark.parametrize("bits", WIDTHS)
def test_prefill_combine_matches_literal_restatement(bits):
    from oracle import oracle as orc

    codes, norms = hand_matrix(9, 256, bits)
    xs = hand_inputs(5, 256)
    y = orc.cq_matmul(codes, norms, 256, xs, bits=bits)
    single = orc.cq_matmul(codes, norms, 256, xs, mode=2, bits=bits)
    cb = orc.codebook(bits)
    for t in range(5):
        for r in range(9):
            want = pyref.prefill_row(codes[r], norms[r], xs[t], cb, t < 4, bits)
            assert y[t, r].view(np.uint32) == f32(want).view(np.uint32), (bits, t, r)
            block = pyref.prefill_row(codes[r], norms[r], xs[t], cb, True, bits)
            assert single[t, r].view(np.uint32) == f32(block).view(np.uint32), (bits, t, r)


def test_two_bit_lane_rule_is_not_the_four_bit_one():
    """The same 2-bit codes combined under the 4-bit lane rule give other
    floats on these inputs: the oracle follows the 2-bit rule."""
    from oracle import oracle as orc

    codes, norms = hand_matrix(9, 256, 2)
    x = hand_inputs(1, 256)[0]
    cb = orc.codebook(2)
    table, cbs = pyref.code_table(cb, 2)
    y = orc.cq_matmul(codes, norms, 256, x[None], bits=2)[0]
    differ = 0
    for r in range(9):
        c = pyref.unpack_lsb(codes[r], 2)
        lanes = [f32(0)] * 4
        for g in range(2):
            q, sx = pyref.prep_group(x, g)
            s = [0, 0, 0, 0]
            for p in range(128):
                s[(p % 32) // 8] += table[c[g * 128 + p]] * int(q[p])
            sc = (sx * cbs) * pyref._f16(norms[r][g])
            lanes = [pyref.fma32(f32(s[l]), sc, lanes[l]) for l in range(4)]
        other = (lanes[0] + lanes[1]) + (lanes[2] + lanes[3])
        assert abs(float(y[r]) - float(other)) <= 1e-4 * (1 + abs(float(other)))  # the same dot product
        differ += int(y[r].view(np.uint32) != f32(other).view(np.uint32))
    assert differ > 0


@pytest.mark.parametrize("bits", [2, 3, 5])
def test_pack_matches_nearest_centroid(bits):
    """The engine's packer at widths the reference's packer does not write:
    rotate, f32 norm, nearest centroid (ties low), ternary centroids k stored
    as code (k + 3) % 4, LSB-first bytes, f16 norms."""
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(bits)
    rows, d = 4, 300
    w = (rng.standard_normal((rows, d)) * 0.02).astype(np.float32)
    codes, norms = nb.cq_pack(w, bits)
    cb = orc.codebook(bits)
    width = pyref.code_width(bits)
    for r in range(rows):
        idx = []
        for g in range(3):
            buf = np.zeros(128, np.float32)
            seg = w[r, g * 128:(g + 1) * 128]
            buf[:len(seg)] = seg
            v = pyref.rotate(buf)
            ss = f32(0)
            for t in v:
                ss = f32(ss + f32(t * t))
            norm = np.sqrt(ss)
            assert norms[r, g] == np.float16(norm).view(np.uint16)
            denom = max(norm, f32(1e-12))
            for t in v:
                k = orc.nearest(float(f32(t / denom)), cb)
                idx.append((k + 3) % 4 if bits == 5 else k)
        assert list(pyref.unpack_lsb(codes[r], width)) == idx


def test_ternary_codes_select_centroids():
    """Ternary code 3 is the negative centroid, 0 zero, 1 the positive one,
    and code 2 (never written) reads as zero (qlinear.rs:225-227, 250-251)."""
    from oracle import oracle as orc

    codes = np.zeros((1, 32), np.uint8)
    codes[0, 0] = 0b10_01_00_11  # p = 0..3: codes 3, 0, 1, 2
    norms = np.array([[np.float16(1.0).view(np.uint16)]], np.uint16)
    row = orc.cq_row(codes, norms, 128, 0, bits=5)
    g = np.zeros(128, np.float32)
    c = orc.codebook(5)
    g[0], g[1], g[2], g[3] = c[0], c[1], c[2], 0.0
    assert np.array_equal(row, pyref.rotate(g))


def test_mixed_archive_runs_through_the_oracle():
    import needle_b200 as nb
    from oracle import oracle as orc

    plain = orc.Model(nb.synth_cact(**SMALL))
    mixed = orc.Model(nb.synth_cact(bits=MIXED_BITS, **SMALL))
    ids = np.arange(9, dtype=np.uint32) * 37 % 1000
    a = plain.session().forward(ids)[0]
    b = mixed.session().forward(ids)[0]
    assert np.all(np.isfinite(b)) and not np.array_equal(a, b)
    assert nb.synth_cact(bits=4, **SMALL) == nb.synth_cact(**SMALL)


def test_fused_parts_must_share_a_width():
    """qlinear.rs:517: q|k|v|gate at 2 and 4 bits is refused; 2-bit next to
    ternary is one code width and loads."""
    import needle_b200 as nb
    from oracle import oracle as orc

    with pytest.raises(RuntimeError, match="code width"):
        orc.Model(nb.synth_cact(bits=dict(q=2, k=4), **SMALL))
    orc.Model(nb.synth_cact(bits=dict(q=2, k=5, v=2, gate=5), **SMALL))
    with pytest.raises(RuntimeError):
        nb.synth_cact(bits=dict(q=6), **SMALL)
