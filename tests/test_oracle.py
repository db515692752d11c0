"""The CPU oracle against the reference's own known answers (its unit tests'
inputs and expected values) and against an independent pure-Python
restatement on small inputs. No GPU needed."""

import json
import os

import numpy as np
import pytest

import pyref
from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


# ---- crates/needle-core/src/rng.rs:94-98 and rng.rs:77-88

def test_permutation_matches_numpy():
    kat = golden("reference_kat.json")["mt19937_permutation"]
    assert list(orc.mt_permutation(kat["seed"], kat["n"])) == kat["expect"]
    assert list(orc.mt_permutation(11, 16)) == list(np.random.RandomState(11).permutation(16))


def test_hada_perms_are_numpy_permutations():
    p1, p2 = orc.hada_perms(1024)
    assert np.array_equal(p1, np.random.RandomState(11).permutation(1024))
    assert np.array_equal(p2, np.random.RandomState(13).permutation(1024))
    s1, s2 = orc.hada_perms(1024, split=True)
    want = np.concatenate([np.random.RandomState(11).permutation(512), 512 + np.random.RandomState(988).permutation(512)])
    assert np.array_equal(s1, want)


# ---- crates/needle-core/src/quant.rs:293-321

def test_fwht_matches_dense():
    n = 16
    h = np.array([[(-1) ** bin(i & j).count("1") for j in range(n)] for i in range(n)], np.float64) / np.sqrt(n)
    x = np.sin(np.arange(n, dtype=np.float32) * np.float32(0.37)).astype(np.float32)
    assert np.max(np.abs(orc.rotate(x) - x.astype(np.float64) @ h)) < 1e-5
    assert np.array_equal(orc.rotate(x), pyref.rotate(x))


def test_nearest_ties_low():
    cb = [-1.0, 0.0, 1.0]
    assert orc.nearest(0.5, cb) == 1
    assert orc.nearest(-0.5, cb) == 0
    assert orc.nearest(5.0, cb) == 2
    assert orc.nearest(-5.0, cb) == 0


def test_pack_round_trips():
    # pack_lsb at 4 bits (quant.rs:185-198): byte j holds codes 2j | 2j+1 << 4
    rng = np.random.default_rng(0)
    w = rng.standard_normal((3, 256)).astype(np.float32)
    codes, norms = orc.cq_pack(w)
    idx = np.empty((3, 256), np.int64)
    idx[:, 0::2] = codes & 15
    idx[:, 1::2] = codes >> 4
    repacked = (idx[:, 0::2] | (idx[:, 1::2] << 4)).astype(np.uint8)
    assert np.array_equal(repacked, codes)


def test_codebook_is_lloyd_max_over_sqrt_group():
    import struct

    cb = orc.codebook(4, 128)
    assert len(cb) == 16 and np.all(np.diff(cb) > 0)
    # quant.rs:31 (LM4[0]) and quant.rs:46 (LM4[15]) over sqrt(128), in f64
    lo = struct.unpack("<d", (0xC005AE0F408928FB).to_bytes(8, "little"))[0]
    hi = struct.unpack("<d", (0x4005ED98D06F2A4A).to_bytes(8, "little"))[0]
    assert cb[0] == np.float32(lo / np.sqrt(128.0)) and cb[15] == np.float32(hi / np.sqrt(128.0))


# ---- crates/needle-engine/src/qlinear.rs:976-1006 (kernels_match_reference)

def test_kernels_match_reference_tolerance():
    out, din = 37, 384
    i = np.arange(out * din)
    w = ((((i * 7919) % 1000).astype(np.float32) / np.float32(500.0) - np.float32(1.0)) * np.float32(0.05)).reshape(out, din)
    w = w.astype(np.float32)
    codes, norms = orc.cq_pack(w)
    deq = np.stack([orc.cq_row(codes, norms, din, r) for r in range(out)])
    x = (((np.arange(din) * 31) % 97).astype(np.float32) / np.float32(48.0) - np.float32(1.0)).astype(np.float32)
    y = orc.cq_matmul(codes, norms, din, x)[0]
    want = deq.astype(np.float64) @ x.astype(np.float64)
    assert np.all(np.abs(y - want) < 0.02 * (1 + np.abs(want)))
    # the pure-Python restatement agrees bit for bit on a few rows
    cb = orc.codebook(4, 128)
    for r in (0, 5, 36):
        assert pyref.decode_row(codes[r], norms[r], x, cb) == y[r]
    for rows in (2, 3, 5):
        xs = np.sin(np.arange(rows * din, dtype=np.float32) * np.float32(0.37)).astype(np.float32).reshape(rows, din)
        yy = orc.cq_matmul(codes, norms, din, xs)
        for t in range(rows):
            for r in (1, 20):
                assert pyref.prefill_row(codes[r], norms[r], xs[t], cb, t < rows // 4 * 4) == yy[t, r]


def test_two_bit_kernels_match_reference():
    """qlinear.rs:1008-1033 on its own inputs: a hand-built 2-bit matrix
    (byte codes (37 i) % 251, f16 norms 0.5 + 0.01 i) and inputs cos(0.21 i);
    the decode combine of one row and the prefill combine of five (the
    first four block tokens, the fifth the remainder) agree bit for bit
    with the pure-Python restatement of decode_row_ref / prefill_row_ref."""
    kat = golden("reference_kat.json")["two_bit_kernels_match_reference"]
    out, din = kat["out"], kat["in"]
    groups = din // 128
    codes = ((np.arange(out * din // 4) * 37) % 251).astype(np.uint8).reshape(out, din // 4)
    norms = (np.float32(0.5) + np.arange(out * groups, dtype=np.float32) * np.float32(0.01)).astype(np.float16)
    norms = norms.view(np.uint16).reshape(out, groups)
    xs = np.cos(np.arange(5 * din, dtype=np.float32) * np.float32(0.21)).astype(np.float32).reshape(5, din)
    cb = orc.codebook(2, 128)
    y1 = orc.cq_matmul(codes, norms, din, xs[:1], bits=2)[0]
    for o in range(out):
        assert pyref.decode_row(codes[o], norms[o], xs[0], cb, bits=2) == y1[o]
    y5 = orc.cq_matmul(codes, norms, din, xs, bits=2)
    for t in range(5):
        for o in range(out):
            assert pyref.prefill_row(codes[o], norms[o], xs[t], cb, t < kat["block_rows"], bits=2) == y5[t, o]


def _reference_attention_caches():
    """The caches infer.rs:3035-3051 fills (LayerState::reserve(800, 2, 48,
    64): keys [slot][kvh][48], values transposed [kvh * 64 + d][1600]), as
    [slot][kvh][...] arrays."""
    nkv, qk, vd, slots, cap = 2, 48, 64, 800, 1600
    i = np.arange(slots * nkv * qk)
    k8 = (((i * 37) % 251) - 125).astype(np.int8).reshape(slots, nkv, qk)
    i = np.arange(nkv * vd * cap + 16)
    v8t = (((i * 53) % 249) - 124).astype(np.int8)
    v8 = v8t[: nkv * vd * cap].reshape(nkv, vd, cap)[:, :, :slots].transpose(2, 0, 1).copy()
    i = np.arange(slots * nkv)
    ks = (np.float32(0.01) + (i % 7).astype(np.float32) * np.float32(0.003)).astype(np.float32).reshape(slots, nkv)
    vs = (np.float32(0.02) + (i % 5).astype(np.float32) * np.float32(0.002)).astype(np.float32).reshape(slots, nkv)
    q = (np.sin(np.arange(qk, dtype=np.float32) * np.float32(0.3)) * np.float32(3.0)).astype(np.float32)
    return k8, ks, v8, vs, q


def _slot_of(p, attend):
    """infer.rs:1748-1753."""
    if attend is not None and p >= attend[0]:
        return (p - attend[0]) % attend[1] + attend[0]
    return p


@pytest.mark.timeout(600)
def test_attention_matches_reference_cases():
    """infer.rs:3035-3075's seven key sets and spans (one key; 37 and 300
    keys; 416 + 44 keys under a (416, 256) span; two runs under a (41, 256)
    span, one of them wrapping the ring; a run with an empty second one),
    nested and not, both kv heads, on the caches that test builds: the
    oracle's attend_head_ref agrees bit for bit with the pure-Python
    restatement of infer.rs:1871-2004."""
    k8, ks, v8, vs, q = _reference_attention_caches()
    cases = [((0, 1), (0, 0), None), ((0, 37), (0, 0), None), ((0, 300), (0, 0), None),
             ((0, 416), (416, 460), (416, 256)), ((0, 41), (250, 297), (41, 256)),
             ((0, 41), (290, 560), (41, 256)), ((0, 20), (20, 20), (41, 256))]
    for a, b, attend in cases:
        slots = np.array([_slot_of(p, attend) for p in list(range(*a)) + list(range(*b))], np.int64)
        for nested in (False, True):
            for kvh in (0, 1):
                got = orc.attend_head(k8, ks, v8, vs, q, kvh, slots, nested)
                want = pyref.attend_head(k8, ks, v8, vs, q, kvh, slots, nested)
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (a, b, attend, nested, kvh)


@pytest.mark.timeout(600)
@pytest.mark.parametrize("scale", [1.0, 12.0])
def test_mlp_matches_python(scale):
    """The post block's Hadamard MLP (infer.rs:1610-1634: conditioning
    softmax, three Kronecker stages of two 32 x 32 x 32 passes, perm_fma,
    SiLU) on one 768-wide row with seeded weights held as f16 values: the
    oracle against the pure-Python restatement, bit for bit. scale 12 drives
    the SiLU and the softmax into their saturated ranges."""
    rng = np.random.default_rng(int(scale * 10))
    h16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    d = 768
    h2 = (rng.standard_normal(d) * scale).astype(np.float32)
    w = dict(d1=h16(1 + 0.1 * rng.standard_normal(d)), d2=h16(1 + 0.1 * rng.standard_normal(1024)),
             b2=h16(0.1 * rng.standard_normal(1024)), d3=h16(1 + 0.1 * rng.standard_normal(1024)),
             d4=h16(1 + 0.1 * rng.standard_normal(d)), kron=h16(0.2 * rng.standard_normal((6, 1024))),
             cond_v=h16(0.05 * rng.standard_normal(d * 8)), cond_u=h16(0.1 * rng.standard_normal(8 * 1024)),
             perm1=rng.permutation(1024), perm2=rng.permutation(1024))
    got = orc.mlp(h2, **w)
    want = pyref.mlp_native(h2, w["d1"], w["d2"], w["b2"], w["d3"], w["d4"], w["kron"], w["cond_v"], w["cond_u"],
                            w["perm1"], w["perm2"])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.timeout(600)
@pytest.mark.parametrize("site", [False, True])
def test_mhc_read_matches_python(site):
    """The mHC read (infer.rs:1359-1393: rms of the four lanes, int8 without
    rotation, the 24 int8 gate dots, the pre gates, u), the engram gate and
    the input norm (1397-1418) on one seeded 4 x 768 row: the oracle against
    the pure-Python restatement, bit for bit, with and without an engram
    site."""
    rng = np.random.default_rng(41 + int(site))
    d = 768
    h16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    x = (rng.standard_normal(4 * d) * 0.7).astype(np.float32)
    phi_q = rng.integers(-127, 128, (24, 4 * d), dtype=np.int8)
    phi_s = (np.abs(rng.standard_normal(24)) * 1e-3 + 1e-4).astype(np.float32)
    a_pre, b_pre = np.float32(0.8), h16(0.3 * rng.standard_normal(4))
    norm_in = h16(0.1 * rng.standard_normal(d))
    kr = (rng.standard_normal(d) * 0.5).astype(np.float32) if site else None
    vr = (rng.standard_normal(d) * 0.2).astype(np.float32) if site else None
    lane = 2
    p, u, x1, h = orc.mhc_read(x, phi_q, phi_s, a_pre, b_pre, lane, norm_in, kr, vr)
    pw, uw = pyref.mhc_read_row(x, phi_q, phi_s, a_pre, b_pre, lane)
    x1w, hw = pyref.gate_norm_row(uw, norm_in, kr, vr)
    for got, want in ((p, pw), (u, uw), (x1, x1w), (h, hw)):
        assert np.array_equal(got.view(np.uint32), np.asarray(want, np.float32).view(np.uint32))


@pytest.mark.timeout(600)
def test_post_block_matches_python():
    """The post block of one row (infer.rs:1564-1606: the post norm and the
    gated residual, the pre-MLP norm, the Hadamard MLP, the post gates, the
    residual gates through the f64 Sinkhorn, the mHC write of the four
    lanes) with seeded weights: the oracle against the pure-Python
    restatement, bit for bit."""
    rng = np.random.default_rng(77)
    h16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    d = 768
    mw = [h16(1 + 0.1 * rng.standard_normal(d)), h16(1 + 0.1 * rng.standard_normal(1024)),
          h16(0.1 * rng.standard_normal(1024)), h16(1 + 0.1 * rng.standard_normal(1024)),
          h16(1 + 0.1 * rng.standard_normal(d)), h16(0.2 * rng.standard_normal((6, 1024))),
          h16(0.05 * rng.standard_normal(d * 8)), h16(0.1 * rng.standard_normal(8 * 1024)),
          rng.permutation(1024), rng.permutation(1024)]
    x = (rng.standard_normal(4 * d) * 0.5).astype(np.float32)
    o, x1, u = (rng.standard_normal((3, d)) * 0.5).astype(np.float32)
    pr = (rng.standard_normal(24) * 0.7).astype(np.float32)
    post_norm, pre_hada = h16(0.1 * rng.standard_normal(d)), h16(0.1 * rng.standard_normal(d))
    attn_gate, a_post, a_res = np.float32(0.3), np.float32(0.9), np.float32(1.1)
    b_post, b_res = h16(0.2 * rng.standard_normal(4)), h16(0.5 * rng.standard_normal(16))
    lane = 1
    got, got_mlp = orc.post_row(x, o, x1, pr, u, lane, post_norm, pre_hada, attn_gate, a_post, b_post, a_res, b_res, *mw)
    want, want_mlp = pyref.post_row(x, o, x1, pr, u, lane, post_norm, pre_hada, attn_gate, a_post, b_post, a_res, b_res, mw)
    assert np.array_equal(got_mlp.view(np.uint32), want_mlp.view(np.uint32))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.timeout(300)
@pytest.mark.parametrize("history", [0, 1, 2])
def test_conv_rope_matches_python(history):
    """The conv taps, q / k head norms and RoPE of one row (infer.rs:
    1437-1486) at position 0 (no earlier rows), 1 and later, seeded weights:
    the oracle against the pure-Python restatement, bit for bit."""
    rng = np.random.default_rng(5 + history)
    h16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    rows = [(rng.standard_normal(800) * 0.6).astype(np.float32) for _ in range(3)]
    rows = rows[:1 + history] + [None] * (2 - history)
    taps = [h16(0.5 * rng.standard_normal(3 * n)) for n in (576, 96, 128)]
    q_norm, k_norm = h16(0.1 * rng.standard_normal(48)), h16(0.1 * rng.standard_normal(48))
    ang = rng.uniform(-3, 3, 24)
    cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    got = orc.conv_rope(rows[0], rows[1], rows[2], *taps, q_norm, k_norm, cs, sn)
    want = pyref.conv_rope_row(rows, *taps, q_norm, k_norm, cs, sn)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("p0,n_prev,t", [(0, 0, 5), (37, 3, 1), (200, 120, 1), (50, 2, 4), (9, 0, 1)])
def test_rope_rows_match_python(p0, n_prev, t):
    """The RoPE tables and a session's rows (infer.rs:938-946, 1716-1744): a
    chunk's direct angles, the single-token recurrence after 3 and after 120
    single tokens, a chunk after single tokens, a lone first token: the
    oracle against the pure-Python restatement, bit for bit (both on the
    platform's f64 pow / sin / cos)."""
    theta = np.float32(100000.0)
    got_c, got_s = orc.rope_rows(theta, 48, p0, n_prev, t)
    want_c, want_s = pyref.rope_rows(theta, 48, p0, n_prev, t)
    assert np.array_equal(got_c.view(np.uint32), want_c.view(np.uint32))
    assert np.array_equal(got_s.view(np.uint32), want_s.view(np.uint32))


def test_engram_slots_match_python():
    """The engram hash (infer.rs:1262-1272) at the Needle 3 geometry (orders
    2 and 3, three heads, 18432 slots) over seeded token streams with the
    vocabulary's extremes: the oracle's slots against the pure-Python
    restatement, including the positions too short for an n-gram."""
    rng = np.random.default_rng(12)
    toks = rng.integers(0, 16384, 300).astype(np.uint32)
    toks[:3] = (0, 16383, 0)
    got = orc.engram_slots(toks, (2, 3), 3, 3, 18432)
    for pos in range(len(toks)):
        for oi, order in enumerate((2, 3)):
            for h in range(3):
                want = -1 if pos + 1 < order else pyref.engram_slot(toks, pos, oi, order, h, 3, 18432)
                assert got[pos, oi, h] == want, (pos, oi, h)


@pytest.mark.parametrize("pos", [0, 2, 5, 9, 40])
def test_engram_conv_matches_python(pos):
    """The engram's dilated conv over its int8 value history (infer.rs:
    1307-1320, engram_tap 667-687; four taps, dilation 3) at the first
    positions, where taps fall before position 0, and later: the oracle
    against the pure-Python restatement, bit for bit."""
    rng = np.random.default_rng(100 + pos)
    d = 768
    v8 = rng.integers(-128, 128, (pos + 1, d), dtype=np.int8)
    vs = (np.abs(rng.standard_normal((pos + 1, d // 32))) * 0.02 + 1e-4).astype(np.float32)
    taps = np.asarray(0.5 * rng.standard_normal((4, d)), np.float32).astype(np.float16).astype(np.float32)
    got = orc.engram_conv(taps, v8, vs, pos, 3)
    want = pyref.engram_conv(taps, v8, vs, pos, 3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_row_matches_unpack():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((4, 384)) * 0.02).astype(np.float32)
    codes, norms = orc.cq_pack(w)
    cb = orc.codebook(4, 128)
    r = orc.cq_row(codes, norms, 384, 2)
    # cq_unpack (quant.rs:259-283): cb[idx] * norm, rotated per group
    idx = np.empty(384, np.int64)
    idx[0::2] = codes[2] & 15
    idx[1::2] = codes[2] >> 4
    for g in range(3):
        nrm = norms[2, g:g + 1].view(np.float16).astype(np.float32)[0]
        grp = np.array([cb[k] * nrm for k in idx[g * 128:(g + 1) * 128]], np.float32)
        assert np.array_equal(r[g * 128:(g + 1) * 128], pyref.rotate(grp))


# ---- crates/needle-engine/src/infer.rs:3018-3032, 3078-3084

def test_vector_lane_sums_equal_the_scalar_loop():
    # the matmuls' exact int8 lane sums (vectorised where the host allows)
    # against the plain loop of qlinear.rs:327-337, extremes included
    assert orc.lib().orc_lane_sums_check(7, 4096) == 0


def test_vector_inline_exp_equals_the_scalar_one():
    # the SiLU / gate divide through the eight-wide inline exp against the
    # scalar nexp of infer.rs:353-366, specials included, bit for bit
    assert orc.lib().orc_nexp_check(11, 200000) == 0


def test_vector_quantizer_equals_the_scalar_one():
    # quant_i8 (qlinear.rs:77-88) eight values at a time against the plain
    # loop, and its half-away rounding against std::round, bit for bit
    assert orc.lib().orc_quant_check(5, 20000) == 0


def test_dot16_matches_the_scalar_order():
    i = np.arange(768)
    x = ((((i * 37) % 101).astype(np.float32) - np.float32(50.0)) * np.float32(0.013)).astype(np.float32)
    y = ((((i * 53) % 97).astype(np.float32) - np.float32(48.0)) * np.float32(0.021)).astype(np.float32)
    assert orc.dot16(x, y) == pyref.dot16(x, y)


def test_nexp_is_close_to_exp():
    for i in range(-200, 200):
        x = np.float32(i * 0.37)
        a, b = orc.nexp(x), np.exp(np.float64(x))
        assert abs(a - b) <= 2e-7 * max(b, 1e-30), (x, a, b)
        if i % 17 == 0:
            assert np.float32(a) == pyref.nexp(x)


def test_quant_and_prep_group_match_python():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(300) * 3).astype(np.float32)
    q, s = orc.quant_i8(x)
    q2, s2 = pyref.quant_i8(x)
    assert np.array_equal(q, q2) and np.float32(s) == s2
    for g in range(3):
        q, s = orc.prep_group(x, g)
        q2, s2 = pyref.prep_group(x, g)
        assert np.array_equal(q, q2) and np.float32(s) == s2
    # all-zero input: scale 1, codes 0
    q, s = orc.quant_i8(np.zeros(48, np.float32))
    assert s == 1.0 and not q.any()


def test_chunk_exp_order():
    rng = np.random.default_rng(3)
    for l in (1, 2, 3, 4, 5, 7, 8, 9, 12, 13, 19, 32, 37):
        s = (rng.standard_normal(l) * 4).astype(np.float32)
        m = np.float32(s.max())
        a, ta = orc.chunk_exp(s, m)
        b, tb = pyref.chunk_exp(s, m)
        assert np.array_equal(a, b) and np.float32(ta) == tb, l


def test_key_chunks():
    for n in (1, 15, 16, 63, 64, 255, 256, 257, 300, 700, 1024, 2048):
        for nested in (False, True):
            assert orc.key_chunks(n, nested, 2) == pyref.key_chunks(n, nested, 2)
    assert orc.key_chunks(300, False, 2) == (4, 80)
    assert orc.key_chunks(700, True, 2) == (3, 240)


# ---- infer.rs:3035-3075: the attention cases (ref path), checked for the
# invariants the reference relies on: one chunk normalises by its own sum;
# every output is a convex mix of dequantized values.

def _attn_fixture():
    nkv, qk, vd, slots = 2, 48, 64, 800
    k8 = (((np.arange(slots * nkv * qk) * 37) % 251) - 125).astype(np.int8).reshape(slots, nkv, qk)
    v8 = (((np.arange(slots * nkv * vd) * 53) % 249) - 124).astype(np.int8).reshape(slots, nkv, vd)
    ks = (0.01 + (np.arange(slots * nkv) % 7) * 0.003).astype(np.float32).reshape(slots, nkv)
    vs = (0.02 + (np.arange(slots * nkv) % 5) * 0.002).astype(np.float32).reshape(slots, nkv)
    q = (np.sin(np.arange(qk, dtype=np.float32) * np.float32(0.3)) * np.float32(3.0)).astype(np.float32)
    return k8, ks, v8, vs, q


@pytest.mark.parametrize("keys", [(0, 1), (0, 37), (0, 300)])
@pytest.mark.parametrize("nested", [False, True])
def test_attention_is_a_convex_mix(keys, nested):
    k8, ks, v8, vs, q = _attn_fixture()
    slots = np.arange(*keys)
    for kvh in (0, 1):
        out = orc.attend_head(k8, ks, v8, vs, q, kvh, slots, nested)
        vals = v8[slots, kvh, :].astype(np.float32) * vs[slots, kvh][:, None]
        assert np.all(out <= vals.max(0) + 1e-4) and np.all(out >= vals.min(0) - 1e-4)


def test_sinkhorn_matches_python():
    z = (np.arange(16, dtype=np.float32) * np.float32(0.3) - np.float32(2.0)).astype(np.float32)
    # through the oracle's post block indirectly is heavy; the restatement
    # itself must be doubly stochastic after 20 rounds
    h = pyref.sinkhorn64(z).reshape(4, 4).astype(np.float64)
    assert np.allclose(h.sum(0), 1, atol=1e-6) and np.allclose(h.sum(1), 1, atol=1e-5)


# ---- archive handling (cact.rs:122-135, 580-606)

def test_corrupt_archives_are_rejected(small_archive):
    ok = orc.Model(small_archive)
    assert ok.num_layers == 3
    bad_tag = bytearray(small_archive)
    bad_tag[0:4] = (0x05E12A83).to_bytes(4, "little")
    with pytest.raises(RuntimeError, match="Needle 2"):
        orc.Model(bytes(bad_tag))
    with pytest.raises(RuntimeError, match="past the end|truncated"):
        orc.Model(small_archive[: len(small_archive) // 2])
    with pytest.raises(RuntimeError, match="not a complete"):
        orc.Model(small_archive[:100])


def test_oracle_forward_is_deterministic_and_chunked(small_archive):
    """Feeding 40 tokens at once equals feeding 32 then 8 (forward_native cuts
    feeds into chunks of 32 from the feed start, infer.rs:1105-1131)."""
    m = orc.Model(small_archive)
    ids = np.random.default_rng(4).integers(0, m.vocab, 40).astype(np.uint32)
    a = m.session().forward(ids)
    s = m.session()
    s.forward(ids[:32], orc.OUT_NONE)
    b = s.forward(ids[32:])
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    # a 30-token chunk ends in two remainder rows (30 % 4): positions 28-29
    # take the other prefill combine, which changes every later value
    c = m.session()
    c.forward(ids[:30], orc.OUT_NONE)
    d = c.forward(ids[30:])
    assert not np.array_equal(a.view(np.uint32), d.view(np.uint32)), "chunk boundaries change the arithmetic"


def test_attention_span_identity_and_ring_wrap():
    """Session::attend in the oracle (infer.rs:1749-1825): with every layer
    global, a sink of 0 and a ring longer than the feed, the span is plain
    attention; a ring that wraps inside a 32-token chunk (slots reused)
    runs and is deterministic."""
    import needle_b200 as nb
    from conftest import SMALL

    shape = dict(SMALL)
    shape.update(sliding_window=0, global_layers=())
    m = orc.Model(nb.synth_cact(**shape))
    ids = (np.arange(45) * 29 % 1000).astype(np.uint32)
    plain = m.session().forward(ids)[0]
    s = m.session()
    s.set_attend(0, 1 << 20)
    assert np.array_equal(s.forward(ids)[0].view(np.uint32), plain.view(np.uint32))
    outs = []
    for _ in range(2):
        s = m.session()
        s.set_attend(5, 20)
        outs.append(s.forward(ids)[0])
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    assert not np.array_equal(outs[0], plain)


def test_quant_i8_nan_is_zero():
    """A NaN input quantizes to 0, as Rust's saturating `as i8` (and NEON's
    fcvtas) have it: the attention of a row with no visible key under an
    attention span (0/0) reaches the out projection's A8 this way."""
    x = np.array([1.0, np.nan, -2.0, 0.5], np.float32)
    q, s = orc.quant_i8(x)
    assert q[1] == 0 and q[0] == 64 and q[2] == -127


def test_rollback_and_refeed_reproduce_the_logits(small_archive):
    """Session::rollback (model.rs:81-113) keeps what the dropped positions
    did not touch: feeding the same tokens again after a rollback gives the
    same logits, through a prefill chunk and through one-token steps (the
    RoPE recurrence continues from the kept row)."""
    m = orc.Model(small_archive)
    ids = (np.arange(48) * 31 % 1000).astype(np.uint32)
    s = m.session()
    s.forward(ids[:33])
    want_chunk = s.forward(ids[33:40])[0]
    steps = [s.forward(ids[k:k + 1])[0] for k in range(40, 46)]
    s.rollback(6)
    again = [s.forward(ids[k:k + 1])[0] for k in range(40, 46)]
    for a, b in zip(steps, again):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    s.rollback(13)
    assert np.array_equal(s.forward(ids[33:40])[0].view(np.uint32), want_chunk.view(np.uint32))
    with pytest.raises(RuntimeError):
        s.rollback(33)


def test_truncate_recomputes_from_scratch(small_archive):
    m = orc.Model(small_archive)
    ids = (np.arange(60) * 17 % 1000).astype(np.uint32)
    s = m.session()
    s.forward(ids)
    s.truncate(20)
    assert len(s) == 20
    fresh = m.session()
    fresh.forward(ids[:20])
    a = s.forward(ids[20:23])[0]
    b = fresh.forward(ids[20:23])[0]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.timeout(120)
def test_team_resizes_and_runs_back_to_back():
    # every slice of every job runs exactly once, with jobs issued straight
    # after each resize (new threads that have not yet run included)
    assert orc.lib().orc_team_stress(300) == 0
    assert orc.team_size() == 1


@pytest.mark.timeout(300)
def test_team_does_not_change_a_result(small_archive):
    """One sequence's forward split over a worker team (the reference's
    team.rs role: matmul rows, attention heads, post-block rows) gives the
    single thread's logits and tokens bit for bit, through prefill chunks,
    one-token steps and a sequence-parallel batch."""
    m = orc.Model(small_archive)
    ids = (np.arange(70) * 37 % 1000).astype(np.uint32)
    runs = []
    try:
        for team in (1, 3, 8):
            orc.set_team(team)
            assert orc.team_size() == team
            s = m.session()
            first = s.forward(ids[:45])[0]
            steps = [s.forward(ids[k:k + 1])[0] for k in range(45, 52)]
            toks = m.generate(ids[:33], 9)
            batch = m.prefill_batch(np.stack([ids[:40], ids[10:50]]), threads=2)
            runs.append([first.view(np.uint32), *(x.view(np.uint32) for x in steps), toks, batch.view(np.uint32)])
    finally:
        orc.set_team(1)
    for other in runs[1:]:
        assert all(np.array_equal(a, b) for a, b in zip(runs[0], other))


def test_vector_fwht_equals_the_scalar_butterflies():
    # quant.rs:91-105 on 128 points eight values at a time, bit for bit
    assert orc.lib().orc_fwht_check(13, 5000) == 0


def test_vector_attention_value_sums_equal_the_key_loop():
    # attention's P·V digit-plane sums (infer.rs:1871-2004) on VNNI hosts
    # against the plain key loop, values over all of int8
    assert orc.lib().orc_pv_check(9, 2000) == 0


@pytest.mark.timeout(300)
def test_avx2_and_vnni_lane_sums_give_the_same_streams(small_archive, tmp_path):
    """The 4-bit matmuls run their lane sums on AVX-512 VNNI where the host
    has it and on AVX2 otherwise (ORC_NO_VNNI forces the latter; the choice
    is made when the library loads, so the AVX2 run is a subprocess): both
    give the same logits and tokens bit for bit."""
    import hashlib
    import subprocess
    import sys

    path = tmp_path / "small.cact"
    path.write_bytes(small_archive)
    code = (
        "import sys, hashlib, numpy as np\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "from oracle import oracle as orc\n"
        "m = orc.Model(open(sys.argv[1], 'rb').read())\n"
        "ids = (np.arange(60) * 41 % 1000).astype(np.uint32)\n"
        "toks, lg = m.generate(ids, 8, want_logits=True)\n"
        "print(orc.lib().orc_vnni(), hashlib.sha256(lg.tobytes() + toks.tobytes()).hexdigest())\n"
    )
    runs = {}
    for off in ("0", "1"):
        env = dict(os.environ)
        env.pop("ORC_NO_VNNI", None)
        if off == "1":
            env["ORC_NO_VNNI"] = "1"
        out = subprocess.check_output([sys.executable, "-c", code, str(path)], env=env, text=True).split()
        runs[off] = out
    assert runs["1"][0] == "0"
    assert runs["0"][1] == runs["1"][1]
