"""ctypes view of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, as the checker and the timed CPU baseline. The product path never
imports it.
"""

import ctypes as C
import os

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = C.CDLL(path)
        P, I, U32, I64, F = C.c_void_p, C.c_int, C.c_uint32, C.c_int64, C.c_float
        sig = {
            "orc_last_error": (C.c_char_p, []),
            "orc_f32_to_f16": (C.c_uint16, [F]),
            "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_nexp": (F, [F]),
            "orc_dot16": (F, [P, P, I]),
            "orc_quant_i8": (F, [P, I, P]),
            "orc_rotate": (None, [P, I]),
            "orc_nearest": (I, [F, P, I]),
            "orc_codebook": (I, [I, I, P]),
            "orc_mt_permutation": (None, [U32, I, P]),
            "orc_hada_perms": (None, [I, I, P, P]),
            "orc_cq_pack": (None, [P, I, I, P, P]),
            "orc_prep_group": (F, [P, I, I, P]),
            "orc_chunk_exp": (F, [P, I, F]),
            "orc_key_chunks": (None, [I64, I, I, P, P]),
            "orc_cq_matmul": (I, [P, P, I, I, I, P, I, I, P]),
            "orc_cq_row": (I, [P, P, I, I, I, I, P]),
            "orc_lane_sums_check": (I, [C.c_uint64, I]),
            "orc_nexp_check": (I, [C.c_uint64, I]),
            "orc_quant_check": (I, [C.c_uint64, I]),
            "orc_set_team": (None, [I]),
            "orc_team_size": (I, []),
            "orc_team_stress": (I, [I]),
            "orc_vnni": (I, []),
            "orc_pv_check": (I, [C.c_uint64, I]),
            "orc_fwht_check": (I, [C.c_uint64, I]),
            "orc_mlp": (I, [P, I, P, P, P, P, P, P, P, P, P, P, P]),
            "orc_mhc_read": (I, [P, I, P, P, F, P, I, P, P, P, P, P, P, P]),
            "orc_post_row": (I, [I, P, P, F, F, P, F, P, P, P, P, P, P, P, P, P, P, P, I, P, P, P, P, P, P]),
            "orc_conv_rope": (I, [P, P, P, P, P, P, P, P, P, P, P]),
            "orc_rope_rows": (I, [F, I, I64, I, I, P, P]),
            "orc_engram_slots": (None, [P, I, P, I, I, I, I, P]),
            "orc_engram_conv": (None, [P, P, P, I64, I, I, I, P]),
            "orc_attend_head": (None, [P, P, P, P, I, I, I, P, I, P, I, I, P]),
            "orc_model_load": (P, [P, C.c_uint64]),
            "orc_model_free": (None, [P]),
            "orc_model_dims": (I, [P, P]),
            "orc_session_new": (P, [P]),
            "orc_session_free": (None, [P]),
            "orc_session_clone": (P, [P]),
            "orc_session_len": (I, [P]),
            "orc_session_set_attend": (None, [P, I64, I64]),
            "orc_session_rollback": (I, [P, P, I64]),
            "orc_session_rewind_zeroed": (I, [P, P, I64]),
            "orc_session_truncate": (I, [P, P, I64]),
            "orc_forward": (I, [P, P, P, I, I, P]),
            "orc_head_logits": (None, [P, P, P]),
            "orc_head_logits_sparse": (None, [P, P, P, I, P]),
            "orc_last_hidden": (I, [P, P]),
            "orc_masked_argmax": (U32, [P, I, P]),
            "orc_engine_expf": (C.c_float, [C.c_float]),
            "orc_fast_exp": (C.c_float, [C.c_float]),
            "orc_dot8": (C.c_float, [P, P, I]),
            "orc_probe_pool": (None, [P, I, I, I, I, I, P, P, P, P, P]),
            "orc_head_present": (I, [P, I]),
            "orc_embed": (I, [P, P, I, P]),
            "orc_confidence": (I, [P, P, I, P]),
            "orc_cells": (I, [P, P, I, P]),
            "orc_softmax_stats": (None, [P, I, P, P]),
            "orc_candidate_order": (I, [P, I, I, P]),
            "orc_trace": (None, [I]),
            "orc_trace_get": (I, [C.c_char_p, P, I]),
            "orc_generate": (I, [P, P, I, I, P, P, P]),
            "orc_generate_batch": (I, [P, I, P, I, I, P, P, I]),
            "orc_prefill_batch": (I, [P, I, P, I, P, I]),
            "orc_batch_new": (P, [P, I]),
            "orc_batch_free": (None, [P]),
            "orc_batch_prefill": (I, [P, P, I, I]),
            "orc_batch_step": (I, [P, P, P, I]),
            "orc_op_zcn": (None, [P, P, I, I, P]),
            "orc_op_rope": (None, [P, I, F, P]),
            "orc_op_silu": (None, [P, C.c_int64, P]),
            "orc_op_gather": (I, [P, P, I, P]),
            "orc_synth_cact": (I, [I, I, I, I, C.c_uint64, C.c_uint64, C.c_uint64, F, P, I, C.c_uint, P, C.c_uint64,
                                   C.POINTER(C.c_uint64)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p) if a is not None else None


# Needle 3's geometry knobs (crates/needle-core/src/config.rs:60-103).
NEEDLE3 = dict(num_layers=20, vocab=16384, engram_slots=18432, sliding_window=1024, global_layers=(4, 9, 14, 19),
               engram_sites=(3, 7, 11, 15, 19))
TERNARY = 5


def cq_roles(num_layers=20, engram_sites=(3, 7, 11, 15, 19), **_):
    """Role of each CQ record in archive order (cact.rs:279-352)."""
    roles = ["embedding"] + ["q", "k", "v", "gate", "out"] * num_layers + ["phi_pre", "phi_post", "phi_res"]
    return roles + ["table", "key", "value"] * len(engram_sites)


def synth_cact(seed=0, std=0.02, bits=None, heads=(), **shape) -> bytes:
    """The random-init archive written from the reference's exporter
    (cact.rs:279-475) by the oracle, independently of the engine's writer:
    the same knobs as the engine's synth_cact (bits: one width, a dict role
    -> bits, or a list in record order; heads: probe head codes 1-3)."""
    g = dict(NEEDLE3)
    g.update(shape)
    roles = cq_roles(g["num_layers"], g["engram_sites"])
    if bits is None:
        plan = []
    elif isinstance(bits, int):
        plan = [bits] * len(roles)
    elif isinstance(bits, dict):
        plan = [bits.get(r, 4) for r in roles]
    else:
        plan = list(bits)
    plan = np.ascontiguousarray(plan, np.int32)
    gm = sum(1 << l for l in g["global_layers"])
    es = sum(1 << l for l in g["engram_sites"])
    n = C.c_uint64(0)
    args = (g["num_layers"], g["vocab"], g["engram_slots"], g["sliding_window"], gm, es, seed, std,
            _p(plan) if len(plan) else None, len(plan), sum(1 << c for c in set(heads)))
    if lib().orc_synth_cact(*args, None, 0, C.byref(n)) != 0:
        raise RuntimeError(lib().orc_last_error().decode())
    buf = np.zeros(n.value, np.uint8)
    if lib().orc_synth_cact(*args, _p(buf), n.value, C.byref(n)) != 0:
        raise RuntimeError(lib().orc_last_error().decode())
    return buf.tobytes()


def mlp(h2, d1, d2, b2, d3, d4, kron, cond_v, cond_u, perm1, perm2):
    """mlp_native (infer.rs:1610-1634) on one row with the given weights."""
    h2 = np.ascontiguousarray(h2, np.float32)
    d = len(h2)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    i64 = lambda a: np.ascontiguousarray(a, np.int64)
    out = np.zeros(d, np.float32)
    args = [f(d1), f(d2), f(b2), f(d3), f(d4), f(kron), f(cond_v), f(cond_u), i64(perm1), i64(perm2)]
    if lib().orc_mlp(_p(h2), d, *[_p(a) for a in args], _p(out)) != 0:
        raise ValueError("bad MLP arguments")
    return out


def mhc_read(x, phi_q, phi_s, a_pre, b_pre, lane, norm_in, kr=None, vr=None):
    """The mHC read, engram gate and input norm of one row (infer.rs:
    1359-1418): (p [24], u, x1, h)."""
    x = np.ascontiguousarray(x, np.float32)
    d = len(x) // 4
    f = lambda a: np.ascontiguousarray(a, np.float32)
    p, u, x1, h = np.zeros(24, np.float32), np.zeros(d, np.float32), np.zeros(d, np.float32), np.zeros(d, np.float32)
    rc = lib().orc_mhc_read(_p(x), d, _p(np.ascontiguousarray(phi_q, np.int8)), _p(f(phi_s)), float(a_pre), _p(f(b_pre)),
                            int(lane), _p(f(kr)) if kr is not None else None, _p(f(vr)) if vr is not None else None,
                            _p(f(norm_in)), _p(p), _p(u), _p(x1), _p(h))
    if rc != 0:
        raise ValueError("bad mHC read arguments")
    return p, u, x1, h


def post_row(x, o, x1, pr, u, lane, post_norm, pre_hada, attn_gate, a_post, b_post, a_res, b_res, d1, d2, b2, d3, d4,
             kron, cond_v, cond_u, perm1, perm2):
    """The post block of one row (infer.rs:1564-1606): (the new lanes
    [4 d], the MLP output [d])."""
    f = lambda a: np.ascontiguousarray(a, np.float32)
    i64 = lambda a: np.ascontiguousarray(a, np.int64)
    xs = f(x).copy()
    d = len(xs) // 4
    mlp_out = np.zeros(d, np.float32)
    rc = lib().orc_post_row(d, _p(f(post_norm)), _p(f(pre_hada)), float(attn_gate), float(a_post), _p(f(b_post)),
                            float(a_res), _p(f(b_res)), _p(f(d1)), _p(f(d2)), _p(f(b2)), _p(f(d3)), _p(f(d4)), _p(f(kron)),
                            _p(f(cond_v)), _p(f(cond_u)), _p(i64(perm1)), _p(i64(perm2)), int(lane), _p(f(o)), _p(f(x1)),
                            _p(f(pr)), _p(f(u)), _p(xs), _p(mlp_out))
    if rc != 0:
        raise ValueError("bad post block arguments")
    return xs, mlp_out


def conv_rope(cur, prev1, prev2, q_taps, k_taps, v_taps, q_norm, k_norm, cs, sn):
    """The conv taps, head norms and RoPE of one row (infer.rs:1437-1486);
    prev1 / prev2 None before position 0. Returns the q | k | v row [800]."""
    f = lambda a: np.ascontiguousarray(a, np.float32)
    out = np.zeros(800, np.float32)
    opt = lambda a: _p(f(a)) if a is not None else None
    rc = lib().orc_conv_rope(_p(f(cur)), opt(prev1), opt(prev2), _p(f(q_taps)), _p(f(k_taps)), _p(f(v_taps)),
                             _p(f(q_norm)), _p(f(k_norm)), _p(f(cs)), _p(f(sn)), _p(out))
    if rc != 0:
        raise ValueError("bad conv arguments")
    return out


def rope_rows(theta, qk, p0, n_prev, t):
    """The session RoPE rows of infer.rs:1716-1744 after n_prev single-token
    rows up to p0 - 1: (cos, sin) [t][qk / 2] of rows p0 .. p0 + t - 1."""
    cs, sn = np.zeros((t, qk // 2), np.float32), np.zeros((t, qk // 2), np.float32)
    if lib().orc_rope_rows(float(theta), qk, int(p0), int(n_prev), int(t), _p(cs), _p(sn)) != 0:
        raise ValueError("bad RoPE arguments")
    return cs, sn


def engram_slots(tokens, orders, heads, stride, slots):
    """The engram hash's table slot per (position, order index, head), -1
    before a full n-gram (infer.rs:1262-1272)."""
    tokens = np.ascontiguousarray(tokens, np.uint32)
    orders = np.ascontiguousarray(orders, np.int32)
    out = np.zeros((len(tokens), len(orders), heads), np.int64)
    lib().orc_engram_slots(_p(tokens), len(tokens), _p(orders), len(orders), heads, stride, slots, _p(out))
    return out


def engram_conv(taps, v8, vs, pos, dil):
    """The engram's dilated conv over the int8 value history at position
    pos (infer.rs:1307-1320): v [d]."""
    taps = np.ascontiguousarray(taps, np.float32)
    v8 = np.ascontiguousarray(v8, np.int8)
    vs = np.ascontiguousarray(vs, np.float32)
    d = taps.shape[1]
    out = np.zeros(d, np.float32)
    lib().orc_engram_conv(_p(taps), _p(v8), _p(vs), int(pos), taps.shape[0], int(dil), d, _p(out))
    return out


def set_team(threads: int) -> None:
    """Split one sequence's matmul rows, attention heads and post-block rows
    over `threads` host threads (1: none), as the reference's worker team
    does; results do not depend on it."""
    lib().orc_set_team(int(threads))


def team_size() -> int:
    return lib().orc_team_size()


def f32_to_f16_bits(x: float) -> int:
    return lib().orc_f32_to_f16(float(x))


def nexp(x: float) -> float:
    return lib().orc_nexp(float(x))


def dot16(x, y) -> float:
    x = np.ascontiguousarray(x, np.float32)
    y = np.ascontiguousarray(y, np.float32)
    return lib().orc_dot16(_p(x), _p(y), len(x))


def quant_i8(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(len(x), np.int8)
    s = lib().orc_quant_i8(_p(x), len(x), _p(q))
    return q, s


def rotate(x):
    y = np.array(x, np.float32, copy=True)
    lib().orc_rotate(_p(y), len(y))
    return y


def nearest(x: float, cb) -> int:
    cb = np.ascontiguousarray(cb, np.float32)
    return lib().orc_nearest(float(x), _p(cb), len(cb))


def codebook(bits: int, group: int = 128):
    n = lib().orc_codebook(bits, group, None)
    out = np.zeros(n, np.float32)
    lib().orc_codebook(bits, group, _p(out))
    return out


def mt_permutation(seed: int, n: int):
    out = np.zeros(n, np.int64)
    lib().orc_mt_permutation(seed, n, _p(out))
    return out


def hada_perms(n: int, split: bool = False):
    a = np.zeros(n, np.int64)
    b = np.zeros(n, np.int64)
    lib().orc_hada_perms(n, int(split), _p(a), _p(b))
    return a, b


def cq_pack(w):
    w = np.ascontiguousarray(w, np.float32)
    rows, d = w.shape
    g = (d + 127) // 128
    packed = np.zeros((rows, g * 64), np.uint8)
    norms = np.zeros((rows, g), np.uint16)
    lib().orc_cq_pack(_p(w), rows, d, _p(packed), _p(norms))
    return packed, norms


def prep_group(x, g):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(128, np.int8)
    s = lib().orc_prep_group(_p(x), len(x), g, _p(q))
    return q, s


def chunk_exp(s, m):
    s = np.array(s, np.float32, copy=True)
    tot = lib().orc_chunk_exp(_p(s), len(s), float(m))
    return s, tot


def key_chunks(n, nested, nkv):
    c = np.zeros(1, np.int64)
    k = np.zeros(1, np.int64)
    lib().orc_key_chunks(int(n), int(nested), int(nkv), _p(c), _p(k))
    return int(c[0]), int(k[0])


def cq_matmul(codes, norms, in_dim, x, mode=0, bits=4):
    """y = x @ W^T with the reference's kernels: decode (T == 1), prefill
    (block/remainder rule) otherwise; mode 2 = single-row kernel per token.
    ``bits`` is the record bits (2, 3, 4, or 5 = ternary)."""
    codes = np.ascontiguousarray(codes, np.uint8)
    norms = np.ascontiguousarray(norms, np.uint16)
    x = np.ascontiguousarray(x, np.float32).reshape(-1, in_dim)
    out = norms.shape[0]
    y = np.zeros((x.shape[0], out), np.float32)
    rc = lib().orc_cq_matmul(_p(codes), _p(norms), out, in_dim, bits, _p(x), x.shape[0], mode, _p(y))
    if rc != 0:
        raise RuntimeError(lib().orc_last_error().decode())
    return y


def cq_row(codes, norms, in_dim, r, bits=4):
    codes = np.ascontiguousarray(codes, np.uint8)
    norms = np.ascontiguousarray(norms, np.uint16)
    out = np.zeros(in_dim, np.float32)
    if lib().orc_cq_row(_p(codes), _p(norms), norms.shape[0], in_dim, bits, r, _p(out)) != 0:
        raise RuntimeError(lib().orc_last_error().decode())
    return out


def attend_head(k8, ks, v8, vs, q, kvh, slots, nested):
    """attend_head_ref over caches k8 [slot][nkv][qk], v8 [slot][nkv][vd]."""
    nkv, qk = k8.shape[1], k8.shape[2]
    vd = v8.shape[2]
    slots = np.ascontiguousarray(slots, np.int64)
    out = np.zeros(vd, np.float32)
    q = np.ascontiguousarray(q, np.float32)
    lib().orc_attend_head(_p(np.ascontiguousarray(k8)), _p(np.ascontiguousarray(ks, np.float32)),
                          _p(np.ascontiguousarray(v8)), _p(np.ascontiguousarray(vs, np.float32)),
                          nkv, qk, vd, _p(q), kvh, _p(slots), len(slots), int(nested), _p(out))
    return out


def engine_expf(x: float) -> float:
    """agent.rs:1130-1145."""
    return lib().orc_engine_expf(float(x))


def fast_exp(x: float) -> float:
    """linalg.rs:262-277."""
    return lib().orc_fast_exp(float(x))


def dot8(a, b):
    """linalg.rs:242-257."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return np.float32(lib().orc_dot8(_p(a), _p(b), len(a)))


def probe_pool(cells, probes, gain, query, row_bias):
    """heads.rs:12-56 over cells [t, l1, d]; probes [l1, k, d], gain [l1,
    k], query [q, d], row_bias [q, l1 * k]: the pooled [q * d]."""
    cells = np.ascontiguousarray(cells, np.float32)
    t, l1, d = cells.shape
    k = gain.shape[1]
    q = query.shape[0]
    out = np.zeros(q * d, np.float32)
    args = [np.ascontiguousarray(a, np.float32) for a in (probes, gain, query, row_bias)]
    lib().orc_probe_pool(_p(cells), t, l1, d, k, q, *[_p(a) for a in args], _p(out))
    return out


def softmax_stats(x):
    """agent.rs:1241-1252: (max, sum exp(l - max)) as the call sampler has them."""
    x = np.ascontiguousarray(x, np.float32)
    m = np.zeros(1, np.float32)
    z = np.zeros(1, np.float64)
    lib().orc_softmax_stats(_p(x), len(x), _p(m), _p(z))
    return m[0], z[0]


def candidate_order(x, k=128):
    """agent.rs:335-343: the first k unmasked candidates by (logit desc, id
    asc), and how many are unmasked."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(k, np.int32)
    live = lib().orc_candidate_order(_p(x), len(x), k, _p(out))
    return out[:min(k, live)], live


def op_zcn(x, s):
    """infer.rs:426-443 over rows x [T, n] with weights s [n]."""
    x = np.ascontiguousarray(x, np.float32)
    s = np.ascontiguousarray(s, np.float32)
    out = np.zeros_like(x)
    lib().orc_op_zcn(_p(x), _p(s), x.shape[0], x.shape[1], _p(out))
    return out


def op_rope(x, theta=100000.0):
    """RoPE of rows x [T, 672] (12 q heads, 2 k heads of 48) at positions
    0..T-1 (infer.rs:1474-1483, 1716-1744)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_op_rope(_p(x), x.shape[0], float(theta), _p(out))
    return out


def op_silu(x):
    """infer.rs:2463-2496."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_op_silu(_p(x), x.size, _p(out))
    return out


def masked_argmax(x, allow_bits=None):
    x = np.ascontiguousarray(x, np.float32)
    return lib().orc_masked_argmax(_p(x), len(x), _p(allow_bits) if allow_bits is not None else None)


OUT_NONE, OUT_LAST_LOGITS, OUT_LAST_HIDDEN, OUT_ALL_LOGITS, OUT_HIDDEN = 0, 1, 2, 3, 4


class Model:
    """The packed model as the reference's native path runs it."""

    def __init__(self, archive: bytes):
        buf = np.frombuffer(archive, np.uint8)
        self._h = lib().orc_model_load(_p(buf), len(buf))
        if not self._h:
            raise RuntimeError(lib().orc_last_error().decode())
        dims = np.zeros(9, np.int32)
        lib().orc_model_dims(self._h, _p(dims))
        (self.vocab, self.out_rows, self.d_model, self.num_layers, self.num_heads, self.num_kv_heads,
         self.qk_head_dim, self.v_head_dim, self.max_seq_len) = (int(v) for v in dims)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None

    def session(self):
        return Session(self)

    def has_head(self, code):
        return lib().orc_head_present(self._h, code) == 1

    def embed(self, ids):
        """heads.rs:77-90 over a fresh session fed ids (needle_embed's
        computation after tokenizing)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        dim = lib().orc_embed(self._h, _p(ids), len(ids), None)
        if dim < 0:
            raise RuntimeError(lib().orc_last_error().decode())
        out = np.zeros(dim, np.float32)
        lib().orc_embed(self._h, _p(ids), len(ids), _p(out))
        return out

    def confidence(self, ids):
        """heads.rs:68-74."""
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(1, np.float32)
        if lib().orc_confidence(self._h, _p(ids), len(ids), _p(out)) != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return out[0]

    def cells(self, ids):
        """infer.rs:1195-1211: [t, L + 1, d] lane means of a fresh session."""
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros((len(ids), self.num_layers + 1, self.d_model), np.float32)
        if lib().orc_cells(self._h, _p(ids), len(ids), _p(out)) != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return out

    def gather(self, ids):
        """qlinear.rs:309-323 (QMat::row) of the embedding for each id."""
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros((len(ids), self.d_model), np.float32)
        if lib().orc_op_gather(self._h, _p(ids), len(ids), _p(out)) != 0:
            raise RuntimeError("id outside the vocabulary")
        return out

    def head_logits(self, h):
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros(self.out_rows, np.float32)
        lib().orc_head_logits(self._h, _p(h), _p(out))
        return out

    def head_logits_sparse(self, h, ids):
        h = np.ascontiguousarray(h, np.float32)
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(self.out_rows, np.float32)
        lib().orc_head_logits_sparse(self._h, _p(h), _p(ids), len(ids), _p(out))
        return out

    def generate(self, prompt, steps, masks=None, want_logits=False):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(steps, np.uint32)
        first = np.zeros(self.out_rows, np.float32) if want_logits else None
        rc = lib().orc_generate(self._h, _p(prompt), len(prompt), steps,
                                _p(np.ascontiguousarray(masks, np.uint8)) if masks is not None else None,
                                _p(out), _p(first) if first is not None else None)
        if rc != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return (out, first) if want_logits else out

    def generate_batch(self, prompts, steps, masks=None, threads=None):
        prompts = np.ascontiguousarray(prompts, np.uint32)
        S, n = prompts.shape
        out = np.zeros((S, steps), np.uint32)
        threads = threads or os.cpu_count() or 1
        rc = lib().orc_generate_batch(self._h, S, _p(prompts), n, steps,
                                      _p(np.ascontiguousarray(masks, np.uint8)) if masks is not None else None,
                                      _p(out), threads)
        if rc != 0:
            raise RuntimeError("oracle batch generation failed")
        return out

    def prefill_batch(self, prompts, threads=None, want_logits=True):
        prompts = np.ascontiguousarray(prompts, np.uint32)
        S, n = prompts.shape
        out = np.zeros((S, self.out_rows), np.float32) if want_logits else None
        threads = threads or os.cpu_count() or 1
        rc = lib().orc_prefill_batch(self._h, S, _p(prompts), n, _p(out) if out is not None else None, threads)
        if rc != 0:
            raise RuntimeError("oracle batch prefill failed")
        return out


class Batch:
    """S oracle sessions stepped together on host threads (the CPU baseline
    of the batched decode config)."""

    def __init__(self, model: Model, num_seqs: int, threads=None):
        self.model = model
        self.num_seqs = num_seqs
        self.threads = threads or os.cpu_count() or 1
        self._h = lib().orc_batch_new(model._h, num_seqs)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_batch_free(self._h)
            self._h = None

    def prefill(self, prompts):
        prompts = np.ascontiguousarray(prompts, np.uint32)
        if lib().orc_batch_prefill(self._h, _p(prompts), prompts.shape[1], self.threads) != 0:
            raise RuntimeError("oracle batch prefill failed")

    def step(self, masks=None):
        out = np.zeros(self.num_seqs, np.uint32)
        m = _p(np.ascontiguousarray(masks, np.uint8)) if masks is not None else None
        if lib().orc_batch_step(self._h, m, _p(out), self.threads) != 0:
            raise RuntimeError("oracle batch step failed")
        return out


class Session:
    def __init__(self, model: Model, handle=None):
        self.model = model
        self._h = handle or lib().orc_session_new(model._h)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_session_free(self._h)
            self._h = None

    def clone(self):
        return Session(self.model, lib().orc_session_clone(self._h))

    def __len__(self):
        return lib().orc_session_len(self._h)

    def set_attend(self, sink, ring):
        lib().orc_session_set_attend(self._h, sink, ring)

    def rollback(self, n):
        """model.rs:81-113."""
        if lib().orc_session_rollback(self.model._h, self._h, n) != 0:
            raise RuntimeError(lib().orc_last_error().decode())

    def rewind_zeroed(self, length):
        """model.rs:116-126."""
        lib().orc_session_rewind_zeroed(self.model._h, self._h, length)

    def truncate(self, length):
        """model.rs:128-145."""
        if lib().orc_session_truncate(self.model._h, self._h, length) != 0:
            raise RuntimeError(lib().orc_last_error().decode())

    def forward(self, ids, outputs=OUT_LAST_LOGITS):
        ids = np.ascontiguousarray(ids, np.uint32)
        n = len(ids)
        m = self.model
        rows = {OUT_NONE: 0, OUT_LAST_LOGITS: 1, OUT_LAST_HIDDEN: 1, OUT_ALL_LOGITS: n, OUT_HIDDEN: n}[outputs]
        width = m.d_model if outputs in (OUT_LAST_HIDDEN, OUT_HIDDEN) else m.out_rows
        out = np.zeros((rows, width), np.float32)
        rc = lib().orc_forward(m._h, self._h, _p(ids), n, outputs, _p(out))
        if rc < 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return out

    def last_hidden(self):
        out = np.zeros(self.model.d_model, np.float32)
        lib().orc_last_hidden(self._h, _p(out))
        return out


class trace:
    """Record the oracle's named intermediates (per layer ``L{l}.{name}``)."""

    def __enter__(self):
        lib().orc_trace(1)
        return self

    def __exit__(self, *a):
        lib().orc_trace(0)

    @staticmethod
    def get(name):
        n = lib().orc_trace_get(name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.zeros(n, np.float32)
        lib().orc_trace_get(name.encode(), _p(out), n)
        return out
