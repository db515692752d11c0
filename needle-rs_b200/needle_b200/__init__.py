"""Python view of libneedle3.so, the B200 engine for Needle 3.

Mirrors the reference engine's model-level interface
(crates/needle-engine/src/model.rs: ``Model::{forward, prefill, session,
head_logits, head_logits_sparse}``, ``Session``) over the C ABI declared in
include/needle_engine.h, batched: a ``Batch`` is S sessions fed in lockstep.
There is no CPU fallback; importing fails if the CUDA library is missing.
"""

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libneedle3.so")

OUT_NONE, OUT_LAST_LOGITS, OUT_LAST_HIDDEN, OUT_ALL_LOGITS, OUT_HIDDEN = 0, 1, 2, 3, 4
SITES = dict(none=0, qkvg=1, out=2, lm_head=3, engram_kv=4, attention=5, post=6, mhc=7, conv=8)
ND_DEVICE = 1

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build()")
        L = C.CDLL(LIB_PATH)
        P, I, U64 = C.c_void_p, C.c_int, C.c_uint64
        sig = {
            "nd_last_error": (C.c_char_p, []),
            "nd_model_load": (I, [P, U64, I, C.POINTER(P)]),
            "nd_model_free": (None, [P]),
            "nd_model_dims": (I, [P, P]),
            "nd_batch_new": (I, [P, I, I, C.POINTER(P)]),
            "nd_batch_free": (None, [P]),
            "nd_batch_len": (I, [P]),
            "nd_batch_set_attend": (I, [P, I, I]),
            "nd_batch_rollback": (I, [P, I]),
            "nd_batch_rewind_zeroed": (I, [P, I]),
            "nd_batch_truncate": (I, [P, I]),
            "nd_batch_forward": (I, [P, P, I, I, P, I]),
            "nd_batch_step": (I, [P, P, P, I]),
            "nd_batch_last_hidden": (I, [P, P, I]),
            "nd_head_logits": (I, [P, P, I, P, I]),
            "nd_head_logits_sparse": (I, [P, P, P, I, P]),
            "nd_batch_stream": (P, [P]),
            "nd_batch_embed": (I, [P, P, I, P, C.POINTER(I), I]),
            "nd_batch_confidence": (I, [P, P, I, P, I]),
            "nd_batch_candidates": (I, [P, P, P, P, I, P, P, P, P, I]),
            "nd_cq_pack": (I, [P, I, I, I, P, P]),
            "nd_cqmat_new": (I, [I, P, P, I, I, I, C.POINTER(P)]),
            "nd_cqmat_free": (None, [P]),
            "nd_cqmat_apply": (I, [P, P, I, I, P, I, C.POINTER(C.c_float)]),
            "nd_cqmat_time_rotating": (I, [P, I, I, I, I, C.POINTER(C.c_float)]),
            "nd_op_zcn": (I, [P, P, I, P, P]),
            "nd_op_rope": (I, [P, I, C.c_float, P, P]),
            "nd_op_silu": (I, [P, C.c_longlong, P, P]),
            "nd_op_gather": (I, [P, P, I, P, P]),
            "nd_synth_cact": (I, [I, I, I, I, U64, U64, U64, C.c_float, P, I, C.c_uint, P, U64, C.POINTER(U64)]),
            "nd_batch_debug": (I, [P, C.c_char_p, P, C.c_longlong]),
            "nd_batch_debug_layer": (I, [P, I]),
            "nd_launch_count": (C.c_longlong, []),
            "nd_batch_time_site": (I, [P, I]),
            "nd_batch_site_time": (I, [P, C.POINTER(C.c_double), C.POINTER(I)]),
            "needle_load": (I, [P, U64]),
            "needle_init": (I, [C.c_char_p, C.c_char_p, C.c_char_p]),
            "needle_complete": (I, [C.c_char_p, I, P, I]),
            "needle_embed": (I, [C.c_char_p, P, I]),
            "needle_reset": (None, []),
            "needle_last_error": (C.c_char_p, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _err():
    return RuntimeError(lib().nd_last_error().decode(errors="replace"))


def _p(a):
    if a is None:
        return None
    if isinstance(a, int):
        return C.c_void_p(a)
    if hasattr(a, "data_ptr"):  # a torch tensor on the device
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


NEEDLE3_DEFAULTS = dict(num_layers=20, vocab=16384, engram_slots=18432, sliding_window=1024,
                        global_layers=(4, 9, 14, 19), engram_sites=(3, 7, 11, 15, 19))


def launch_count() -> int:
    """Kernel launches this process has issued through the engine."""
    return lib().nd_launch_count()


TERNARY = 5  # record bits of ternary codes (crates/needle-core/src/quant.rs:11-12)


def cq_roles(num_layers=20, engram_sites=(3, 7, 11, 15, 19), **_):
    """The CQ records of an archive in record order
    (crates/needle-core/src/cact.rs:279-352): embedding; per layer q, k, v,
    gate, out; phi_pre, phi_post, phi_res; per engram site table, key,
    value."""
    roles = ["embedding"]
    for _l in range(num_layers):
        roles += ["q", "k", "v", "gate", "out"]
    roles += ["phi_pre", "phi_post", "phi_res"]
    for _s in engram_sites:
        roles += ["table", "key", "value"]
    return roles


HEAD_EMBEDDING, HEAD_CONFIDENCE, HEAD_ROUTER = 1, 2, 3  # probe head codes (cact.rs:354-360)


def synth_cact(seed=0, std=0.02, bits=None, heads=(), **shape) -> bytes:
    """A random-init Needle 3 archive (every tensor ~N(0, std^2)), CQ
    matrices packed by the reference's quantizer, in the reference's record
    order (crates/needle-core/src/cact.rs:279-475). ``bits`` sets the record
    bits of the CQ matrices (2, 3, 4 or TERNARY): one width for all, a dict
    role -> width (roles as cq_roles names them, others 4), or a list in
    record order. A fused projection's parts (q, k, v, gate; key, value)
    must share the code width (ternary packs at 2). ``heads`` lists probe
    head codes to append (HEAD_EMBEDDING, HEAD_CONFIDENCE, HEAD_ROUTER)."""
    g = dict(NEEDLE3_DEFAULTS)
    g.update(shape)
    gm = sum(1 << l for l in g["global_layers"])
    es = sum(1 << l for l in g["engram_sites"])
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
    n = C.c_uint64(0)
    args = (g["num_layers"], g["vocab"], g["engram_slots"], g["sliding_window"], gm, es, seed, std,
            _p(plan) if len(plan) else None, len(plan), sum(1 << c for c in set(heads)))
    if lib().nd_synth_cact(*args, None, 0, C.byref(n)) != 0:
        raise _err()
    buf = np.zeros(n.value, np.uint8)
    if lib().nd_synth_cact(*args, _p(buf), n.value, C.byref(n)) != 0:
        raise _err()
    return buf.tobytes()


def code_width(bits):
    """Bits a code of a record takes in memory (ternary packs at 2)."""
    return 2 if bits == TERNARY else bits


class CQMat:
    """One CQ matrix (codes [out][6][16 * width], f16 norms [out][6]) of
    record bits 2, 3, 4 or TERNARY on a GPU: the engine's A8 + CQ matmul on
    host rows (needle_engine.h, nd_cqmat_apply)."""

    def __init__(self, codes, norms, device=0, bits=4):
        codes = np.ascontiguousarray(codes, np.uint8)
        norms = np.ascontiguousarray(norms, np.uint16)
        self.out = norms.shape[0]
        self.bits = bits
        if codes.size != self.out * 6 * 16 * code_width(bits):
            raise ValueError("codes do not match out x 6 groups at this width")
        h = C.c_void_p()
        if lib().nd_cqmat_new(device, _p(codes), _p(norms), self.out, 768, bits, C.byref(h)) != 0:
            raise _err()
        self._h = h.value

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().nd_cqmat_free(self._h)
                self._h = None
        except Exception:  # interpreter shutdown
            pass

    def __call__(self, x, T=1, reps=0):
        """y [M][out] for x [M][768]; with reps > 0 returns (y, ms per run)."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, 768)
        y = np.zeros((x.shape[0], self.out), np.float32)
        ms = C.c_float(0.0)
        if lib().nd_cqmat_apply(self._h, _p(x), x.shape[0], T, _p(y), reps, C.byref(ms)) != 0:
            raise _err()
        return (y, ms.value) if reps > 0 else y

    @staticmethod
    def time_rotating(mats, M, T=1, reps=10):
        """Mean ms per matmul launch over the CQMats in turn, back to back,
        on the activations of mats[0]'s last call (nd_cqmat_time_rotating):
        with the matrices together larger than L2 each launch reads its
        weights from HBM."""
        arr = (C.c_void_p * len(mats))(*[m._h for m in mats])
        ms = C.c_float(0.0)
        if lib().nd_cqmat_time_rotating(arr, len(mats), M, T, reps, C.byref(ms)) != 0:
            raise _err()
        return ms.value


def cq_pack(w, bits=4):
    """crates/needle-core/src/quant.rs:233-256 (group 128) at record bits 2,
    3, 4 or TERNARY."""
    w = np.ascontiguousarray(w, np.float32)
    rows, d = w.shape
    g = (d + 127) // 128
    codes = np.zeros((rows, g * 16 * code_width(bits)), np.uint8)
    norms = np.zeros((rows, g), np.uint16)
    if lib().nd_cq_pack(_p(w), rows, d, bits, _p(codes), _p(norms)) != 0:
        raise _err()
    return codes, norms


class Model:
    """A packed model resident on one GPU (`Model::quantized`)."""

    def __init__(self, archive: bytes, device: int = 0):
        buf = np.frombuffer(archive, np.uint8)
        h = C.c_void_p()
        if lib().nd_model_load(_p(buf), len(buf), device, C.byref(h)) != 0:
            raise _err()
        self._h = h
        self.device = device
        dims = np.zeros(9, np.int32)
        lib().nd_model_dims(self._h, _p(dims))
        (self.vocab, self.out_rows, self.d_model, self.num_layers, self.num_heads, self.num_kv_heads,
         self.qk_head_dim, self.v_head_dim, self.max_seq_len) = (int(v) for v in dims)

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().nd_model_free(self._h)
                self._h = None
        except Exception:  # interpreter shutdown
            pass

    def batch(self, num_seqs: int, max_len: int) -> "Batch":
        return Batch(self, num_seqs, max_len)

    def session(self, max_len: int = None) -> "Batch":
        """One sequence (`Model::session`)."""
        return Batch(self, 1, max_len or self.max_seq_len)


class Batch:
    """S sessions fed in lockstep on the model's GPU."""

    def __init__(self, model: Model, num_seqs: int, max_len: int):
        h = C.c_void_p()
        if lib().nd_batch_new(model._h, num_seqs, max_len, C.byref(h)) != 0:
            raise _err()
        self._h = h
        self.model = model
        self.num_seqs = num_seqs
        self.max_len = max_len

    def __del__(self):
        try:
            if getattr(self, "_h", None):
                lib().nd_batch_free(self._h)
                self._h = None
        except Exception:  # interpreter shutdown
            pass

    def __len__(self):
        return lib().nd_batch_len(self._h)

    def rollback(self, n):
        """Session::rollback for every sequence (model.rs:81-113)."""
        if lib().nd_batch_rollback(self._h, n) != 0:
            raise _err()

    def rewind_zeroed(self, length):
        """Session::rewind_zeroed for every sequence (model.rs:116-126)."""
        if lib().nd_batch_rewind_zeroed(self._h, length) != 0:
            raise _err()

    def truncate(self, length):
        """Session::truncate for every sequence (model.rs:128-145)."""
        if lib().nd_batch_truncate(self._h, length) != 0:
            raise _err()

    def set_attend(self, sink, ring):
        """Session::attend for every sequence (model.rs:63-66): the first
        `sink` positions and the ring of the last `ring`; ring 0 = none."""
        if lib().nd_batch_set_attend(self._h, sink, ring) != 0:
            raise _err()

    @property
    def stream(self) -> int:
        return lib().nd_batch_stream(self._h) or 0

    def forward(self, ids, outputs=OUT_LAST_LOGITS, out=None):
        """`Model::forward` for every sequence: ids [S, t] (host array, or a
        device tensor with ``out`` also on the device)."""
        m = self.model
        dev = hasattr(ids, "data_ptr")
        if dev:
            S, t = ids.shape
        else:
            ids = np.ascontiguousarray(ids, np.int32).reshape(self.num_seqs, -1)
            S, t = ids.shape
        rows = {OUT_NONE: 0, OUT_LAST_LOGITS: 1, OUT_LAST_HIDDEN: 1, OUT_ALL_LOGITS: t, OUT_HIDDEN: t}[outputs]
        width = m.d_model if outputs in (OUT_LAST_HIDDEN, OUT_HIDDEN) else m.out_rows
        if out is None and not dev and rows:
            out = np.zeros((S, rows, width), np.float32)
        rc = lib().nd_batch_forward(self._h, _p(ids), t, outputs, _p(out), ND_DEVICE if dev else 0)
        if rc < 0:
            raise _err()
        return out

    prefill = forward  # `Model::prefill` equals `forward` without an attention span

    def step(self, allow_bits=None, next_ids=None):
        """One greedy decode step: argmax of the last logits under the masks,
        fed back; returns the chosen ids [S]."""
        dev = next_ids is not None and hasattr(next_ids, "data_ptr")
        if next_ids is None:
            next_ids = np.zeros(self.num_seqs, np.int32)
        if allow_bits is not None and not dev:
            allow_bits = np.ascontiguousarray(allow_bits, np.uint8)
        if lib().nd_batch_step(self._h, _p(allow_bits), _p(next_ids), ND_DEVICE if dev else 0) != 0:
            raise _err()
        return next_ids

    def last_hidden(self):
        out = np.zeros((self.num_seqs, self.model.d_model), np.float32)
        if lib().nd_batch_last_hidden(self._h, _p(out), 0) != 0:
            raise _err()
        return out

    def head_logits(self, h):
        h = np.ascontiguousarray(h, np.float32).reshape(-1, self.model.d_model)
        out = np.zeros((h.shape[0], self.model.out_rows), np.float32)
        if lib().nd_head_logits(self._h, _p(h), h.shape[0], _p(out), 0) != 0:
            raise _err()
        return out

    def head_logits_sparse(self, h, ids):
        h = np.ascontiguousarray(h, np.float32)
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(self.model.out_rows, np.float32)
        if lib().nd_head_logits_sparse(self._h, _p(h), _p(ids), len(ids), _p(out)) != 0:
            raise _err()
        return out

    def embed(self, ids):
        """needle_embed's computation for every sequence of this fresh batch
        (heads.rs:63-90): ids [S, T]; returns [S, dim] unit vectors."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(self.num_seqs, -1)
        dim = C.c_int(0)
        if lib().nd_batch_embed(self._h, None, 0, None, C.byref(dim), 0) != 0:
            raise _err()
        out = np.zeros((self.num_seqs, dim.value), np.float32)
        if lib().nd_batch_embed(self._h, _p(ids), ids.shape[1], _p(out), C.byref(dim), 0) != 0:
            raise _err()
        return out

    def confidence(self, ids):
        """heads.rs:68-74 for every sequence of this fresh batch: [S]."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(self.num_seqs, -1)
        out = np.zeros(self.num_seqs, np.float32)
        if lib().nd_batch_confidence(self._h, _p(ids), ids.shape[1], _p(out), 0) != 0:
            raise _err()
        return out

    def candidates(self, allow=None, allow_order=None, k=128, logits=None):
        """The call step's start over the last logits, or over host
        ``logits`` [S][out_rows] (agent.rs:295-343): per sequence the first
        k candidates by (logit desc, id asc), -1 past the live count, and
        the softmax max and sum. Returns (ids [S][k], m [S], z [S], live
        [S])."""
        S = self.num_seqs
        ids = np.zeros((S, k), np.int32)
        m = np.zeros(S, np.float32)
        z = np.zeros(S, np.float64)
        live = np.zeros(S, np.int32)
        a1 = None if allow is None else np.ascontiguousarray(allow, np.uint8)
        a2 = None if allow_order is None else np.ascontiguousarray(allow_order, np.uint8)
        lg = None if logits is None else np.ascontiguousarray(logits, np.float32).reshape(S, self.model.out_rows)
        if lib().nd_batch_candidates(self._h, _p(lg), _p(a1), _p(a2), k, _p(ids), _p(m), _p(z), _p(live), 0) != 0:
            raise _err()
        return ids, m, z, live

    def time_site(self, site):
        """Record CUDA events around every launch of a site (see SITES)."""
        if lib().nd_batch_time_site(self._h, SITES[site] if isinstance(site, str) else site) != 0:
            raise _err()

    def site_time(self):
        """(summed kernel milliseconds, launches) of the timed site."""
        ms = C.c_double(0)
        n = C.c_int(0)
        if lib().nd_batch_site_time(self._h, C.byref(ms), C.byref(n)) != 0:
            raise _err()
        return ms.value, n.value

    def debug(self, name):
        n = lib().nd_batch_debug(self._h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.zeros(n, np.float32)
        lib().nd_batch_debug(self._h, name.encode(), _p(out), n)
        return out

    def debug_layer(self, layer):
        lib().nd_batch_debug_layer(self._h, layer)


# ------------------------------------------------------- standalone row ops


def _stream_of(t):
    import torch

    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def op_zcn(x, s, out=None):
    """infer.rs:426-443 on the GPU: rows x [T, 768] (a float32 CUDA tensor),
    weights s [768]; returns out [T, 768] (nd_op_zcn)."""
    import torch

    out = torch.empty_like(x) if out is None else out
    if lib().nd_op_zcn(_p(x), _p(s), x.shape[0], _p(out), _stream_of(x)) != 0:
        raise _err()
    return out


def op_rope(x, theta=100000.0, out=None):
    """RoPE at positions 0..T-1 of x [T, 672] (12 q heads, 2 k heads of 48)."""
    import torch

    out = torch.empty_like(x) if out is None else out
    if lib().nd_op_rope(_p(x), x.shape[0], theta, _p(out), _stream_of(x)) != 0:
        raise _err()
    return out


def op_silu(x, out=None):
    """silu_native elementwise over a float32 CUDA tensor."""
    import torch

    out = torch.empty_like(x) if out is None else out
    if lib().nd_op_silu(_p(x), x.numel(), _p(out), _stream_of(x)) != 0:
        raise _err()
    return out


def op_gather(model, ids, out=None):
    """QMat::row of the model's embedding for int32 CUDA ids [T]."""
    import torch

    T = ids.shape[0]
    out = torch.empty((T, model.d_model), dtype=torch.float32, device=ids.device) if out is None else out
    if lib().nd_op_gather(model._h, _p(ids), T, _p(out), _stream_of(ids)) != 0:
        raise _err()
    return out
