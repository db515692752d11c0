"""Helpers shared by the parity tests: bit-exact comparison and a report
of the first intermediate buffer where the GPU leaves the oracle."""

import numpy as np


def bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def describe_diff(name, got, want):
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    if got.shape != want.shape:
        return f"{name}: shape {got.shape} vs {want.shape}"
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    if len(bad) == 0:
        return f"{name}: identical"
    k = bad[0]
    rel = np.max(np.abs(got - want)) / max(1e-30, float(np.max(np.abs(want))))
    return f"{name}: {len(bad)}/{len(got)} differ, first at {k}: {got[k]!r} vs {want[k]!r}; max rel {rel:.3g}"


def first_divergence(gpu_model, oracle_model, ids):
    """Run one chunk (ids [t], t <= 32) on a fresh session of each and name
    the first per-layer buffer that differs."""
    from oracle import oracle as orc

    t = len(ids)
    lines = []
    with orc.trace():
        s = oracle_model.session()
        s.forward(np.asarray(ids, np.uint32), orc.OUT_LAST_LOGITS)
        tr = {}
        for l in range(oracle_model.num_layers):
            for n in ("u", "p", "x1", "proj", "qkv", "att", "o", "xs"):
                tr[f"L{l}.{n}"] = orc.trace.get(f"L{l}.{n}")
    for l in range(oracle_model.num_layers):
        b = gpu_model.batch(1, max(64, t))
        b.debug_layer(l)
        b.forward(np.asarray(ids, np.int32).reshape(1, t))
        pairs = [
            ("u", b.debug("snap.u"), tr[f"L{l}.u"]),
            ("x1", b.debug("snap.x1"), tr[f"L{l}.x1"]),
            ("proj", b.debug("snap.proj"), tr[f"L{l}.proj"]),
            ("q", b.debug("snap.qbuf").reshape(t, 576), tr[f"L{l}.qkv"].reshape(t, 800)[:, :576]),
            ("att", b.debug("snap.att"), tr[f"L{l}.att"]),
            ("o", b.debug("snap.o"), tr[f"L{l}.o"]),
            ("xs", b.debug("snap.xs"), tr[f"L{l}.xs"]),
        ]
        for name, g, w in pairs:
            if not bits_equal(g, w):
                lines.append(f"layer {l} " + describe_diff(name, g, w))
                return "\n".join(lines)
        lines.append(f"layer {l}: all buffers identical")
        del b
    return "\n".join(lines)
