"""A second, pure-Python restatement of a few reference functions, used only
on small inputs to pin the C++ oracle: every f32 op is one numpy float32 op,
and fused multiply-adds are rounded once from the exact rational value.

Citations are needle-rs paths (crates/needle-engine/src/...).
"""

from fractions import Fraction

import numpy as np

f32 = np.float32


def round_f32(x: Fraction) -> np.float32:
    """The float32 nearest to the exact rational x, ties to even."""
    if x == 0:
        return f32(0.0)
    d = f32(float(x))  # within one float32 ulp of the answer
    best = None
    for c in (np.nextafter(d, f32(-np.inf)), d, np.nextafter(d, f32(np.inf))):
        if not np.isfinite(c):
            continue
        err = abs(Fraction(float(c)) - x)
        if best is None or err < best[0] or (err == best[0] and (int(c.view(np.uint32)) & 1) == 0):
            best = (err, c)
    return f32(best[1])


def fma32(a, b, c) -> np.float32:
    return round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def dot16(x, y):
    """infer.rs:405-416 (scalar arm)."""
    a = [[f32(0)] * 4 for _ in range(4)]
    for c in range(len(x) // 16):
        for j in range(4):
            for l in range(4):
                i = c * 16 + j * 4 + l
                a[j][l] = fma32(x[i], y[i], a[j][l])
    t = [((a[2][l] + a[3][l]) + a[1][l]) + a[0][l] for l in range(4)]
    return (t[0] + t[1]) + (t[2] + t[3])


def bits(u):
    return np.array([u], np.uint32).view(np.float32)[0]


def nexp(x):
    """infer.rs:353-366."""
    x = f32(min(max(f32(x), bits(0xC2B0C0A5)), bits(0x42B0C0A5)))
    k = f32(np.rint(x * bits(0x3FB8AA3B)))
    r = fma32(k, bits(0xBF318000), x)
    r = fma32(k, bits(0x395E8083), r)
    p = fma32(bits(0x39506967), r, bits(0x3AB743CE))
    p = fma32(r, p, bits(0x3C088908))
    p = fma32(r, p, bits(0x3D2AA9C1))
    p = fma32(r, p, bits(0x3E2AAAAA))
    p = fma32(r, p, f32(0.5))
    y = fma32(r * r, p, r)
    s = np.array([((int(k) << 23) + 0x3F800000) & 0xFFFFFFFF], np.uint32).view(np.float32)[0]
    return fma32(s, y, s)


K127 = bits(0x3C010204)


def quant_i8(x):
    """qlinear.rs:77-88, 137-139."""
    x = np.asarray(x, np.float32)
    m = f32(0)
    for v in x:
        m = max(m, abs(v))
    s = m * K127 if m > 0 else f32(1.0)
    inv = f32(1.0) / s
    q = []
    for v in x:
        t = float(v * inv)
        r = np.floor(abs(t) + 0.5) * np.sign(t)  # half away from zero
        q.append(int(min(max(r, -128), 127)))
    return np.array(q, np.int8), f32(s)


def fwht(x):
    x = list(np.asarray(x, np.float32))
    n = len(x)
    h = 1
    while h < n:
        for i in range(0, n, 2 * h):
            for j in range(i, i + h):
                a, b = x[j], x[j + h]
                x[j], x[j + h] = a + b, a - b
        h *= 2
    return x


def rotate(x):
    s = f32(1.0 / np.sqrt(len(x)))
    return np.array([v * s for v in fwht(x)], np.float32)


def prep_group(x, g):
    """qlinear.rs:152-164, natural order."""
    buf = np.zeros(128, np.float32)
    seg = np.asarray(x[g * 128:(g + 1) * 128], np.float32)
    buf[:len(seg)] = seg
    return quant_i8(rotate(buf))


def int8_codebook(cb):
    """qlinear.rs:211-216."""
    m = f32(0)
    for v in cb:
        m = max(m, abs(f32(v)))
    s = m * K127 if m > 0 else f32(1.0)
    inv = f32(1.0) / s
    out = []
    for v in cb:
        t = float(f32(v) * inv)
        out.append(int(min(max(np.floor(abs(t) + 0.5) * np.sign(t), -128), 127)))
    return out, f32(s)


TERNARY = 5  # quant.rs:11-12


def code_width(bits):
    return 2 if bits == TERNARY else bits


def unpack_lsb(codes_row, width):
    """quant.rs:208-225: 8 codes per `width` bytes, LSB-first."""
    c = np.asarray(codes_row, np.uint8)
    out = []
    for k in range(0, len(c), width):
        word = 0
        for b in range(width):
            word |= int(c[k + b]) << (8 * b)
        out += [(word >> (i * width)) & ((1 << width) - 1) for i in range(8)]
    return np.array(out, np.int64)


def unpack4(codes_row):
    return unpack_lsb(codes_row, 4)


def code_table(cb, bits):
    """qlinear.rs:222-227, 244-256: code -> int8 value (ternary codes 3, 0,
    1 select centroids 0, 1, 2; codes past the codebook read 0)."""
    vals, cbs = int8_codebook(cb)
    width = code_width(bits)
    table = []
    for c in range(1 << width):
        k = (0 if c == 3 else c + 1) if bits == TERNARY else c
        table.append(vals[k] if k < len(vals) else 0)
    return table, cbs


def act_pos(p, width):
    """qlinear.rs:145-147."""
    return (p % 4) * 32 + p // 4 if width == 2 else (p % 2) * 64 + p // 2


def lane_sums(codes, table, q, width, g):
    """qlinear.rs:327-337, literally: the group's activations stored at
    act_pos, lane (p % 64) / 16 for width 2, (p % 32) / 8 otherwise."""
    xq = [0] * 128
    for p in range(128):
        xq[act_pos(p, width)] = int(q[p])
    s = [0, 0, 0, 0]
    for p in range(128):
        lane = (p % 64) // 16 if width == 2 else (p % 32) // 8
        s[lane] += table[codes[g * 128 + p]] * xq[act_pos(p, width)]
    return s


def _f16(n):
    return np.array([n], np.uint16).view(np.float16)[0].astype(np.float32)


def decode_row(codes_row, norms_row, x, cb, bits=4):
    """qlinear.rs:327-350: prep every group, the decode lane sums, the
    four-lane fma combine."""
    table, cbs = code_table(cb, bits)
    width = code_width(bits)
    codes = unpack_lsb(codes_row, width)
    lanes = [f32(0)] * 4
    for g in range(len(norms_row)):
        q, sx = prep_group(x, g)
        s = lane_sums(codes, table, q, width, g)
        sc = (sx * cbs) * _f16(norms_row[g])
        for l in range(4):
            lanes[l] = fma32(f32(s[l]), sc, lanes[l])
    return (lanes[0] + lanes[1]) + (lanes[2] + lanes[3])


def prefill_row(codes_row, norms_row, x, cb, block, bits=4):
    """qlinear.rs:353-363."""
    table, cbs = code_table(cb, bits)
    width = code_width(bits)
    codes = unpack_lsb(codes_row, width)
    acc = f32(0)
    for g in range(len(norms_row)):
        q, sx = prep_group(x, g)
        s = sum(lane_sums(codes, table, q, width, g))
        norm = _f16(norms_row[g])
        sc = (norm * cbs) * sx if block else norm * (cbs * sx)
        acc = fma32(f32(s), sc, acc)
    return acc


def lexpf(x):
    return f32(np.exp(np.float64(f32(x))))


def chunk_exp(s, m):
    """infer.rs:2279-2317 (scalar arm)."""
    s = list(np.asarray(s, np.float32))
    l, i = len(s), 0
    a = [f32(0)] * 4
    b = [f32(0)] * 4
    while i + 8 <= l:
        for k in range(4):
            e = nexp(s[i + k] - f32(m)); s[i + k] = e; a[k] = a[k] + e
        for k in range(4):
            e = nexp(s[i + 4 + k] - f32(m)); s[i + 4 + k] = e; b[k] = b[k] + e
        i += 8
    while i + 4 <= l:
        for k in range(4):
            e = nexp(s[i + k] - f32(m)); s[i + k] = e; a[k] = a[k] + e
        i += 4
    t = [a[k] + b[k] for k in range(4)]
    total = (t[0] + t[1]) + (t[2] + t[3])
    if l - i >= 2:
        e0, e1 = lexpf(s[i] - f32(m)), lexpf(s[i + 1] - f32(m))
        s[i], s[i + 1] = e0, e1
        total = (e0 + total) + e1
        i += 2
    if l - i == 1:
        e = lexpf(s[i] - f32(m)); s[i] = e; total = total + e
    return np.array(s, np.float32), total


def key_chunks(n, nested, nkv):
    """infer.rs:2093-2101."""
    k = 1 if nested else max(1, 2 * 4 // nkv)
    c = -(-n // 256)
    if k * 64 <= n and c < k:
        c = k
    chunk = -(-(-(-n // max(c, 1))) // 16) * 16
    return (-(-n // chunk) if chunk else 0), chunk


def sinkhorn64(z):
    """infer.rs:2501-2525."""
    z = np.asarray(z, np.float32)
    e = [0.0] * 16
    for r in range(4):
        m = float(max(max(z[r * 4], z[r * 4 + 1]), max(z[r * 4 + 2], z[r * 4 + 3])))
        for c in range(4):
            e[r * 4 + c] = float(np.exp(np.float64(z[r * 4 + c]) - m))
    for _ in range(20):
        for r in range(4):
            inv = 1.0 / ((e[r * 4] + e[r * 4 + 1]) + (e[r * 4 + 2] + e[r * 4 + 3]))
            for c in range(4):
                e[r * 4 + c] *= inv
        for c in range(4):
            inv = 1.0 / ((e[c] + e[4 + c]) + (e[8 + c] + e[12 + c]))
            for r in range(4):
                e[r * 4 + c] *= inv
    return np.array(e, np.float32)


def engine_expf(x):
    """agent.rs:1130-1145."""
    x = f32(min(max(f32(x), f32(-88.37626)), f32(88.37626)))
    n = f32(np.rint(x * f32(1.4426950408889634)))
    x = fma32(n, f32(-0.6933594), x)
    x = fma32(n, f32(2.1219444e-4), x)
    p = f32(1.9875691e-4)
    for c in (1.3981999e-3, 8.333452e-3, 4.1665796e-2, 1.6666665e-1, 0.5):
        p = fma32(p, x, f32(c))
    y = fma32(x * x, p, x)
    two_n = np.array([((int(n) + 127) << 23) & 0xFFFFFFFF], np.uint32).view(np.float32)[0]
    return fma32(two_n, y, two_n)


def softmax_stats(x):
    """agent.rs:1241-1252 with lane_exp_sums' scalar arm (1189-1197)."""
    x = np.asarray(x, np.float32)
    m = f32(-np.inf)
    for v in x:  # f32::max on aarch64 (FMAXNM): -0 < +0
        m = v if (v > m or (v == m and not np.signbit(v))) else m
    main = len(x) // 4 * 4
    lanes = [f32(0)] * 4
    for i in range(0, main, 4):
        for j in range(4):
            lanes[j] = f32(lanes[j] + engine_expf(f32(x[i + j] - m)))
    z = float(f32((lanes[0] + lanes[1]) + (lanes[2] + lanes[3])))
    for v in x[main:]:
        if v > f32(-1e30):
            z += float(np.exp(np.float64(v) - np.float64(m)))
    return m, z


def candidate_order(x, k):
    """agent.rs:335-343."""
    x = np.asarray(x, np.float32)
    order = [i for i in range(len(x)) if x[i] > f32(-1e30)]
    order.sort(key=lambda i: (-float(x[i]), i))
    return order[:k], len(order)


def fast_exp(x):
    """linalg.rs:262-277 (round half away, unfused)."""
    x = f32(min(max(f32(x), f32(-87.33654)), f32(88.72283)))
    t = f32(x * f32(1.4426950408889634))
    k = f32(np.floor(abs(t) + 0.5) * np.sign(t))
    r = f32(f32(x - f32(k * f32(0.6933594))) - f32(k * f32(-2.1219444e-4)))
    p = f32(1.9875691e-4)
    for c in (1.3981999e-3, 8.333452e-3, 4.1665796e-2, 1.6666665e-1, 5e-1):
        p = f32(f32(p * r) + f32(c))
    y = f32(f32(f32(f32(p * r) * r) + r) + f32(1.0))
    two = np.array([((int(k) + 127) << 23) & 0xFFFFFFFF], np.uint32).view(np.float32)[0]
    return f32(y * two)


def dot8(a, b):
    """linalg.rs:242-257."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    acc = [f32(0)] * 8
    ch = len(a) // 8
    for c in range(ch):
        for i in range(8):
            acc[i] = f32(acc[i] + f32(a[c * 8 + i] * b[c * 8 + i]))
    s = f32(f32(f32(f32(acc[0] + acc[4]) + f32(acc[1] + acc[5])) + f32(acc[2] + acc[6])) + f32(acc[3] + acc[7]))
    for i in range(ch * 8, len(a)):
        s = f32(s + f32(a[i] * b[i]))
    return s


def softmax_inplace(x):
    """linalg.rs:309-323 (max as aarch64 FMAXNM)."""
    m = f32(-np.inf)
    for v in x:
        m = v if (v > m or (v == m and not np.signbit(v))) else m
    if m == -np.inf:
        return [f32(0)] * len(x)
    e = [f32(0) if v == -np.inf else fast_exp(f32(v - m)) for v in x]
    s = f32(0)
    for v in e:
        s = f32(s + v)
    inv = f32(f32(1.0) / s)
    return [f32(v * inv) for v in e]


def rms_unit(x):
    """linalg.rs:291-297."""
    ss = f32(0)
    for v in x:
        ss = f32(ss + f32(v * v))
    ms = f32(ss / f32(len(x)))
    r = f32(f32(1.0) / np.sqrt(f32(ms + f32(1e-6))))
    return [f32(v * r) for v in x]


def probe_pool(cells, probes, gain, query, row_bias):
    """heads.rs:12-56."""
    cells = np.asarray(cells, np.float32)
    t, l1, d = cells.shape
    k, q = gain.shape[1], query.shape[0]
    inv = f32(f32(1.0) / f32(np.sqrt(np.float64(d))))
    m = l1 * k
    r = []
    for lk in range(m):
        l = lk // k
        probe = probes.reshape(m, d)[lk]
        scores = softmax_inplace([f32(dot8(cells[ti, l], probe) * inv) for ti in range(t)])
        acc = [f32(0)] * d
        for ti in range(t):
            for c in range(d):
                acc[c] = f32(acc[c] + f32(scores[ti] * cells[ti, l, c]))
        g = gain.reshape(-1)[lk]
        r.append([f32(v * g) for v in rms_unit(acc)])
    out = []
    for qi in range(q):
        u = softmax_inplace([f32(f32(dot8(r[j], query[qi]) * inv) + row_bias.reshape(q, m)[qi, j]) for j in range(m)])
        dst = [f32(0)] * d
        for j in range(m):
            for c in range(d):
                dst[c] = f32(dst[c] + f32(u[j] * r[j][c]))
        out += dst
    return np.array(out, np.float32)


INV_SQRT_QK = bits(0x3E13CD3A)
Q21 = bits(0x49FFFFF8)
C21 = bits(0x35000004)


def round_away(v):
    """Rust's f32::round on a finite value: half away from zero."""
    t = float(v)
    return int(np.floor(abs(t) + 0.5) * np.sign(t))


def attend_head(k8, ks, v8, vs, q, kvh, slots, nested):
    """infer.rs:1871-2004 (attend_head_ref): the int8 query, the key chunks,
    per chunk the scores ((ks * dot) * qs for the block keys, (ks * qs) * dot
    for the last len % 4), chunk_exp, the value-scaled weights, the 21-bit
    digits (2208-2214), the digit planes' integer P.V sums and their fma
    combine, then the merge of the chunks. Caches k8 [slot][nkv][qk], v8
    [slot][nkv][vd], ks / vs [slot][nkv] (the reference keeps V transposed;
    the integer sums are the same)."""
    nkv = k8.shape[1]
    vd = v8.shape[2]
    q8, s = quant_i8(q)
    qs = f32(s * INV_SQRT_QK)
    n = len(slots)
    _, chunk = key_chunks(n, nested, nkv)
    parts = []
    for c0 in range(0, n, chunk):
        sl = list(slots[c0:c0 + chunk])
        ln = len(sl)
        blocked = ln // 4 * 4
        dots = [int(np.dot(q8.astype(np.int64), k8[p, kvh].astype(np.int64))) for p in sl]
        sc = [f32(ks[p, kvh]) for p in sl]
        sv = [f32(f32(sc[i] * f32(dots[i])) * qs) if i < blocked else f32(f32(sc[i] * qs) * f32(dots[i]))
              for i in range(ln)]
        m = f32(-np.inf)
        for v in sv:
            m = max(m, v)
        e, total = chunk_exp(sv, m)
        w = [f32(e[i] * f32(vs[sl[i], kvh])) for i in range(ln)]
        wmax = f32(0)
        for v in w:
            wmax = max(wmax, v)
        qw = f32(Q21 / wmax)
        wq = [round_away(f32(w[i] * qw)) for i in range(ln)]
        hi = np.array([v >> 14 for v in wq], np.int64)
        mid = np.array([(v >> 7) & 127 for v in wq], np.int64)
        lo = np.array([v & 127 for v in wq], np.int64)
        cw = f32(wmax * C21)
        vals = v8[sl, kvh, :].astype(np.int64)
        sh, sm, sl_ = hi @ vals, mid @ vals, lo @ vals
        o = [f32(fma32(f32(16384), f32(sh[d]), fma32(f32(128), f32(sm[d]), f32(sl_[d]))) * cw) for d in range(vd)]
        parts.append((m, total, o))
    if len(parts) == 1:
        _, total, o = parts[0]
        inv = f32(f32(1) / total)
        return np.array([f32(v * inv) for v in o], np.float32)
    big = f32(-1e30)
    for m, _, _ in parts:
        big = max(big, m)
    acc = [f32(0)] * vd
    total = f32(0)
    for m, sm_, o in parts:
        wgt = lexpf(f32(m - big))
        acc = [fma32(o[d], wgt, acc[d]) for d in range(vd)]
        total = fma32(wgt, sm_, total)
    inv = f32(f32(1) / total)
    return np.array([f32(a * inv) for a in acc], np.float32)


def cond_weights(h2, cond_v):
    """infer.rs:1640-1694 (scalar arm): logits in four accumulator sets by
    j % 4 (fma chains over j), ((C + D) + B) + A, then the softmax with the
    engine's sum tree."""
    acc = [[f32(0)] * 8 for _ in range(4)]
    for j, hv in enumerate(h2):
        for k in range(8):
            acc[j % 4][k] = fma32(hv, cond_v[j * 8 + k], acc[j % 4][k])
    lg = [((acc[2][k] + acc[3][k]) + acc[1][k]) + acc[0][k] for k in range(8)]
    m = f32(-np.inf)
    for v in lg:
        m = max(m, v)
    e = [lexpf(f32(v - m)) for v in lg]
    total = e[7] + ((e[6] + (e[5] + e[4])) + ((e[3] + e[2]) + (e[1] + e[0])))
    inv = f32(f32(1) / total)
    return [f32(v * inv) for v in e]


def mix8(ct, rows, transpose):
    """infer.rs:2343-2460 (scalar arm 2442-2459): out[r][c] = sum over j of
    ct[j][r] * rows[j][c], an fma chain over j from 0; with transpose the
    value lands at out[c][r]."""
    out = [f32(0)] * 1024
    for r in range(32):
        for c in range(32):
            o = f32(0)
            for j in range(32):
                o = fma32(ct[j * 32 + r], rows[j * 32 + c], o)
            out[c * 32 + r if transpose else r * 32 + c] = o
    return out


def kron_native(z, a, b):
    """infer.rs:2322-2330."""
    return mix8(mix8(a, z, True), b, False)


def mlp_native(h2, d1, d2, b2, d3, d4, kron, cond_v, cond_u, perm1, perm2):
    """infer.rs:1610-1634, with axpy16 (494-528), perm_fma (689-713) and
    silu_native (2463-2496) in their scalar forms."""
    h2 = [f32(v) for v in h2]
    d = len(h2)
    w = cond_weights(h2, cond_v)
    z = [f32(0)] * 1024
    for j in range(d):
        z[j] = f32(h2[j] * f32(d1[j]))
    t = kron_native(z, kron[0], kron[1])
    cond = [f32(1)] * 1024
    for k in range(8):
        for i in range(1024):
            cond[i] = fma32(f32(cond_u[k * 1024 + i]), w[k], cond[i])
    z = [fma32(t[perm1[j]], f32(cond[j] * f32(d2[j])), f32(b2[j])) for j in range(1024)]
    z = [f32(v / f32(nexp(f32(-v)) + f32(1))) for v in z]
    t = kron_native(z, kron[2], kron[3])
    z = [f32(t[perm2[j]] * f32(d3[j])) for j in range(1024)]
    t = kron_native(z, kron[4], kron[5])
    return np.array([f32(t[j] * f32(d4[j])) for j in range(d)], np.float32)


def rinv(ss, n):
    """infer.rs:420-422: 1 / sqrtf(ss / n + 1e-6)."""
    return f32(f32(1) / np.sqrt(f32(f32(ss) / f32(n)) + f32(1e-6)))


def zcn(x, s):
    """infer.rs:425-443 (scalar arm): t = x * r, out = fma(t, s, t)."""
    r = rinv(dot16(x, x), len(x))
    out = []
    for v, w in zip(x, s):
        t = f32(f32(v) * r)
        out.append(fma32(t, f32(w), t))
    return out


def mhc_read_row(x, phi_q, phi_s, a_pre, b_pre, lane):
    """infer.rs:1359-1393 for one row: the lanes normalised by one rms, int8
    without rotation, the gate projections (int8 dots), the pre gates (own
    lane +4, the others -4), the block input u."""
    x = [f32(v) for v in x]
    nc = len(x)
    d = nc // 4
    r = rinv(dot16(x, x), nc)
    q8, sx = quant_i8([f32(v * r) for v in x])
    q8 = q8.astype(np.int64)
    p = [f32(f32(sx * f32(phi_s[k])) * f32(int(np.dot(np.asarray(phi_q[k], np.int64), q8)))) for k in range(len(phi_s))]
    hp = []
    for j in range(4):
        off = f32(4.0) if j == lane else f32(-4.0)
        z = f32(f32(f32(p[j] * f32(a_pre)) + off) + f32(b_pre[j]))
        hp.append(f32(f32(1) / f32(lexpf(f32(-z)) + f32(1))))
    u = [f32(x[k] * hp[0]) for k in range(d)]
    for b in range(1, 4):
        u = [fma32(x[b * d + k], hp[b], u[k]) for k in range(d)]
    return p, u


def gate_norm_row(u, norm_in, kr=None, vr=None):
    """infer.rs:1397-1418 for one row: the engram gate (the site's key and
    value rows), then the input ZC-RMSNorm. Returns (x1, h)."""
    xr = [f32(v) for v in u]
    d = len(xr)
    if kr is not None:
        kr = [f32(v) for v in kr]
        rx, rk = rinv(dot16(xr, xr), d), rinv(dot16(kr, kr), d)
        a = [f32(v * rx) for v in xr]
        b = [f32(v * rk) for v in kr]
        alpha = f32(f32(1) / f32(lexpf(f32(f32(-dot16(a, b)) / np.sqrt(f32(d)))) + f32(1)))
        xr = [fma32(f32(vr[k]), alpha, xr[k]) for k in range(d)]
    return xr, zcn(xr, norm_in)


def post_row(x, o, x1, pr, u, lane, post_norm, pre_hada, attn_gate, a_post, b_post, a_res, b_res, mlp_weights):
    """infer.rs:1564-1606 for one row: the gated residual x2, the pre-MLP
    norm, the MLP, the post gates (own lane 0, others -4), the residual gates
    through Sinkhorn, then the mHC write of each lane from y = (x2 + mlp) - u
    and the old lanes. Returns (the new lanes, the MLP output)."""
    x = [f32(v) for v in x]
    d = len(x) // 4
    ga = f32(f32(1) / f32(lexpf(f32(-f32(attn_gate))) + f32(1)))
    on = zcn(o, post_norm)
    x2 = [fma32(on[k], ga, f32(x1[k])) for k in range(d)]
    h2 = zcn(x2, pre_hada)
    mlp = mlp_native(h2, *mlp_weights)
    hpost = []
    for j in range(4):
        off = f32(0.0) if j == lane else f32(-4.0)
        z = f32(f32(f32(f32(pr[4 + j]) * f32(a_post)) + off) + f32(b_post[j]))
        hpost.append(f32(f32(2) / f32(lexpf(f32(-z)) + f32(1))))
    zres = [fma32(f32(pr[8 + k]), f32(a_res), f32(b_res[k])) for k in range(16)]
    hres = sinkhorn64(zres)
    y = [f32(f32(x2[ch] + mlp[ch]) - f32(u[ch])) for ch in range(d)]
    new = list(x)
    for a in range(4):
        for ch in range(d):
            v = f32(y[ch] * hpost[a])
            for b in range(4):
                v = fma32(x[b * d + ch], f32(hres[a * 4 + b]), v)
            new[a * d + ch] = v
    return np.array(new, np.float32), mlp


def conv_rope_row(rows, q_taps, k_taps, v_taps, q_norm, k_norm, cs, sn, nh=12, nkv=2, qk=48, vd=64):
    """infer.rs:1437-1486 for one row: each of q | k | v through its three
    conv taps (o = w0 * x0, then fma over the taps; a missing row before
    position 0 multiplies zero), then each q and k head's zcn_inplace and
    RoPE: x[f] = fma(-sin, x[f + half], cos * x[f]), x[f + half] =
    fma(sin, x[f], cos * x[f + half])."""
    qd, kd, vdim, half = nh * qk, nkv * qk, nkv * vd, qk // 2
    out = [f32(0)] * (qd + kd + vdim)
    for start, cw, w in ((0, qd, q_taps), (qd, kd, k_taps), (qd + kd, vdim, v_taps)):
        w = np.asarray(w, np.float32).reshape(3, cw)
        o = [f32(w[0][k] * f32(rows[0][start + k])) for k in range(cw)]
        for j in (1, 2):
            r = rows[j]
            o = [fma32(w[j][k], f32(r[start + k]) if r is not None else f32(0), o[k]) for k in range(cw)]
        out[start:start + cw] = o
    for hh in range(nh + nkv):
        off = hh * qk if hh < nh else qd + (hh - nh) * qk
        scale = q_norm if hh < nh else k_norm
        x = zcn(out[off:off + qk], scale)
        for f in range(half):
            a, b = x[f], x[f + half]
            x[f] = fma32(f32(-f32(sn[f])), b, f32(f32(cs[f]) * a))
            x[f + half] = fma32(f32(sn[f]), a, f32(f32(cs[f]) * b))
        out[off:off + qk] = x
    return np.array(out, np.float32)


def rope_tables(theta, qk):
    """infer.rs:938-946: freq = powf(theta, i * (-2 / qk)) (libm on f64,
    rounded once), and its sine and cosine."""
    import math

    coef = f32(f32(-2.0) / f32(qk))
    freq = [f32(math.pow(float(f32(theta)), float(f32(f32(k) * coef)))) for k in range(qk // 2)]
    return freq, [f32(math.sin(float(f))) for f in freq], [f32(math.cos(float(f))) for f in freq]


def rope_rows(theta, qk, p0, n_prev, t):
    """infer.rs:1716-1744 for a session that fed n_prev single-token rows up
    to p0 - 1, then t rows from p0: a chunk (or a token with no newest row
    before it) takes sincosf(freq * pos); a single token right after the
    newest row takes the recurrence cos = fma(-sd, s0, cd * c0), sin =
    fma(sd, c0, cd * s0)."""
    import math

    freq, sd, cd = rope_tables(theta, qk)

    def direct(p):
        a = [float(f32(f * f32(p))) for f in freq]
        return [f32(math.cos(v)) for v in a], [f32(math.sin(v)) for v in a]

    def recur(c0, s0):
        return ([fma32(f32(-sd[f]), s0[f], f32(cd[f] * c0[f])) for f in range(len(freq))],
                [fma32(sd[f], c0[f], f32(cd[f] * s0[f])) for f in range(len(freq))])

    c = s = None
    if n_prev > 0:
        c, s = direct(p0 - n_prev)
        for _ in range(p0 - n_prev + 1, p0):
            c, s = recur(c, s)
    if t == 1 and n_prev > 0:
        c, s = recur(c, s)
        return np.array([c], np.float32), np.array([s], np.float32)
    rows = [direct(p0 + i) for i in range(t)]
    return np.array([r[0] for r in rows], np.float32), np.array([r[1] for r in rows], np.float32)


def engram_slot(tokens, pos, oi, order, h, stride, slots):
    """infer.rs:1262-1272: acc = SEED * (oi * stride + h + 1), then for each
    of the n-gram's tokens (newest first, 0 before position 0) acc = (acc ^
    tok) * PRIME, all mod 2^32; acc ^= acc >> 15; the slot is acc % slots
    (config.rs:11-12 for the constants)."""
    mask = 0xFFFFFFFF
    acc = (0x9E3779B9 * (oi * stride + h + 1)) & mask
    for j in range(order):
        tok = int(tokens[pos - j]) if pos >= j else 0
        acc = ((acc ^ tok) * 0x01000193) & mask
    acc ^= acc >> 15
    return acc % slots


def engram_conv(taps, v8, vs, pos, dil):
    """infer.rs:1307-1320 with engram_tap (667-687): tap j reads the int8
    history at pos - j * dil (stopping before position 0), dequantized per
    32-wide group, into an fma chain over the taps."""
    etaps, d = np.asarray(taps).shape
    dst = [f32(0)] * d
    for j in range(etaps):
        p = pos - j * dil
        if p < 0:
            break
        for ch in range(d):
            deq = f32(f32(vs[p][ch // 32]) * f32(int(v8[p][ch])))
            dst[ch] = fma32(f32(taps[j][ch]), deq, dst[ch])
    return np.array(dst, np.float32)
