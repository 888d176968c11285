"""A step-for-step restatement, in numpy fp32, of the CTA's exact ordered sum
(ordered_sum_nonneg_cta): the fp32 prediction scans (Hillis-Steele within a
warp, then over the warp totals), the grid offsets rne(t/u) by the 1.5 * 2^23
add, ties and crossings counted in one 64-bit scan, warp 0's preparation of
each crossing's run (its offset and its ties' round-ups for either parity of
m), the walk over the crossings, and the fallbacks. Test infrastructure: it
lets the CPU suite check the algorithm on many inputs; the GPU tests check
the kernel itself."""
import numpy as np

F = np.float32
CMAX, TMAX = 64, 256


def fadd(a, b):
    return F(F(a) + F(b))


def field(v):
    return (int(F(v).view(np.uint32)) >> 23) & 0xFF


def sequential_from(t, s, start):
    for i in range(start, t.size):
        s = fadd(s, t[i])
    return s


def warp_inclusive_scan(vals):
    """Hillis-Steele over 32 lanes, each step lane l += lane l - o (fp32)."""
    inc = np.array(vals, dtype=F)
    for o in (1, 2, 4, 8, 16):
        nxt = inc.copy()
        for lane in range(o, 32):
            nxt[lane] = fadd(inc[lane], inc[lane - o])
        inc = nxt
    return inc


def model_sum(t, nt=512, ept_max=16):
    """(sum, path): the CTA's result for the non-negative terms t, and
    'fast', 'fallback' (walk gave up part way) or 'seq' (whole sequential)."""
    t = np.ascontiguousarray(t, dtype=F)
    n = t.size
    ept = (n + nt - 1) // nt
    with np.errstate(invalid="ignore"):
        bad = ept > ept_max or bool(np.any(~(t >= 0))) or bool(np.any(t > F(3.402823466e38)))
    if bad:
        return sequential_from(t, F(0), 0), "seq"
    nw = nt // 32
    v = np.zeros((nt, ept), dtype=F)
    for tid in range(nt):
        for k in range(ept):
            i = tid * ept + k
            if i < n:
                v[tid, k] = t[i]
    # 1. fp32 prediction: per-thread sums, warp scans, warp-total scans
    tsum = np.zeros(nt, dtype=F)
    for tid in range(nt):
        s = F(0)
        for k in range(ept):
            s = fadd(s, v[tid, k])
        tsum[tid] = s
    inc = np.stack([warp_inclusive_scan(tsum[w * 32:(w + 1) * 32]) for w in range(nw)])
    ex = np.zeros_like(inc)
    ex[:, 1:] = inc[:, :-1]
    wf = inc[:, 31].copy()
    woff_in = warp_inclusive_scan(np.concatenate([wf, np.zeros(32 - nw, dtype=F)]))
    X0 = np.zeros(nt, dtype=F)
    xnext = np.zeros(nt, dtype=F)
    for w in range(nw):
        w_start = woff_in[w - 1] if w else F(0)
        for lane in range(32):
            X0[w * 32 + lane] = fadd(w_start, ex[w, lane])
        for lane in range(32):
            xnext[w * 32 + lane] = X0[w * 32 + lane + 1] if lane < 31 else woff_in[w]
    # 2. grid offsets, ties, crossings; one exclusive scan in element order
    crossings, ties = [], []
    acc = 0
    for tid in range(nt):
        X = X0[tid]
        for k in range(ept):
            i = tid * ept + k
            P = xnext[tid] if k + 1 == ept else fadd(X, v[tid, k])
            b, bn = field(X), field(P)
            q = 1 << 52
            if b == bn and 23 <= b <= 254 and i != n - 1:
                f = F(v[tid, k] * F(2.0) ** (150 - b))
                if f < F(4194304.0):
                    g = fadd(f, F(12582912.0))
                    r = int(g.view(np.uint32)) - 0x4B400000
                    dr = F(F(g - F(12582912.0)) - f)
                    if abs(dr) == F(0.5):
                        q = (r - (1 if dr > 0 else 0)) | (1 << 40)
                    else:
                        q = r
            if i < n:
                if q >> 52:
                    crossings.append((i, acc & 0xFFFFFFFF, b, (acc >> 40) & 0xFFF))
                elif (q >> 40) & 0xFFF:
                    ties.append((acc & 0xFFFFFFFF, q & 0xFFFFFFFF))
                acc += q
            X = P
    nc, ntie = len(crossings), len(ties)
    if nc > CMAX or ntie > TMAX:
        return sequential_from(t, F(0), 0), "fallback"
    # 3. warp 0: each crossing's run, then the walk
    prep = []
    for r in range(nc):
        c, cqx, b, ct = crossings[r]
        st = crossings[r - 1][0] + 1 if r else 0
        q0 = crossings[r - 1][1] if r else 0
        t0 = crossings[r - 1][3] if r else 0
        up0 = up1 = 0
        for j in range(t0, ct):
            o = ((ties[j][0] - q0) + ties[j][1]) & 0xFFFFFFFF
            up0 += (o + up0) & 1
            up1 += (1 + o + up1) & 1
        prep.append((t[c], b, (cqx - q0) & 0xFFFFFFFF, up0, up1, c > st))
    s, done, ok = F(0), 0, True
    for r in range(nc):
        tc, b, q, up0, up1, run = prep[r]
        m = (int(s.view(np.uint32)) & 0x7FFFFF) | 0x800000
        mend = (m + q + (up1 if m & 1 else up0)) & 0xFFFFFFFF
        if run and (field(s) != b or mend >= 1 << 24):
            ok = False
            break
        if run:
            s = np.uint32((b << 23) | (mend & 0x7FFFFF)).view(F)
        s = fadd(s, tc)
        done = r + 1
    if ok:
        return s, "fast"
    start = crossings[done - 1][0] + 1 if done else 0
    return sequential_from(t, s, start), "fallback"
