"""The arithmetic behind the sampler's exact warp scan (pocketforge_b200/csrc/
scan.cuh), restated on the host and checked against numpy float32 additions.

The reference adds its normalising sum and its cumulative scan one float at a
time (src/engine.cpp:895-1003).  The kernel reproduces every partial sum from
integer maps: while the running sum c = R * g stays in one binade (g = 2^(E-23),
R in [2^23, 2^24)), adding t maps R to R + alpha + beta * (R mod 2), and these
maps compose.  The device checks its own code bit for bit against the float
loop (tests/test_kernels_gpu.py); these tests pin the same rules without a GPU:
single additions including exact halfway cases, the composition law in any
bracketing, and the windowed scan (16 terms per lane composed as a tree, a
lane scan, the first event walked term by term) on rows with ties, zeros, tiny,
NaN and inf terms."""
import numpy as np
import pytest

F32 = np.float32
CAP = 1 << 26
PER, LANES = 16, 32
KMIN = F32(2.0 ** -100)


def map_of(t, mult):
    x = F32(t) * F32(mult)
    if not x < F32(2.0 ** 25):
        return (CAP, 0)
    a = int(x)
    f = x - F32(a)
    if f < F32(0.5):
        return (a, 0)
    if f > F32(0.5):
        return (a + 1, 0)
    return (a + 1, -1) if a & 1 else (a, 1)


def map_then(p, q):
    par = p[0] & 1
    return (min(p[0] + q[0] + (q[1] if par else 0), CAP), p[1] if p[1] != 0 else (-q[1] if par else q[1]))


def map_apply(p, r):
    return r + p[0] + (p[1] if r & 1 else 0)


def binade(c):
    e = int((np.array(c, F32).view(np.uint32) >> 23) & 0xFF) - 127
    return e, F32(2.0 ** (e - 23)), F32(2.0 ** (23 - e))


def quarter_ulp(c):
    e = int(np.array(c, F32).view(np.uint32) >> 23)
    return F32(np.array((e - 25) << 23, np.uint32).view(F32)) if e >= 26 else F32(0)


def serial(a, stop):
    c = F32(0)
    for i, t in enumerate(a):
        c = F32(c + t)
        if stop(c):
            return i, c
    return len(a), c


def windowed(a, stop, desc):
    """scan.cuh's ordered_scan_warp, lane by lane."""
    n, c, pos = len(a), F32(0), 0
    while pos < n:
        if not (c >= KMIN and c < np.inf):
            k, stopped = pos, False
            while k < n:
                c = F32(c + a[k])
                if stop(c):
                    stopped = True
                    break
                if c >= KMIN and c < np.inf:
                    break
                if c != c:
                    k = n
                    break
                k += 1
            if stopped or k >= n:
                return k, c
            pos = k + 1
            continue
        if desc and a[pos] < quarter_ulp(c):
            return n, c
        _, g, mult = binade(c)
        R = int(F32(c) * mult)
        ws = pos & ~3
        terms = [[a[i] if pos <= i < n else F32(0) for i in range(ws + PER * L, ws + PER * L + PER)]
                 for L in range(LANES)]
        inc = []
        for L in range(LANES):  # each lane's maps as a tree
            m = [map_of(t, mult) for t in terms[L]]
            s = 1
            while s < PER:
                for j in range(0, PER - s, 2 * s):
                    m[j] = map_then(m[j], m[j + s])
                s *= 2
            inc.append(m[0])
        o = 1
        while o < LANES:  # the shuffle scan over lanes
            inc = [map_then(inc[L - o], inc[L]) if L >= o else inc[L] for L in range(LANES)]
            o *= 2
        ends = [map_apply(p, R) for p in inc]
        hit = [e >= (1 << 24) or stop(F32(e) * g) for e in ends]
        if not any(hit):
            c, pos = F32(ends[-1]) * g, ws + LANES * PER
            continue
        src = hit.index(True)
        r = map_apply(inc[src - 1], R) if src else R
        for j, t in enumerate(terms[src]):
            rn = map_apply(map_of(t, mult), r)
            i = ws + PER * src + j
            if rn >= (1 << 24):
                c = F32(F32(r) * g + a[i])
                if stop(c):
                    return i, c
                pos = i + 1
                break
            if stop(F32(rn) * g):
                return i, F32(rn) * g
            r = rn
        else:
            raise AssertionError("a flagged lane holds no event")
    return n, c


def test_single_additions_including_halfway_cases():
    rng = np.random.default_rng(1)
    checked = 0
    for _ in range(4000):
        e = int(rng.integers(-40, 40))
        R = int(rng.integers(1 << 23, 1 << 24))
        c = F32(R * 2.0 ** (e - 23))
        _, g, mult = binade(c)
        k = int(rng.integers(0, 1 << int(rng.integers(1, 22))))
        t = F32((k + rng.choice([0.5, 0.25, 0.75, 0.0, rng.uniform()])) * float(g))  # ties: (k + 1/2) g
        want = F32(c + t)
        if want >= F32(2.0 ** (e + 1)):
            continue
        assert F32(map_apply(map_of(t, mult), R)) * g == want
        checked += 1
    assert checked > 3000


def test_composition_in_any_bracketing():
    rng = np.random.default_rng(2)
    for _ in range(300):
        mult = F32(2.0 ** 20)
        ts = [F32(x) for x in rng.integers(0, 8, 12) * 0.5 / 2 ** 20 + rng.choice([0, 1e-7], 12)]
        maps = [map_of(t, mult) for t in ts]
        left = maps[0]
        for m in maps[1:]:
            left = map_then(left, m)
        right = maps[-1]
        for m in reversed(maps[:-1]):
            right = map_then(m, right)
        tree = list(maps)
        while len(tree) > 1:
            tree = [map_then(tree[i], tree[i + 1]) if i + 1 < len(tree) else tree[i] for i in range(0, len(tree), 2)]
        for R in (1 << 23, (1 << 23) + 1, 12345678, 12345679):
            step = R
            for m in maps:
                step = map_apply(m, step)
            assert map_apply(left, R) == map_apply(right, R) == map_apply(tree[0], R) == step


def _rows(rng):
    rows = []
    for mode in range(6):
        for _ in range(4):
            n = int(rng.integers(1, 1800))
            U = rng.uniform(size=n)
            if mode == 0:
                z = np.exp(-10.0 ** rng.uniform(-1, 2) * U)
            elif mode == 1:
                z = rng.integers(0, 64, n) * 0.125
            elif mode == 2:
                z = np.ldexp(rng.integers(0, 4096, n).astype(np.float64), -rng.integers(0, 30, n))
            elif mode == 3:
                z = np.where(U < 0.2, 0.0, np.exp(-30.0 * rng.uniform(size=n)))
            elif mode == 4:
                z = np.ldexp(1.0, -24 - rng.integers(0, 3, n)) * (1 + rng.integers(0, 3, n))
                z[0] = 1.0
            else:
                z = U
            rows.append(z.astype(F32))
    nan_row = np.ones(700, F32)
    nan_row[300] = np.nan
    inf_row = np.full(700, 0.5, F32)
    inf_row[350] = np.inf
    rows += [nan_row, inf_row, np.full(600, F32(1e-40)), np.full(600, F32(3e37)), np.full(900, F32(2.0 ** -101))]
    return rows


@pytest.mark.filterwarnings("ignore::RuntimeWarning")  # the 3e37 row overflows to inf on purpose
@pytest.mark.parametrize("sorted_rows", [False, True])
def test_windowed_scan_matches_float_loop(sorted_rows):
    rng = np.random.default_rng(3 + sorted_rows)
    for a in _rows(rng):
        if sorted_rows:
            if not np.isfinite(a).all():
                continue
            a = -np.sort(-a)
        tot = float(np.nansum(a.astype(np.float64)))
        u, p = F32(rng.uniform() * tot), F32((0.5 + 0.5 * rng.uniform()) * tot)
        for stop in (lambda c: False, lambda c: u <= c or c >= p, lambda c: F32(0) <= c):
            i1, c1 = serial(a, stop)
            i2, c2 = windowed(a, stop, sorted_rows)
            assert i1 == i2, (len(a), i1, i2)
            assert (c1 == c2 and np.signbit(c1) == np.signbit(c2)) or (np.isnan(c1) and np.isnan(c2)), (c1, c2)
