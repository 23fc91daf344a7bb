"""CPU model of the exact left-to-right sum of non-negative floats that
sum_in_order_par (leaf_b200/csrc/decoder_math.cuh) computes with a whole
block: runs of additions inside one binade of the running sum are integer
increments of its bits, every predicted binade change or exact-half tie is a
plain float addition, and each run is checked before it is applied.  Here in
numpy, row by row, against numpy's sequential float32 cumulative sum (the
order of the reference's `for (col) square += value * value`).  The GPU
kernels are checked against the oracle in tests/test_gpu_decoder_ops.py;
this test pins the arithmetic argument itself on the CPU."""
import numpy as np
import pytest

ELEM_SAT = 1 << 23


def _binade(x):
    return (np.asarray(x, np.float32).view(np.uint32) >> 23).astype(np.int64)


def _sequential(v):
    return np.cumsum(v, dtype=np.float32)[-1] if v.size else np.float32(0)


def ordered_sum_model(v: np.ndarray, approx_order_seed: int = 0):
    """Returns (sum, heads, runs added element by element)."""
    v = np.asarray(v, np.float32)
    n = v.size
    if n == 0:
        return np.float32(0), 0, 0
    # Approximate prefix sums in another order (blocks of 4, then a scan).
    blocks = v.reshape(-1, 4).astype(np.float64).sum(axis=1) if n % 4 == 0 else v.astype(np.float64)
    reps = 4 if n % 4 == 0 else 1
    base = np.concatenate([[0.0], np.cumsum(blocks)[:-1]]).astype(np.float32)
    P = np.empty(n, np.float32)
    for j in range(reps):  # the running approximation inside each block, in float32
        prev = base if j == 0 else P[j - 1::reps]
        P[j::reps] = (prev + v[j::reps]).astype(np.float32)
    if not np.isfinite(P[-1]):
        return _sequential(v), 0, 1
    before = np.concatenate([[np.float32(0)], P[:-1]]).astype(np.float32)
    E = _binade(before)
    # Increment of each addition in its binade: f = v / u exactly (float64).
    k = 150 - np.maximum(E, 1)
    f = v.astype(np.float64) * np.ldexp(1.0, k)
    tie = (f - np.floor(f)) == 0.5
    F = np.where(f < ELEM_SAT, np.rint(f), ELEM_SAT).astype(np.int64)
    head = tie | (_binade(P) != E)
    head[0] = True
    inc = np.where(head, 0, F)
    C = np.concatenate([[0], np.cumsum(inc)])  # sum of increments before each element
    hpos = np.flatnonzero(head)
    nxt = np.append(hpos[1:], n)
    s = np.float32(0)
    fallbacks = 0
    for h, e in zip(hpos, nxt):
        s = np.float32(s + v[h])
        run = int(C[e] - C[h + 1])
        Eh = int(_binade(P[h]))
        b = int(np.float32(s).view(np.uint32))
        nb = b + min(run, ELEM_SAT)
        if (b >> 23) == Eh and (nb >> 23) == Eh:
            s = np.uint32(nb).view(np.float32)
        else:
            fallbacks += 1
            for i in range(h + 1, e):
                s = np.float32(s + v[i])
    return s, len(hpos), fallbacks


def _rows(kind, rng, rows, n):
    g = rng.standard_normal((rows, n))
    if kind == "normal":
        x = g
    elif kind == "small":
        x = g * 1e-3
    elif kind == "outliers":
        x = g * np.where(rng.random(g.shape) < 0.01, 100, 1)
    elif kind == "tiny":
        x = g * 1e-20
    elif kind == "zeros":
        x = np.where(rng.random(g.shape) < 0.8, 0.0, g)
    elif kind == "grid":
        x = np.trunc(g * 8) / 8
    elif kind == "pow2":
        x = np.ldexp(1.0, rng.integers(-10, 10, g.shape)) * (1 + rng.integers(0, 4, g.shape) / 4)
    elif kind == "ones":
        x = np.sign(g)
    elif kind == "huge":
        x = g * 1e18
    else:
        raise ValueError(kind)
    x = x.astype(np.float32)
    return (x * x).astype(np.float32)


@pytest.mark.parametrize("kind", ["normal", "small", "outliers", "tiny", "zeros", "grid", "pow2", "ones", "huge"])
@pytest.mark.parametrize("n", [4, 64, 2048])
def test_piece_sum_bit_exact(kind, n):
    rng = np.random.default_rng(abs(hash((kind, n))) % 2**32)
    rows = 40 if n == 2048 else 200
    squares = _rows(kind, rng, rows, n)
    with np.errstate(over="ignore", invalid="ignore"):
        for r in range(rows):
            got, heads, _ = ordered_sum_model(squares[r])
            want = _sequential(squares[r])
            assert got.view(np.uint32) == want.view(np.uint32) or (np.isnan(got) and np.isnan(want)), \
                (kind, n, r, got, want)


def test_typical_rows_need_few_heads():
    # Rows of 2048 squares of N(0, 1) values: ~15 heads and almost never a
    # run added element by element.
    rng = np.random.default_rng(1)
    squares = _rows("normal", rng, 100, 2048)
    stats = [ordered_sum_model(r)[1:] for r in squares]
    heads = np.mean([h for h, _ in stats])
    fallbacks = sum(f for _, f in stats)
    assert 5 <= heads <= 40, heads
    assert fallbacks <= 2, fallbacks
