"""Random well-typed programs, version 2: a restatement of src/testing/random-graph.js.

The differential fuzz corpus of the reference's GPU protocol (src/gpu/harness-m4.js:125-172) is
``corpus_program(i, f32=True)`` for i = 1..2000.  The generator must reproduce the reference's
programs exactly, so every random draw happens in the same order as in JavaScript, including
draws skipped by short-circuit evaluation; ``Math.round`` rounds half up; ``Math.min`` /
``Math.max`` return NaN when any argument is NaN; ``Math.exp`` returns Infinity instead of
raising.  Pinned by golden/measurements.json's m4.semantics.corpus counts (tests/test_corpus.py).
"""
from __future__ import annotations

import math

from .ir import Graph, broadcast_shapes, size
from .rng import Rng

MAX_SIZE = 96
BOUND = 1e3
INPUT_RANGE = (-2.0, 2.0)
GENERATED = {"add": 3, "sub": 3, "mul": 3, "div": 3, "neg": 1, "exp": 2, "log": 2, "relu": 3, "tanh": 2,
             "matmul": 4, "sum": 3, "broadcast": 2, "reshape": 3, "transpose": 3, "softmax": 2, "logSoftmax": 2}
TARGETS = ("matmul", "transpose", "reshape", "broadcast", "sum")
_INF = math.inf


def _nan(x):
    return x != x


def js_min(*xs):
    return math.nan if any(_nan(x) for x in xs) else min(xs)


def js_max(*xs):
    return math.nan if any(_nan(x) for x in xs) else max(xs)


def js_exp(x):
    try:
        return math.exp(x)
    except OverflowError:
        return _INF


def js_log(x):
    if _nan(x) or x < 0:
        return math.nan
    if x == 0:
        return -_INF
    return math.log(x)


def js_mul(a, b):
    return a * b  # IEEE: inf * 0 is NaN, as in JavaScript


def js_round(v):
    """Math.round(v * 1024) / 1024 (half rounds up, toward +inf)."""
    return math.floor(v * 1024 + 0.5) / 1024


def _mul_iv(a, b):
    p = [js_mul(a[0], b[0]), js_mul(a[0], b[1]), js_mul(a[1], b[0]), js_mul(a[1], b[1])]
    return [js_min(*p), js_max(*p)]


def _magnitude(iv):
    return js_max(abs(iv[0]), abs(iv[1]))


def _interval(g, nid, iv, square_aware=False):
    n = g.nodes[nid]
    ins = [iv.get(i) for i in n.inputs]
    a = ins[0] if ins else None
    b = ins[1] if len(ins) > 1 else None
    op = n.op
    if op == "input":
        return list(INPUT_RANGE)
    if op == "const":
        v = n.attrs["value"]
        return [float(v), float(v)] if isinstance(v, (int, float)) else [js_min(*v), js_max(*v)]
    if op == "add":
        return [a[0] + b[0], a[1] + b[1]]
    if op == "sub":
        return [a[0] - b[1], a[1] - b[0]]
    if op == "mul":
        if square_aware and n.inputs[0] == n.inputs[1]:
            m = _magnitude(a)
            lo = 0 if (a[0] <= 0 and a[1] >= 0) else js_min(a[0] * a[0], a[1] * a[1])
            return [lo, m * m]
        return _mul_iv(a, b)
    if op == "div":
        if b[0] <= 0 and b[1] >= 0:
            return [-_INF, _INF]
        return _mul_iv(a, [1 / b[1], 1 / b[0]])
    if op == "neg":
        return [-a[1], -a[0]]
    if op == "exp":
        return [js_exp(a[0]), js_exp(a[1])]
    if op == "log":
        return [js_log(a[0]), js_log(a[1])] if a[0] > 0 else [-_INF, _INF]
    if op == "relu":
        return [js_max(0.0, a[0]), js_max(0.0, a[1])]
    if op == "step":
        return [0.0, 1.0]
    if op == "tanh":
        return [math.tanh(a[0]), math.tanh(a[1])]
    if op == "sqrt":
        return [math.sqrt(a[0]), math.sqrt(a[1])] if a[0] >= 0 else [-_INF, _INF]
    if op == "matmul":
        k = g.shape(n.inputs[0])[-1]
        lo, hi = _mul_iv(a, b)
        return [k * lo, k * hi]
    if op == "sum":
        ln = g.shape(n.inputs[0])[n.attrs["axis"]]
        return [ln * a[0], ln * a[1]]
    if op in ("max", "stopGradient", "broadcast", "reshape", "transpose"):
        return list(a)
    raise ValueError(f"no interval rule for {op}")


def factorizations(n, rank):
    if rank == 1:
        return [[n]]
    out = []
    for d in range(1, n + 1):
        if n % d:
            continue
        for rest in factorizations(n // d, rank - 1):
            out.append([d] + rest)
    return out


def _is_involution(perm):
    return all(perm[p] == i for i, p in enumerate(perm))


class _Builder:
    """src/testing/random-graph.js:118-339."""

    def __init__(self, rng):
        self.rng = rng
        self.g = Graph()
        self.iv = {}
        self.pool = []
        self.leaves = 0
        self.strict = False
        self.f32 = False
        self.square_aware = False
        self.operand = None

    def track(self, nid):
        if nid not in self.iv:
            for i in range(nid + 1):
                if i not in self.iv:
                    self.iv[i] = _interval(self.g, i, self.iv, self.square_aware)
        return nid

    def ok(self, nid):
        return _magnitude(self.iv[self.track(nid)]) <= BOUND

    def dim(self):
        if self.strict:
            return self.rng.int(2, 5)
        return 1 if self.rng.chance(0.2) else self.rng.int(2, 6)

    def shape(self, min_rank=0, max_rank=4):
        while True:
            rank = self.rng.int(min_rank, max_rank)
            s = [self.dim() for _ in range(rank)]
            if size(s) <= MAX_SIZE:
                return s

    def input(self, shape):
        nid = self.g.input(f"x{self.leaves}", shape)
        self.leaves += 1
        return self.push(nid)

    def leaf(self, shape):
        if self.rng.chance(0.7):
            return self.input(shape)
        vals = [js_round(v) for v in self.rng.array(size(shape), -2, 2)]
        return self.push(self.g.const(vals, shape))

    def push(self, nid):
        self.track(nid)
        self.pool.append(nid)
        return nid

    def choose(self, flt=None):
        c = [i for i in self.pool if flt is None or flt(self.g.shape(i), i)]
        if not c:
            return None
        r = self.rng.next()
        return c[len(c) - 1 - math.floor(r * r * len(c))]

    def first(self, flt=None):
        if self.operand is None:
            return self.choose(flt)
        return self.operand if (flt is None or flt(self.g.shape(self.operand), self.operand)) else None

    def scalar_const(self, lo, hi):
        return self.track(self.g.const(js_round(self.rng.uniform(lo, hi))))

    def safe_denominator(self, x):
        lo, hi = self.iv[x]
        if lo >= 0.1 or hi <= -0.1:
            return x
        r = self.rng.next()
        g = self.g
        if r < 0.4:
            return self.track(g.add(g.mul(x, x), self.scalar_const(0.2, 1)))
        if r < 0.6:
            return self.track(g.neg(g.add(g.mul(x, x), self.scalar_const(0.2, 1))))
        return self.track(g.exp(self.bounded_for_exp(x)))

    def bounded_for_exp(self, x):
        lo, hi = self.iv[x]
        return x if (hi <= 4 and (not self.f32 or lo >= -40)) else self.track(self.g.tanh(x))

    def safe_sqrt_argument(self, x):
        if self.iv[x][0] >= 0.1:
            return x
        return self.track(self.g.add(self.g.exp(self.bounded_for_exp(x)), self.scalar_const(0.2, 1)))

    def safe_log_argument(self, x):
        if self.iv[x][0] >= 0.1:
            return x
        g = self.g
        if self.rng.chance(0.6):
            return self.track(g.add(g.mul(x, x), self.scalar_const(0.2, 1)))
        return self.track(g.exp(self.bounded_for_exp(x)))

    def partner(self, x):
        xs = self.g.shape(x)

        def fits(s, _i):
            o = broadcast_shapes(xs, s)
            return o is not None and size(o) <= MAX_SIZE
        b = self.choose(fits) if self.rng.chance(0.5) else None
        if b is not None:
            return b
        drop = self.rng.int(0, len(xs)) if self.rng.chance(0.3) else 0
        return self.leaf([1 if self.rng.chance(0.3) else d for d in xs[drop:]])

    def apply(self, op, operand=None):
        g, rng = self.g, self.rng
        self.operand = operand
        if op in ("add", "sub", "mul"):
            a = self.first()
            return getattr(g, op)(a, self.partner(a))
        if op == "div":
            a = self.first()
            return g.div(a, self.safe_denominator(self.partner(a)))
        if op == "log":
            return g.log(self.safe_log_argument(self.first()))
        if op == "exp":
            return g.exp(self.bounded_for_exp(self.first()))
        if op == "sqrt":
            return g.sqrt(self.safe_sqrt_argument(self.first()))
        if op in ("neg", "relu", "tanh"):
            return getattr(g, op)(self.first())
        if op == "matmul":
            return self.matmul(self.first())
        if op == "sum":
            x = self.first(lambda s, _i: len(s) >= 1)
            if x is None:
                return None
            axis = rng.int(0, len(g.shape(x)) - 1)
            return g.sum(x, axis, rng.chance(0.4))
        if op in ("softmax", "logSoftmax"):
            x = self.first(lambda s, _i: len(s) >= 1)
            if x is None:
                return None
            axis = rng.int(0, len(g.shape(x)) - 1)
            return g.softmax(x, axis) if op == "softmax" else g.log_softmax(x, axis)
        if op == "broadcast":
            return self.broadcast(self.first())
        if op == "reshape":
            return self.reshape(self.first())
        if op == "transpose":
            x = self.first(lambda s, _i: len(s) >= 2)
            return None if x is None else self.transpose(x)
        raise ValueError(f"generator has no case for '{op}'")

    def matmul(self, a):
        g, rng = self.g, self.rng
        a_s = g.shape(a)
        if len(a_s) < 2:
            n = size(a_s)
            options = factorizations(n, 2)
            square = [o for o in options if o[0] > 1 and o[1] > 1]
            use_square = len(square) > 0 and rng.chance(0.8)
            a = self.track(g.reshape(a, rng.pick(square if use_square else options)))
            a_s = g.shape(a)
        batch = list(a_s[:-2])
        k = a_s[-1]
        n = self.dim()
        if size(batch + [a_s[-2], n]) > MAX_SIZE or size(batch + [k, n]) > MAX_SIZE:
            return None

        def fits(s, _i):
            return (len(s) == len(a_s) and s[-2] == k and all(d == s[i] for i, d in enumerate(batch))
                    and size(batch + [a_s[-2], s[-1]]) <= MAX_SIZE)
        if self.strict:
            b = self.input(batch + [k, n])
        else:
            b = self.choose(fits) if rng.chance(0.3) else None
            if b is None:
                b = self.leaf(batch + [k, n])
        return g.matmul(a, b)

    def broadcast(self, x):
        g, rng = self.g, self.rng
        xs = g.shape(x)
        lead = [rng.int(2, 4) for _ in range(rng.int(1, 2))] if rng.chance(0.5) else []
        to = lead + [(rng.int(2, 5) if (d == 1 and rng.chance(0.7)) else d) for d in xs]
        if len(to) > 4 or size(to) > MAX_SIZE or (len(to) == len(xs) and all(d == xs[i] for i, d in enumerate(to))):
            return None
        return g.broadcast(x, to)

    def reshape(self, x):
        g, rng = self.g, self.rng
        n = size(g.shape(x))
        allf = [s for s in factorizations(n, rng.int(1, 4)) if len(s) <= 4]
        wide = [s for s in allf if len(s) >= 2 and s[-1] > 1 and s[-2] > 1]
        use_wide = len(wide) > 0 and rng.chance(0.9 if self.strict else 0.7)
        shape = rng.pick(wide if use_wide else allf)
        nid = g.reshape(x, shape)
        return None if nid == x else nid

    def transpose(self, x):
        g, rng = self.g, self.rng
        rank = len(g.shape(x))
        perm = None
        for _ in range(10):
            perm = rng.shuffle(list(range(rank)))
            if not all(p == i for i, p in enumerate(perm)):
                if not _is_involution(perm) or rng.chance(0.1 if self.strict else 0.3):
                    break
        nid = g.transpose(x, perm)
        return None if nid == x else nid

    def weigh(self, x):
        return self.g.mul(x, self.input(self.g.shape(x)))


# ---- targeted programs (random-graph.js:361-412) ----
def _t_matmul(b):
    rank = 2 if b.rng.chance(0.6) else 3
    batch = [b.rng.int(2, 3)] if rank == 3 else []
    m = b.rng.int(2, 5)
    k = b.rng.int(2, 5)
    x = b.input(batch + [m, k])
    i = b.rng.int(1, 2)
    while i > 0:
        if b.rng.chance(0.5):
            x = b.push(b.g.tanh(x))
        y = b.matmul(x)
        if y is None or not b.ok(y):
            break
        x = b.push(y)
        i -= 1
    return x


def _t_transpose(b):
    x0 = b.input(b.shape(3, 4))
    t = b.transpose(x0)
    x = b.push(t if t is not None else x0)
    x = b.push(b.weigh(b.g.tanh(x)))
    if b.rng.chance(0.5):
        t = b.transpose(x)
        x = b.push(t if t is not None else x)
    return x


def _t_reshape(b):
    for _ in range(10):
        x0 = b.input(b.shape(2, 4))
        x = b.push(b.g.tanh(x0))
        r = b.reshape(x)
        if r is None:
            continue
        x = b.push(r)
        x = b.push(b.weigh(x))
        if b.rng.chance(0.4):
            r2 = b.reshape(x)
            if r2 is not None:
                x = b.push(r2)
        return x
    raise RuntimeError("no reshape in 10 tries")


def _t_broadcast(b):
    for _ in range(10):
        x0 = b.input([1 if b.rng.chance(0.5) else d for d in b.shape(1, 3)])
        y = b.broadcast(b.push(b.g.tanh(x0)))
        if y is None:
            continue
        return b.push(b.weigh(b.push(y)))
    raise RuntimeError("no broadcast in 10 tries")


def _t_sum(b):
    x0 = b.input(b.shape(2, 4))
    x = b.push(b.g.tanh(x0))
    axis = b.rng.int(0, len(b.g.shape(x)) - 1)
    return b.push(b.weigh(b.push(b.g.sum(x, axis, b.rng.chance(0.4)))))


TARGETED = {"matmul": _t_matmul, "transpose": _t_transpose, "reshape": _t_reshape, "broadcast": _t_broadcast,
            "sum": _t_sum}


def _try_op(b, op, operand=None):
    """Apply an op, keeping it only if its result is provably within BOUND (random-graph.js:449-460)."""
    before = len(b.g.nodes)
    nid = b.apply(op, operand)
    if nid is None:
        return None
    if not b.ok(nid):
        del b.g.nodes[before:]
        for k in [k for k in b.iv if k >= before]:
            del b.iv[k]
        b.pool = [p for p in b.pool if p < before]
        return None
    return b.push(nid)


class Program:
    __slots__ = ("seed", "focus", "graph", "outputs", "inputs", "bounds")

    def __init__(self, seed, focus, graph, outputs, inputs, bounds):
        self.seed, self.focus, self.graph, self.outputs, self.inputs, self.bounds = \
            seed, focus, graph, outputs, inputs, bounds


def random_program(seed, focus=None, f32=False, with_sqrt=False, square_aware=False):
    """random-graph.js:419-446."""
    rng = Rng(((seed * 31 + TARGETS.index(focus) + 1) & 0xFFFFFFFF) if focus else seed)
    b = _Builder(rng)
    b.f32 = f32
    b.square_aware = square_aware
    last = None
    if focus:
        b.strict = True
        last = TARGETED[focus](b)
        b.strict = False
        i = rng.int(0, 2)
        while i > 0:
            nid = _try_op(b, rng.pick(["add", "mul", "tanh", "exp", "log", "div", "relu", "sum", "softmax"]), last)
            if nid is not None:
                last = nid
            i -= 1
    else:
        i = rng.int(1, 3)
        while i > 0:
            b.input(b.shape())
            i -= 1
        weights = dict(GENERATED)
        if with_sqrt:
            weights["sqrt"] = 3
        ops = [op for op, w in weights.items() for _ in range(w)]
        steps = rng.int(2, 10)
        made = 0
        attempt = 0
        while made < steps and attempt < steps * 20:
            if _try_op(b, rng.pick(ops)) is not None:
                made += 1
            attempt += 1
    consumed = {i for n in b.g.nodes for i in n.inputs}
    outputs = [n.id for n in b.g.nodes if n.op not in ("input", "const") and n.id not in consumed]
    if not outputs:
        outputs = [b.pool[-1]]
    bounds = [b.iv[n.id] if n.id in b.iv else _interval(b.g, n.id, b.iv, b.square_aware) for n in b.g.nodes]
    return Program(seed, focus, b.g, outputs, [n.attrs["name"] for n in b.g.inputs()], bounds)


def corpus_program(i, f32=False, with_sqrt=False, square_aware=False):
    """Corpus program i: odd i general, even i targeted, cycling through TARGETS (random-graph.js:463-467)."""
    if i % 2 == 1:
        return random_program(i, None, f32, with_sqrt, square_aware)
    return random_program(i, TARGETS[(i // 2) % len(TARGETS)], f32, with_sqrt, square_aware)
