"""CUDA source for every launch: the replacement of the reference's WGSL generators.

The reference builds WGSL text per launch (src/gpu/codegen.js:199-215 for
plain kernels, src/fusion/codegen-fused.js:357-362 for fused nodes).  Here a
launch is CUDA C++ that instantiates one of libtcb200's hand-written sm_100a
templates (``tcb/elementwise.cuh``, ``tcb/rowwise.cuh``, ``tcb/matmul.cuh``,
``tcb/reduce.cuh``) with the fused body emitted as straight-line code:

* every body value is computed once per index it is needed at (the
  reference's Emitter memoises per index context, codegen-fused.js:80-148);
* scalar constants are inlined as their exact float32 bits
  (codegen-fused.js:26-27);
* shapes and strides are compile-time constants (NVRTC specialises each
  launch, so index arithmetic is multiply-shift, not the reference's per-axis
  u32 div/mod loop ``gidx``, codegen-fused.js:47-58);
* every load is classified -- direct, row broadcast (``i % P``), column
  broadcast (``i / Q``), scalar, or a general strided gather -- so that direct
  and row-broadcast loads become 128-bit vector loads.
"""
from __future__ import annotations

import math
import struct

from .ir import size, strides, f32

MAX_RANK = 6  # src/gpu/codegen.js:16, kept for the gather rank limit of the interface
WG = 256  # threads per CTA of the 1-D templates (the reference's WG = 64, src/gpu/codegen.js:12)
FUSED_SABOTAGE = ("epilogue-before-bias", "layernorm-tree-short", "softmax-no-max", "fused-bounds-off-by-one")

_BIN = {"add": "tcb::op_add", "sub": "tcb::op_sub", "mul": "tcb::op_mul", "div": "tcb::op_div"}
_UN = {"neg": "tcb::op_neg", "exp": "tcb::op_exp", "log": "tcb::op_log", "relu": "tcb::op_relu",
       "tanh": "tcb::op_tanh", "sqrt": "tcb::op_sqrt", "step": "tcb::op_step", "stopGradient": "tcb::op_copy"}


def f32_literal(v):
    """The exact float32 bits of ``fround(v)`` as a CUDA expression (codegen-fused.js:26-27)."""
    b = struct.unpack("<I", struct.pack("<f", f32(float(v))))[0]
    return f"tcb::bits(0x{b:08x}u)"


def gather_strides(node_op, out_shape, in_shape, perm=None):
    """Source strides that make a gather over the output read the input (src/gpu/lower.js:31-62)."""
    if node_op == "broadcast":
        lead = len(out_shape) - len(in_shape)
        nat = strides(in_shape)
        return [0 if (i < lead or in_shape[i - lead] == 1) else nat[i - lead] for i in range(len(out_shape))]
    if node_op == "transpose":
        nat = strides(in_shape)
        return [nat[p] for p in perm]
    if node_op == "reshape":
        return strides(out_shape)
    raise ValueError(f"not a strided move: {node_op}")


class Gather:
    """A strided re-index ``src = sum_d coord_d(i) * g_d`` over an output shape, simplified.

    ``kind``: 'identity' (src = i), 'scalar' (0), 'rowb' (i % P), 'colb' (i / Q),
    'general'.  Axes of extent 1 are dropped and axes contiguous in both
    spaces are merged before classifying.
    """

    def __init__(self, out_shape, gstrides):
        dims = [(d, g) for d, g in zip(out_shape, gstrides) if d != 1]
        merged = []
        for d, g in dims:
            if merged and merged[-1][1] == g * d and True:
                pd, pg = merged[-1]
                merged[-1] = (pd * d, g)
            elif merged and merged[-1][1] == 0 and g == 0:
                pd, _ = merged[-1]
                merged[-1] = (pd * d, 0)
            else:
                merged.append((d, g))
        self.dims = merged
        nz = [(i, d, g) for i, (d, g) in enumerate(merged) if g != 0]
        n = len(merged)
        self.P = self.Q = None
        if not nz:
            self.kind = "scalar"
        elif n == 1 and merged[0][1] == 1:
            self.kind = "identity"
        elif len(nz) == 1 and nz[0][0] == n - 1 and nz[0][2] == 1:
            self.kind = "rowb"
            self.P = merged[-1][0]
        elif n == 2 and merged[0][1] == 1 and merged[1][1] == 0:
            self.kind = "colb"
            self.Q = merged[1][0]
        else:
            self.kind = "general"

    def expr(self, i, T):
        """C expression of the source index for index expression ``i`` of type T."""
        if self.kind == "scalar":
            return f"(({T})0)"
        if self.kind == "identity":
            return f"({i})"
        if self.kind == "rowb":
            return f"(({i}) % ({T}){self.P}ull)"
        if self.kind == "colb":
            return f"(({i}) / ({T}){self.Q}ull)"
        terms = []
        ost = 1
        out = []
        for d, g in reversed(self.dims):
            out.append((d, g, ost))
            ost *= d
        out.reverse()
        for k, (d, g, s) in enumerate(out):
            if g == 0:
                continue
            q = f"({i})" if s == 1 else f"(({i}) / ({T}){s}ull)"
            if k > 0:
                q = f"({q} % ({T}){d}ull)"
            terms.append(q if g == 1 else f"{q} * ({T}){g}ull")
        return "(" + " + ".join(terms) + ")"

    def key(self):
        return (self.kind, tuple(self.dims))

    def vec4(self):
        """A general gather whose innermost run is contiguous (stride 1, a multiple of 4 long) and whose
        other strides are multiples of 4: 4 consecutive outputs starting at a multiple of 4 read 4
        consecutive, 16-byte aligned source floats."""
        if self.kind != "general" or not self.dims:
            return False
        d, g = self.dims[-1]
        return g == 1 and d % 4 == 0 and all(gg % 4 == 0 for _, gg in self.dims[:-1])


class Ctx:
    """An index context: the base index, or a gathered index computed from a parent context."""

    def __init__(self, key, parent=None, gather=None):
        self.key = key
        self.parent = parent
        self.gather = gather


def idx_type(n):
    return "u32" if n < 2 ** 32 - 1 else "u64"


class Emitter:
    """Straight-line code for a body graph, memoised per (index context, node).

    ``leaf(k, ctx)`` returns the C expression of operand ``a<k>`` read in
    ``ctx`` (it registers the load with the template-specific load plan);
    ``special(nid, ctx)`` may claim a node (the matmul accumulator, a
    reduction result, a row-tier value).  ``lines`` receives the statements
    of the current section; the caller may swap it between sections.
    """

    def __init__(self, body, leaf, special=None):
        self.b = body
        self.leaf = leaf
        self.special = special
        self.memo = {}
        self.lines = []
        self.counter = 0
        self.ctxs = {}

    def child(self, ctx, gather):
        if gather.kind == "identity":
            return ctx
        key = (ctx.key, gather.key())
        c = self.ctxs.get(key)
        if c is None:
            c = self.ctxs[key] = Ctx(key, ctx, gather)
        return c

    def forget(self, pred):
        for k in [k for k in self.memo if pred(k[0])]:
            del self.memo[k]

    def value(self, nid, ctx):
        key = (ctx.key, nid)
        if key in self.memo:
            return self.memo[key]
        if self.special is not None:
            s = self.special(nid, ctx)
            if s is not None:
                self.memo[key] = s
                return s
        node = self.b.nodes[nid]
        op = node.op
        if op == "input":
            v = self.leaf(int(node.attrs["name"][1:]), ctx)
            self.memo[key] = v
            return v
        if op == "const":
            val = node.attrs["value"]
            v = f32_literal(val if isinstance(val, (int, float)) else val[0])
            self.memo[key] = v
            return v
        if op == "reshape":
            v = self.value(node.inputs[0], ctx)
            self.memo[key] = v
            return v
        if op in ("broadcast", "transpose"):
            src = self.b.nodes[node.inputs[0]]
            if src.op == "const":
                v = self.value(src.id, ctx)
            else:
                g = Gather(node.shape, gather_strides(op, node.shape, src.shape, node.attrs.get("perm")))
                v = self.value(src.id, self.child(ctx, g))
            self.memo[key] = v
            return v
        if op in _BIN:
            a = self.value(node.inputs[0], ctx)
            c = self.value(node.inputs[1], ctx)
            expr = f"{_BIN[op]}({a}, {c})"
        elif op in _UN:
            expr = f"{_UN[op]}({self.value(node.inputs[0], ctx)})"
        else:
            raise ValueError(f"fused codegen: no rule for '{op}'")
        name = f"v{self.counter}"
        self.counter += 1
        self.lines.append(f"const float {name} = {expr};")
        self.memo[key] = name
        return name


def _chain_index(ctx, base, T):
    """The C index expression of ``ctx`` given the base context's index expression."""
    if ctx.parent is None:
        return base
    return ctx.gather.expr(_chain_index(ctx.parent, base, T), T)


def _operand_count(body):
    return sum(1 for n in body.nodes if n.op == "input")


# ------------------------------------------------------------------ elementwise
class _EwLoads:
    """Load plan of the elementwise template: W lanes starting at i0."""

    def __init__(self, W, T):
        self.W, self.T = W, T
        self.fields = []   # declarations in Regs<W>
        self.stmts = []    # load statements
        self.per_lane = []  # per-lane load statements
        self.seen = {}

    def leaf(self, k, ctx):
        key = (ctx.key, k)
        if key in self.seen:
            return self.seen[key]
        W, T = self.W, self.T
        ptr = f"reinterpret_cast<const float*>(a.in[{k}])"
        name = f"x{len(self.seen)}"
        g = ctx.gather
        if ctx.parent is None:
            self.fields.append(f"float {name}[W];")
            self.stmts.append(f"tcb::load<W>(r.{name}, {ptr} + i0);")
            ref = f"r.{name}[l]"
        elif ctx.parent.parent is None and g.kind == "rowb" and g.P % 4 == 0:
            self.fields.append(f"float {name}[W];")
            self.stmts.append(f"tcb::load<W>(r.{name}, {ptr} + (({T})i0 % ({T}){g.P}ull));")
            ref = f"r.{name}[l]"
        elif ctx.parent.parent is None and (g.kind == "scalar" or (g.kind == "colb" and g.Q % 4 == 0)):
            self.fields.append(f"float {name};")
            self.stmts.append(f"r.{name} = tcb::ld1({ptr} + {g.expr(f'({T})i0', T)});")
            ref = f"r.{name}"
        elif ctx.parent.parent is None and g.vec4():
            self.fields.append(f"float {name}[W];")
            self.stmts.append(f"tcb::load<W>(r.{name}, {ptr} + {g.expr(f'({T})i0', T)});")
            ref = f"r.{name}[l]"
        else:
            self.fields.append(f"float {name}[W];")
            self.per_lane.append(f"r.{name}[l] = tcb::ld1({ptr} + {_chain_index(ctx, f'(({T})i0 + ({T})l)', T)});")
            ref = f"r.{name}[l]"
        self.seen[key] = ref
        return ref


def _ew_body_struct(body, out_id, n):
    """The `struct Body` of an elementwise body (load plan + straight-line compute), shared by the
    elementwise and the elementwise + column-sum templates."""
    T = idx_type(n)
    loads = _EwLoads("W", T)
    em = Emitter(body, loads.leaf)
    base = Ctx("i")
    out = em.value(out_id, base)
    fields = "\n    ".join(loads.fields) or "float unused_;"
    stmts = "\n    ".join(loads.stmts)
    lanes = "\n      ".join(loads.per_lane)
    per_lane = f"#pragma unroll\n    for (int l = 0; l < W; ++l) {{\n      {lanes}\n    }}" if loads.per_lane else ""
    comp = "\n      ".join(em.lines)
    return f"""struct Body {{
  template <int W> struct Regs {{
    {fields}
  }};
  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {{
    {stmts}
    {per_lane}
  }}
  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[W]) {{
#pragma unroll
    for (int l = 0; l < W; ++l) {{
      {comp}
      o[l] = {out};
    }}
  }}
}};
"""


def _elementwise_source(body, out_id, n, sabotage=None, tag="elementwise"):
    T = idx_type(n)
    loads = _EwLoads("W", T)
    em = Emitter(body, loads.leaf)
    base = Ctx("i")
    out = em.value(out_id, base)
    fields = "\n    ".join(loads.fields) or "float unused_;"
    stmts = "\n    ".join(loads.stmts)
    lanes = "\n      ".join(loads.per_lane)
    per_lane = f"#pragma unroll\n    for (int l = 0; l < W; ++l) {{\n      {lanes}\n    }}" if loads.per_lane else ""
    comp = "\n      ".join(em.lines)
    src = f"""// {tag}: generated from a body of {len(body.nodes)} nodes, {n} elements
#include "tcb/common.cuh"
#define TCB_W 4
struct Body {{
  template <int W> struct Regs {{
    {fields}
  }};
  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {{
    {stmts}
    {per_lane}
  }}
  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[W]) {{
#pragma unroll
    for (int l = 0; l < W; ++l) {{
      {comp}
      o[l] = {out};
    }}
  }}
}};
#include "tcb/elementwise.cuh"
"""
    return src


# ------------------------------------------------------------------ rowwise
def _pow2ceil(x):
    return 1 << max(0, math.ceil(math.log2(max(1, x))))


def rowwise_geometry(R, C, n_leaves, elems_per_thread=16):
    """Threads per row, rows per CTA, vector width, register slots; cache or stream mode."""
    vec = 4 if C % 4 == 0 else 1
    tpr = min(1024, max(32, _pow2ceil(math.ceil(C / elems_per_thread))))
    groups = max(1, 256 // tpr)
    slots = math.ceil(C / (tpr * vec))
    items = slots * vec
    cache = items <= 32 and items * max(1, n_leaves) <= 128
    return {"vec": vec, "tpr": tpr, "groups": groups, "slots": slots, "items": items, "cache": cache,
            "block": tpr * groups}


class _RowLoads:
    """Load plan of the rowwise template: row leaves (once per row) and element leaves (per item)."""

    def __init__(self, body, R, C, T, vec, cache):
        self.body, self.R, self.C, self.T, self.vec, self.cache = body, R, C, T, vec, cache
        self.row = {}      # key -> (name, stmt)
        self.elem = {}     # key -> (name, kind, stmt-builder)
        self.order_row = []
        self.order_elem = []

    def leaf(self, k, ctx):
        T = self.T
        ptr = f"reinterpret_cast<const float*>(a.in[{k}])"
        root = ctx
        while root.parent is not None:
            root = root.parent
        if root.key == "r":
            # a row-context read (possibly through a broadcast of the operand): once per row
            key = (ctx.key, k)
            if key not in self.row:
                name = f"R{len(self.row)}"
                self.row[key] = name
                idx = _chain_index(ctx, f"({T})r", T)
                self.order_row.append(f"const float {name} = active ? tcb::ld1({ptr} + {idx}) : 0.0f;")
            return self.row[key]
        # element context (or a gathered child of it)
        g = ctx.gather
        if ctx.parent is not None and ctx.parent.key == "e" and g.kind == "colb" and g.Q == self.C:
            return self.leaf(k, Ctx("r"))
        key = (ctx.key, k)
        if key in self.elem:
            return self.elem[key]
        name = f"L{len(self.elem)}"
        vec = self.vec
        if ctx.key == "e":
            kind, idx = "vec", "e"
        elif ctx.parent is not None and ctx.parent.key == "e" and g.kind == "rowb" and g.P % 4 == 0:
            kind, idx = "vec", f"(e % ({T}){g.P}ull)"
        elif ctx.parent is not None and ctx.parent.key == "e" and (g.kind == "scalar" or (g.kind == "colb" and g.Q % 4 == 0)):
            kind, idx = "one", g.expr("e", T)
        else:
            kind, idx = "lane", _chain_index(ctx, f"(e + ({T})l)", T)
        if vec == 1 and kind == "vec":
            kind = "lane"
            idx = idx if idx != "e" else "(e + l)"
        self.order_elem.append((name, kind, ptr, idx))
        ref = f"{name}[q]" if self.cache else f"{name}[l]"
        self.elem[key] = ref
        return ref

    def load_stmts(self, slot_var):
        """Statements loading every element leaf of one slot (c, e defined; q base = slot*VEC)."""
        out = []
        V = self.vec
        for name, kind, ptr, idx in self.order_elem:
            dst = f"{name}[{slot_var} * {V} + l]" if self.cache else f"{name}[l]"
            if kind == "vec":
                out.append(f"{{ float t_[{V}]; tcb::load<{V}>(t_, {ptr} + {idx});"
                           f" _Pragma(\"unroll\") for (int l = 0; l < {V}; ++l) {dst} = t_[l]; }}")
            elif kind == "one":
                out.append(f"{{ const float t_ = tcb::ld1({ptr} + {idx});"
                           f" _Pragma(\"unroll\") for (int l = 0; l < {V}; ++l) {dst} = t_; }}")
            else:
                out.append(f"_Pragma(\"unroll\") for (int l = 0; l < {V}; ++l) {dst} = tcb::ld1({ptr} + {idx});")
        return out


def _rowwise_walk(body, loads, reductions, out_id, row_tier, pattern, sabotage, TPR, GROUPS):
    """Emit every phase of a rowwise body: [(row_lines, elem_lines, k, init, combine, reduce_expr)], output."""
    reduced = {}
    em = _row_emitter(body, loads, reduced, row_tier)
    E, ROW = Ctx("e"), Ctx("r")
    phases = []
    for k, rd in enumerate(reductions):
        em.forget(lambda key: key != "r")
        em.lines, em.row_lines = [], []
        v = em.value(rd.inputs[0], E)
        is_max = rd.op == "max"
        red = f"tcb::group_reduce<{TPR}, {GROUPS}, {'true' if is_max else 'false'}>(acc{k}, red)"
        if sabotage == "layernorm-tree-short" and pattern == "layernorm":
            red = f"acc{k}"  # the bug: the cross-thread tree is skipped
        if sabotage == "softmax-no-max" and is_max and pattern in ("softmax", "log-softmax"):
            red = f"((void){red}, 0.0f)"  # the bug: the shift is never taken
        phases.append((list(em.row_lines), list(em.lines), k,
                       "-__int_as_float(0x7f800000)" if is_max else "0.0f",
                       f"tcb::op_max(acc{k}, {v})" if is_max else f"tcb::op_add(acc{k}, {v})", red))
        reduced[rd.id] = f"red{k}"
        em.memo[("r", rd.id)] = f"red{k}"
    em.forget(lambda key: key != "r")
    em.lines, em.row_lines = [], []
    out_row = row_tier(out_id)
    ov = em.value(out_id, ROW if out_row else E)
    return phases, (list(em.row_lines), list(em.lines), ov, out_row)


def _rowwise_source(body, out_id, pattern, sabotage=None):
    """A fused rowwise kernel (template tcb/rowwise.cuh; reference codegen-fused.js:271-354)."""
    reductions = [n for n in body.nodes if n.op in ("sum", "max")]
    S = body.nodes[reductions[0].inputs[0]].shape
    C = S[-1]
    R = size(S) // C
    T = idx_type(R * C)

    def row_tier(nid):
        s = size(body.nodes[nid].shape)
        return s == R and s != R * C

    # a dry run counts the element-tier leaves, which sets the register budget
    geo = rowwise_geometry(R, C, 1)
    dry = _RowLoads(body, R, C, T, geo["vec"], True)
    _rowwise_walk(body, dry, reductions, out_id, row_tier, pattern, None, geo["tpr"], geo["groups"])
    geo = rowwise_geometry(R, C, len(dry.order_elem))
    V, TPR, GROUPS, SLOTS, ITEMS, CACHE = (geo[k] for k in ("vec", "tpr", "groups", "slots", "items", "cache"))
    loads = _RowLoads(body, R, C, T, V, CACHE)
    phases, (orow, oelem, ov, out_row) = _rowwise_walk(body, loads, reductions, out_id, row_tier, pattern,
                                                        sabotage, TPR, GROUPS)

    def lines(xs, ind):
        return ("\n" + " " * ind).join(xs)

    def item_loop(elem_lines, tail, store):
        """Per-element code over this thread's elements of the row; `store` writes o_[] per slot."""
        if CACHE:
            head = f"""_Pragma("unroll")
      for (int s = 0; s < {SLOTS}; ++s) {{
        const u32 c = (u32)(s * {TPR} + t) * {V};
        if (active && c < {C}u) {{
          const {T} e = ({T})r * ({T}){C} + c; (void)e;"""
            foot = "        }\n      }"
            qdef = f"const int q = s * {V} + l; (void)q;"
        else:
            decl = " ".join(f"float {nm}[{V}];" for nm, _, _, _ in loads.order_elem)
            head = f"""for (u32 c = (u32)t * {V}; active && c < {C}u; c += {TPR * V}u) {{
        {{
          const {T} e = ({T})r * ({T}){C} + c; (void)e;
          {decl}
          {lines(loads.load_stmts("0"), 10)}"""
            foot = "        }\n      }"
            qdef = ""
        body_ = f"""
          {"float o_[" + str(V) + "];" if store else ""}
          _Pragma("unroll")
          for (int l = 0; l < {V}; ++l) {{
            {qdef}
            {lines(elem_lines + tail, 12)}
          }}
          {f"tcb::store<{V}>(out + e, o_);" if store else ""}
"""
        return head + body_ + foot

    parts = []
    for row_lines, elem_lines, k, init, comb, red in phases:
        parts.append(lines(row_lines, 6))
        parts.append(f"float acc{k} = {init};")
        parts.append(item_loop(elem_lines, [f"acc{k} = {comb};"], False))
        parts.append(f"const float red{k} = {red};")
    parts.append(lines(orow, 6))
    if out_row:
        parts.append(f"if (active && t == 0) out[r] = {ov};")
    else:
        parts.append(item_loop(oelem, [f"o_[l] = {ov};"], True))
    cache_decl = cache_load = ""
    if CACHE and loads.order_elem:
        cache_decl = " ".join(f"float {nm}[{ITEMS}];" for nm, _, _, _ in loads.order_elem)
        zero = " ".join(f"{nm}[s * {V} + l] = 0.0f;" for nm, _, _, _ in loads.order_elem)
        cache_load = f"""_Pragma("unroll")
    for (int s = 0; s < {SLOTS}; ++s) {{
      const u32 c = (u32)(s * {TPR} + t) * {V};
      const {T} e = ({T})r * ({T}){C} + c; (void)e;
      if (active && c < {C}u) {{
        {lines(loads.load_stmts("s"), 8)}
      }} else {{
        _Pragma("unroll") for (int l = 0; l < {V}; ++l) {{ {zero} }}
      }}
    }}"""
    nw = max(1, TPR // 32)
    src = f"""// rowwise ({pattern}): R={R} C={C}, {TPR} threads per row, {GROUPS} rows per CTA, vec {V}, {'cached' if CACHE else 'streamed'}
#include "tcb/common.cuh"
#include "tcb/rowwise.cuh"
extern "C" __global__ void __launch_bounds__({TPR * GROUPS}) tcb_rowwise(const tcb::Args a) {{
  tcb::grid_dependency_sync();
  __shared__ float red[{GROUPS * nw}];
  float* __restrict__ out = reinterpret_cast<float*>(a.out);
  const int g = threadIdx.x / {TPR};
  const int t = threadIdx.x % {TPR};
  for (u64 row0 = (u64)blockIdx.x * {GROUPS}; row0 < {R}ull; row0 += (u64)gridDim.x * {GROUPS}) {{
    const u64 r = row0 + g;
    const bool active = r < {R}ull;
    {lines(loads.order_row, 4)}
    {cache_decl}
    {cache_load}
      {lines([p for p in parts if p], 6)}
  }}
}}
"""
    return src, geo, R, C


def _row_emitter(body, loads, reduced, row_tier):
    em = Emitter(body, loads.leaf)
    em.row_lines = []

    def special(nid, ctx):
        node = body.nodes[nid]
        if nid in reduced:
            return reduced[nid]
        if ctx.key == "e" and row_tier(nid):
            return _row_value(em, nid)
        if ctx.key == "e" and node.op == "broadcast":
            src = body.nodes[node.inputs[0]]
            if row_tier(src.id) and src.op not in ("input", "const"):
                return _row_value(em, src.id)
        return None

    em.special = special
    return em


def _row_value(em, nid):
    """A row-tier value: computed in the row context, its statements hoisted before the item loop."""
    key = ("r", nid)
    if key in em.memo:
        return em.memo[key]
    saved = em.lines
    em.lines = []
    v = em.value(nid, Ctx("r"))
    em.row_lines.extend(em.lines)
    em.lines = saved
    return v


# ------------------------------------------------------------------ matmul epilogue
def _epilogue_source(body, out_id, sabotage=None, kernel="simt", bn=None, a_t=False, b_t=False, cross_ba=False):
    root = next(n for n in body.nodes if n.op == "matmul")
    ia, ib = (int(body.nodes[i].attrs["name"][1:]) for i in root.inputs)
    a_s, b_s = body.nodes[root.inputs[0]].shape, body.nodes[root.inputs[1]].shape
    batch, M, K, N = size(a_s[:-2]), a_s[-2], a_s[-1], b_s[-1]
    bias_add = None
    if sabotage == "epilogue-before-bias":
        for n in body.nodes:
            if n.op == "add" and root.id in n.inputs and not all(i == root.id for i in n.inputs):
                if n.id != out_id:
                    bias_add = n
                break
    lines = []
    seen = {}

    def leaf(k, ctx):
        key = (ctx.key, k)
        if key not in seen:
            name = f"x{len(seen)}"
            seen[key] = name
            lines.append(f"const float {name} = tcb::ld1(reinterpret_cast<const float*>(a.in[{k}]) + "
                         f"{_chain_index(ctx, 'i', 'u64')});")
        return seen[key]

    def special(nid, ctx):
        if ctx.key == "i" and (nid == root.id or (bias_add is not None and nid == bias_add.id)):
            return "acc"
        return None

    em = Emitter(body, leaf, special)
    em.lines = lines
    base = Ctx("i")
    out = em.value(out_id, base)
    if bias_add is not None:
        other = next(i for i in bias_add.inputs if i != root.id)
        out = f"tcb::op_add({out}, {em.value(other, base)})"
    code = "\n    ".join(lines)
    tc_defs = ""
    if kernel == "tcgen05":
        fs = fused_split_plan(batch, M, K, N, bn, a_t, b_t)
        splitk, part_off = splitk_plan(batch, M, K, N, bn, fs)
        bk = gemm_bk(bn)
        grid, tail, _, tail_off, _ = tail_plan(batch, M, K, N, bn, bk, splitk, fs)
        tc_defs = (f"#define TCB_KP {_kpad(K)}\n#define TCB_BN {bn}\n#define TCB_BK {bk}\n"
                   f"#define TCB_FS_A {int(fs[0])}\n#define TCB_FS_B {int(fs[1])}\n"
                   f"#define TCB_TMA_STORE {int(tma_store_ok(N, splitk))}\n"
                   f"#define TCB_SPLIT_B_OFFSET {0 if fs[0] else 2 * batch * M * _kpad(K) * 4}ull\n"
                   f"#define TCB_STAGES {gemm_stages(bn, bk)}\n"
                   f"#define TCB_SPLITK {splitk}\n#define TCB_PART_OFFSET {part_off}ull\n"
                   f"#define TCB_GRID {grid}\n#define TCB_TAIL_SPLIT {tail}\n"
                   f"#define TCB_TAIL_OFFSET {tail_off}ull\n"
                   f"#define TCB_A_T {int(a_t)}\n#define TCB_B_T {int(b_t)}\n"
                   + ("#define TCB_CROSS_BA 1\n" if cross_ba else ""))
    src = f"""// matmul epilogue ({kernel}): batch {batch}, [{M},{K}] x [{K},{N}]
#include "tcb/common.cuh"
#define TCB_M {M}
#define TCB_N {N}
#define TCB_K {K}
#define TCB_BATCH {batch}
#define TCB_IA {ia}
#define TCB_IB {ib}
{tc_defs}struct Epi {{
  __device__ __forceinline__ static float apply(const tcb::Args& a, float acc, u64 i, u64 row, u64 col, u64 b) {{
    (void)row; (void)col; (void)b;
    {code}
    return {out};
  }}
}};
#include "tcb/{'gemm_tc' if kernel == 'tcgen05' else 'matmul'}.cuh"
"""
    return src, (batch, M, K, N)


# ------------------------------------------------------------------ tensor-core (tcgen05) path
TC_MIN_K = 32    # below this the 3xTF32 split error could exceed gamma_K's share of the budget: CUDA cores
GEMM_BM = 128
SMEM_LIMIT = 227 * 1024
KPAD = 32   # K is padded to a multiple of 32 in the split operands whatever the K-block
TMA_ATOM32 = 1 << 32   # box_cols flag: 128-byte swizzle of 32-byte chunks (MN-major tf32 tiles)


def _kpad(K):
    return (K + KPAD - 1) // KPAD * KPAD


def gemm_stage_bytes(bn, bk):
    return 2 * GEMM_BM * bk * 4 + 2 * bn * bk * 4


GEMM_STAGING = 4 * 2 * 32 * 32 * 4   # output staging: two 32 x 32 float blocks per epilogue warp


def gemm_stages(bn, bk=32):
    return max(2, min(6, (SMEM_LIMIT - 2048 - GEMM_STAGING) // gemm_stage_bytes(bn, bk)))


def gemm_smem(bn, bk=32):
    """Ring + 1 KB of barriers + output staging + 1 KB to align the ring to 1024 bytes."""
    return gemm_stages(bn, bk) * gemm_stage_bytes(bn, bk) + 1024 + GEMM_STAGING + 1024


def tma_store_ok(N, splitk=1):
    """The epilogue writes through TMA stores (to the output, or with split-K to the partial sums) when a
    row of N floats is a multiple of 16 bytes."""
    return N % 4 == 0


def gemm_bk(bn=128):
    """K-block: 16 floats (64-byte swizzle, 4 stages) with the 256-wide tile, else 32 (128-byte, 3 stages):
    the fastest pair measured on 4096^3 (240.8 vs 229.1 TFLOP/s)."""
    import os
    forced = os.environ.get("TCB_GEMM_BK")
    if forced:
        return int(forced)
    return 16 if bn == 256 else 32


def split_bytes(batch, M, K, N, fs=(False, False)):
    """Scratch taken by the split operands (A_hi, A_lo, then B_hi, B_lo), leaving out an operand the
    GEMM splits itself (fs = (fa, fb))."""
    Kp = _kpad(K)
    return (0 if fs[0] else 2 * batch * M * Kp * 4) + (0 if fs[1] else 2 * batch * N * Kp * 4)


def splitk_plan(batch, M, K, N, bn, fs=(False, False)):
    """K splits so that short, wide-K contractions (weight gradients) still cover the SMs.

    Returns (splits, byte offset of the partial sums in scratch).  Each split keeps >= 4 k-blocks.
    """
    tiles = batch * math.ceil(M / GEMM_BM) * math.ceil(N / bn)
    kb = _kpad(K) // 32
    s = 1
    # up to 8 K ranges per tile are reduced inside the GEMM by the last arriver (tail_plan); split-K
    # with a finishing pass only when the SMs need more than that (tiles <= SMs / 9)
    if tiles < SM_COUNT and SM_COUNT // tiles > 8 and kb >= 8:
        s = max(1, min(SM_COUNT // tiles, kb // 4))   # every SM: 2 tiles x 74 ranges, not 2 x 64
        s = math.ceil(kb / math.ceil(kb / s))  # no empty split
    part_off = split_bytes(batch, M, K, N, fs) + 256
    return s, part_off


def ctrl_bytes(rem):
    """A tensor-core launch's control block: its error word (16 bytes) and 4 arrival counters per split
    tile, 64-byte aligned."""
    return (16 + 16 * rem + 63) // 64 * 64


TAIL_MIN_KB = 32   # a last wave is split along K only with at least this many K-blocks: for K = 256 (16 blocks)
#                    the partial tiles' write and re-read cost more than the fuller wave gains (16384 x 256 x
#                    1024: 67.4 us split, 50.0 not; 4096^3: 602 split, 636 not)


def tail_plan(batch, M, K, N, bn, bk, splitk, fs=(False, False)):
    """The persistent GEMM's grid and K-range split of the tiles of its last wave.

    Returns (grid, tail, rem, tail_off, scratch_end).  grid = min(SMs, tiles) CTAs; when the last wave
    would hold rem <= grid/2 tiles and K has at least TAIL_MIN_KB k-blocks, each of them is cut into
    `tail` K ranges (>= 4 k-blocks each, at most 8) so that wave fills the SMs.  With fewer tiles than SMs that is every tile: grid becomes
    tiles x tail, one range per CTA.  The ranges' partial tiles (128 x bn floats each) sit at tail_off
    in scratch, after the control block; scratch_end is the end of that region (0 when nothing is split).
    """
    tiles = batch * math.ceil(M / GEMM_BM) * math.ceil(N / bn) * splitk
    kbs = _kpad(K) // bk
    if splitk == 1 and tiles < SM_COUNT:
        tail = min(SM_COUNT // tiles, kbs // 4, 8)
        if tail < 2:
            return tiles, 1, 0, 0, 0
        grid, rem = tiles * tail, tiles
    else:
        grid = min(SM_COUNT, tiles)
        rem = tiles % grid
        tail = 1
        if splitk == 1 and rem and 2 * rem <= grid and kbs >= TAIL_MIN_KB:
            tail = min(grid // rem, kbs // 4, 8)
        if tail < 2:
            return grid, 1, 0, 0, 0
    tail_off = split_bytes(batch, M, K, N, fs) + max(256, (ctrl_bytes(rem) + 255) // 256 * 256)
    return grid, tail, rem, tail_off, tail_off + rem * tail * GEMM_BM * bn * 4


FS_MAX_REREAD = 8   # split an operand inside the GEMM when at most this many output tiles load each of its tiles
# (8, not 4: C5's weight gradients, whose B is loaded by 8 tiles, 39.64 -> 39.32 ms per step without the split pass)


def fused_split_plan(batch, M, K, N, bn, a_t=False, b_t=False):
    """(fa, fb): which operands the GEMM splits itself (TCB_FS_A / TCB_FS_B) instead of a split pass.

    An operand qualifies when a TMA copy can read it raw (its row stride a multiple of 16 bytes) and it
    is loaded by few output tiles: A by ceil(N / bn) of them, B by ceil(M / 128).  The in-kernel split
    saves the split pass's write and re-read of hi and lo but repeats the conversion (in shared memory)
    for every tile that loads the operand, so an operand shared by many tiles keeps its split pass.
    TCB_GEMM_FUSED overrides: "0" neither, "1" both, "a" / "b" that operand only (when it qualifies)."""
    import os
    ea = M % 4 == 0 if a_t else K % 4 == 0
    eb = K % 4 == 0 if b_t else N % 4 == 0
    mode = os.environ.get("TCB_GEMM_FUSED")
    if mode == "0":
        return False, False
    if mode == "1":
        return ea, eb
    if mode == "a":
        return ea, False
    if mode == "b":
        return False, eb
    most = int(os.environ.get("TCB_GEMM_FS_REREAD", FS_MAX_REREAD))
    return ea and math.ceil(N / bn) <= most, eb and math.ceil(M / GEMM_BM) <= most


def gemm_bn(N):
    """Accumulator width: 256 TMEM columns when N fills them, 64 when N <= 64 (the batched attention
    products with a head dimension of 64: a wider tile would spend half its tensor-core work on
    padding), else 128 (TCB_GEMM_BN overrides)."""
    import os
    forced = os.environ.get("TCB_GEMM_BN")
    if forced:
        return int(forced)
    return 256 if N >= 256 else 64 if N <= 64 else 128


def _tc_epilogue_launch(body, out_id, node_id, op, kind, pattern, inputs, sabotage=None, a_t=False, b_t=False,
                        cross_ba=False):
    root = next(n for n in body.nodes if n.op == "matmul")
    N = body.nodes[root.inputs[1]].shape[-1]
    bn = gemm_bn(N)
    code, (batch, M, K, N) = _epilogue_source(body, out_id, sabotage, kernel="tcgen05", bn=bn, a_t=a_t, b_t=b_t,
                                              cross_ba=cross_ba)
    if batch > 65535 or math.ceil(M / GEMM_BM) > 65535:
        raise ValueError("matmul grid too large")
    Kp = _kpad(K)
    fs = fused_split_plan(batch, M, K, N, bn, a_t, b_t)
    err_off = split_bytes(batch, M, K, N, fs)
    splitk, part_off = splitk_plan(batch, M, K, N, bn, fs)
    bk = gemm_bk(bn)
    grid, tail, rem, _, tail_end = tail_plan(batch, M, K, N, bn, bk, splitk, fs)
    scratch = max(err_off + 256 + (splitk * batch * M * N * 4 if splitk > 1 else 0), tail_end)
    gemm = KernelCall("tcb_gemm_tc", (grid, 1, 1), (320 if any(fs) else 192, 1, 1), gemm_smem(bn, bk), [])
    gemm.err_offset = err_off
    a_bytes = 0 if fs[0] else batch * M * Kp * 4
    b_off = 2 * a_bytes
    b_bytes = batch * N * Kp * 4
    ia, ib = (int(body.nodes[i].attrs["name"][1:]) for i in root.inputs)
    # tensor maps [A_hi or raw A, A_lo, B_hi or raw B, B_lo]: split operands from scratch, raw ones from
    # the launch operand in K-major {K, rows} boxes or MN-major {32, bk} boxes (a raw operand's second
    # slot repeats its map and is not read)
    if fs[0]:
        ra = (("in", ia, M, K, batch, M * 4, K * M * 4, 32 | TMA_ATOM32, bk) if a_t else
              ("in", ia, K, M, batch, K * 4, M * K * 4, bk, GEMM_BM))
        maps = [ra, ra]
    else:
        maps = [("scratch", 0, Kp, M, batch, Kp * 4, M * Kp * 4, bk, GEMM_BM),
                ("scratch", a_bytes, Kp, M, batch, Kp * 4, M * Kp * 4, bk, GEMM_BM)]
    if fs[1]:
        rb = (("in", ib, K, N, batch, K * 4, N * K * 4, bk, bn) if b_t else
              ("in", ib, N, K, batch, N * 4, K * N * 4, 32 | TMA_ATOM32, bk))
        maps += [rb, rb]
    else:
        maps += [("scratch", b_off, Kp, N, batch, Kp * 4, N * Kp * 4, bk, bn),
                 ("scratch", b_off + b_bytes, Kp, N, batch, Kp * 4, N * Kp * 4, bk, bn)]
    if tma_store_ok(N, splitk):
        maps.append(("out", 0, N, M, batch, N * 4, M * N * 4, 32, 32) if splitk == 1 else
                    ("scratch", part_off, N, M, splitk * batch, N * 4, M * N * 4, 32, 32))
    gemm.tma = maps
    if fs[0]:
        first = KernelCall("tcb_gemm_prep", (1, 1, 1), (128, 1, 1))
    else:
        first = KernelCall("tcb_split_a", (Kp // 32, math.ceil(M / 32), batch) if a_t
                           else grid1d(batch * M * Kp, per_thread=4), (256, 1, 1))
    first.err_offset = err_off
    calls = [first]
    if not fs[1]:
        calls.append(KernelCall("tcb_split_b", grid1d(batch * N * Kp, per_thread=4) if b_t
                                else (Kp // 32, math.ceil(N / 32), batch), (256, 1, 1)))
    calls.append(gemm)
    if splitk > 1:
        calls.append(KernelCall("tcb_splitk_finish", grid1d(batch * M * N, per_thread=1), (256, 1, 1)))
    lau = Launch(node_id, op, kind, pattern, inputs, code, calls, scratch_bytes=scratch,
                 info={"mnk": (batch, M, K, N), "bn": bn, "bk": bk, "stages": gemm_stages(bn, bk), "splitk": splitk,
                       "tail_split": tail, "ctrl_bytes": ctrl_bytes(rem), "fused_split": fs,
                       "path": "tcgen05-3xtf32", "a_t": a_t, "b_t": b_t, "ia": ia, "ib": ib, "kp": Kp})
    return lau


def split_multi_source():
    """The module of tcb_split_multi (the operand splits of many GEMMs in one launch)."""
    return '#include "tcb/common.cuh"\n#include "tcb/split.cuh"\n'



# ------------------------------------------------------------------ plain reduce
SM_COUNT = 148


def _reduce_source(op, in_shape, axis):
    outer = size(in_shape[:axis])
    n = in_shape[axis]
    inner = size(in_shape[axis + 1:])
    outs = outer * inner
    split = 1
    if inner > 1 and outs < 2 * SM_COUNT * 256 and n >= 64:
        # at most 65535 chunks: the chunk index is the grid's y coordinate
        split = max(1, min(math.ceil(n / 32), math.ceil(SM_COUNT * 2048 / max(1, outs)), 65535))
    src = f"""// {op} over axis {axis} of {list(in_shape)}: outer {outer}, n {n}, inner {inner}, split {split}
#include "tcb/common.cuh"
#define TCB_OUTER {outer}
#define TCB_N {n}
#define TCB_INNER {inner}
#define TCB_SPLIT {split}
#define TCB_IS_MAX {1 if op == 'max' else 0}
#include "tcb/reduce.cuh"
"""
    return src, (outer, n, inner, split)


# ------------------------------------------------------------------ launches
class KernelCall:
    """One kernel launch of a Launch: entry name, grid, block, dynamic smem, p[] parameters.

    ``tma``: tensor maps to build at launch, each (region, offset, cols, rows, batches, row_stride_bytes,
    batch_stride_bytes, box_cols, box_rows) with region 'scratch' (offset = bytes into scratch), 'in'
    (offset = the launch operand's index) or 'out'; ``err_offset``: where in scratch the
    kernel's error word lives (its address goes in p[15]).  A launch with two outputs (an elementwise
    value and its column sum) names the second through ``out_node`` / ``ptr_params``.
    """
    __slots__ = ("name", "grid", "block", "smem", "params", "tma", "err_offset", "out_node", "ptr_params")

    def __init__(self, name, grid, block, smem=0, params=()):
        self.name, self.grid, self.block, self.smem, self.params = name, tuple(grid), tuple(block), smem, list(params)
        self.tma = None
        self.err_offset = None
        self.out_node = None     # a node whose buffer is this call's `out` instead of the launch's node
        self.ptr_params = ()     # (k, node): p[k] gets that node's device address

    def __repr__(self):
        return f"KernelCall({self.name}, grid={self.grid}, block={self.block})"


class Launch:
    """One node's work: the reference's launch record ``{node, op, kind, pattern, inputs, params, grid, code}``
    (src/gpu/lower.js:108-111, src/fusion/lower-fused.js:37-41) with CUDA source and kernel calls."""
    __slots__ = ("node", "op", "kind", "pattern", "inputs", "code", "calls", "scratch_bytes", "bytes", "info",
                 "nodes")   # `nodes`: every node a launch with two outputs produces (unset otherwise)

    def __init__(self, node, op, kind, pattern, inputs, code, calls, scratch_bytes=0, info=None):
        self.node, self.op, self.kind, self.pattern = node, op, kind, pattern
        self.inputs = list(inputs)
        self.code = code
        self.calls = calls
        self.scratch_bytes = scratch_bytes
        self.bytes = 0
        self.info = info or {}

    def __repr__(self):
        return f"Launch(node={self.node}, kind={self.kind}, pattern={self.pattern}, calls={len(self.calls)})"


def grid1d(n, per_thread=4, block=WG, waves=8):
    """CTAs for a grid-stride 1-D kernel over n elements (at most `waves` CTAs per SM)."""
    chunks = max(1, math.ceil(n / per_thread))
    return (max(1, min(math.ceil(chunks / block), SM_COUNT * waves)), 1, 1)


def copy_source(w=4):
    """An elementwise source that copies its operand (out[i] = in0[i]), `w` floats per step; the element
    count comes from p[0], so one module serves copies of every size (a resident program's feedback)."""
    return f"""// device copy, {w} floats per step
#include "tcb/common.cuh"
#define TCB_W {w}
struct Body {{
  template <int W> struct Regs {{
    float x0[W];
  }};
  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {{
    tcb::load<W>(r.x0, reinterpret_cast<const float*>(a.in[0]) + i0);
  }}
  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[W]) {{
#pragma unroll
    for (int l = 0; l < W; ++l) o[l] = r.x0[l];
  }}
}};
#include "tcb/elementwise.cuh"
"""


def _ew_launch(body, out_id, n, kind, node_id, op, pattern, inputs, sabotage=None, tag="elementwise"):
    code = _elementwise_source(body, out_id, n, tag=tag)
    count = n + 1 if sabotage == "fused-bounds-off-by-one" else n
    call = KernelCall("tcb_elementwise", grid1d(n), (WG, 1, 1), 0, [count])
    return Launch(node_id, op, kind, pattern, inputs, code, [call])


def uses_tensor_cores(a_shape, matmul):
    return matmul == "tiled" and a_shape[-1] >= TC_MIN_K


def _epilogue_launch(body, out_id, node_id, op, kind, pattern, inputs, matmul, sabotage=None, a_t=False, b_t=False,
                     cross_ba=False):
    """`matmul`: 'naive' -> the CUDA-core fp32 kernel; 'tiled' -> tcgen05 3xTF32 when K >= TC_MIN_K.

    `a_t` / `b_t`: the operand's slot holds its transpose (a folded transposeLast2, tensor-core path only).
    `cross_ba`: issue the two mixed 3xTF32 products as A_hi.B_lo then A_lo.B_hi (a transposed product
    computing (A.B)^T = B^T.A^T adds its terms in the order A.B would).
    """
    root = next(n for n in body.nodes if n.op == "matmul")
    if uses_tensor_cores(body.nodes[root.inputs[0]].shape, matmul):
        return _tc_epilogue_launch(body, out_id, node_id, op, kind, pattern, inputs, sabotage, a_t, b_t, cross_ba)
    if a_t or b_t:
        raise ValueError("transposed operands are folded only on the tensor-core path")
    code, (batch, M, K, N) = _epilogue_source(body, out_id, sabotage)
    if batch > 65535:
        raise ValueError("matmul batch above 65535")
    call = KernelCall("tcb_matmul", (math.ceil(N / 128), math.ceil(M / 128), batch), (256, 1, 1), 0, [])
    return Launch(node_id, op, kind, pattern, inputs, code, [call], info={"mnk": (batch, M, K, N)})


def _rowwise_launch(body, out_id, node_id, pattern, inputs, sabotage=None):
    code, geo, R, C = _rowwise_source(body, out_id, pattern, sabotage)
    rows_per_cta = geo["groups"]
    ctas = max(1, min(math.ceil(R / rows_per_cta), SM_COUNT * max(1, 2048 // geo["block"]) * 4))
    call = KernelCall("tcb_rowwise", (ctas, 1, 1), (geo["block"], 1, 1), 0, [])
    return Launch(node_id, "fused", "fused-rowwise", pattern, inputs, code, [call], info={"R": R, "C": C, **geo})


def _reduce_launch(op, in_shape, axis, node_id, inputs):
    code, (outer, n, inner, split) = _reduce_source(op, in_shape, axis)
    outs = outer * inner
    if inner == 1:
        calls = [KernelCall("tcb_reduce_rows", (max(1, min(math.ceil(outer * 32 / 256), SM_COUNT * 8)), 1, 1),
                            (256, 1, 1))]
        scratch = 0
    else:
        gx = max(1, min(math.ceil(outs / 256), SM_COUNT * 8))
        calls = [KernelCall("tcb_reduce_cols", (gx, split, 1), (256, 1, 1))]
        scratch = 0
        if split > 1:
            calls.append(KernelCall("tcb_reduce_finish", (max(1, min(math.ceil(outs / 32), SM_COUNT * 8)), 1, 1),
                                    (256, 1, 1)))
            scratch = split * outs * 4
    return Launch(node_id, op, op, None, inputs, code, calls, scratch_bytes=scratch,
                  info={"outer": outer, "n": n, "inner": inner, "split": split})


def _one_op_body(op, in_shapes, attrs):
    from .ir import Graph
    g = Graph()
    ins = [g.input(f"a{k}", s) for k, s in enumerate(in_shapes)]
    out = g.emit(op, ins, attrs)
    return g, out


def _plain_launch_uncached(op, in_shapes, attrs, matmul):
    body, out = _one_op_body(op, in_shapes, attrs)
    n = size(body.nodes[out].shape)
    if op in ("sum", "max"):
        return _reduce_launch(op, in_shapes[0], attrs["axis"], -1, [])
    if op == "matmul":
        return _epilogue_launch(body, out, -1, "matmul", f"matmul-{matmul}", None, [], matmul)
    if op in _BIN or op in _UN:
        kind = "copy" if op == "stopGradient" else op
        return _ew_launch(body, out, n, kind, -1, op, None, [], tag=f"plain {op}")
    if op in ("broadcast", "transpose", "reshape"):
        return _ew_launch(body, out, n, "gather", -1, op, None, [], tag=f"plain {op} (gather)")
    raise ValueError(f"no lowering for '{op}'")


_plain_cache = {}


_GEMM_ENV = ("TCB_GEMM_FUSED", "TCB_GEMM_FS_REREAD", "TCB_GEMM_BK", "TCB_GEMM_BN")


def _plain_launch(graph, node, matmul):
    """The launch one node gets alone, cached by (op, shapes, attrs, matmul) (src/fusion/lower-fused.js:13-25)
    and by the GEMM tile overrides in the environment, which change a matmul's launch."""
    import json
    import os
    shapes = [list(graph.nodes[i].shape) for i in node.inputs]
    env = [os.environ.get(k) for k in _GEMM_ENV] if node.op == "matmul" else None
    key = json.dumps([node.op, shapes, node.attrs, matmul, env], sort_keys=True)
    one = _plain_cache.get(key)
    if one is None:
        one = _plain_cache[key] = _plain_launch_uncached(node.op, shapes, node.attrs, matmul)
    lau = Launch(node.id, node.op, one.kind, None, node.inputs, one.code, one.calls, one.scratch_bytes, one.info)
    return lau


def _bytes(graph, lau):
    """Amendment 33 (src/fusion/workloads.js:170-172): each distinct operand once at its own size, plus the output."""
    b = sum(size(graph.nodes[i].shape) * 4 for i in dict.fromkeys(lau.inputs))
    return b + size(graph.nodes[lau.node].shape) * 4


def _is_last2_swap(node):
    p = node.attrs.get("perm")
    r = len(p)
    return r >= 2 and p[:-2] == list(range(r - 2)) and p[-2:] == [r - 1, r - 2]


def _matmul_operands(graph, node):
    """(node of the contraction's A, node of its B) as graph ids, for a plain matmul or an epilogue node."""
    if node.op == "matmul":
        return node.inputs[0], node.inputs[1]
    if node.op == "fused" and node.attrs["kind"] == "epilogue":
        from .fuse import body_of
        b = body_of(node)
        root = next(n for n in b.nodes if n.op == "matmul")
        ia, ib = (int(b.nodes[i].attrs["name"][1:]) for i in root.inputs)
        # an operand slot used anywhere else in the body is read at output indices: not foldable
        uses = {}
        for n in b.nodes:
            for i in n.inputs:
                uses[i] = uses.get(i, 0) + 1
        if uses.get(root.inputs[0], 0) != 1 or uses.get(root.inputs[1], 0) != 1 or root.inputs[0] == root.inputs[1]:
            return None
        return node.inputs[ia], node.inputs[ib]
    return None


def foldable_transposes(graph, matmul, keep=()):
    """Plain transposeLast2 nodes read only as tensor-core GEMM operands, or by other such nodes that fold:
    their launch can be dropped and the GEMM's operand split reads the source at the end of the chain
    instead (the split rewrites the layout anyway; two swaps cancel).  Autodiff makes such chains: the
    backward of x^T reads transpose(x^T).  Readers come after what they read, so one pass from the end
    sees every reader's verdict first."""
    keep = set(keep)
    consumers = {}
    for n in graph.nodes:
        for i in n.inputs:
            consumers.setdefault(i, []).append(n)
    folds = set()
    for t in reversed(graph.nodes):
        if t.op != "transpose" or t.id in keep or not _is_last2_swap(t) or t.id not in consumers:
            continue
        ok = True
        for c in consumers[t.id]:
            if c.id in folds:
                continue
            ops = _matmul_operands(graph, c)
            if ops is None or t.id not in ops or not uses_tensor_cores(graph.nodes[ops[0]].shape, matmul):
                ok = False
                break
        if ok:
            folds.add(t.id)
    return folds


def _unfold(graph, i, folds):
    """(the node a GEMM operand slot reads through a chain of folded transposes, whether it is transposed)."""
    t = False
    while i in folds:
        i, t = graph.nodes[i].inputs[0], not t
    return i, t


def _folded_launch(graph, node, matmul, sabotage, folds):
    """The GEMM launch of `node` with folded transposed operands substituted by their sources."""
    from .fuse import body_of
    a, b = _matmul_operands(graph, node)
    a_t, b_t = _unfold(graph, a, folds)[1], _unfold(graph, b, folds)[1]
    if node.op == "matmul":
        shapes = [list(graph.nodes[i].shape) for i in node.inputs]
        body, out = _one_op_body("matmul", shapes, node.attrs)
        lau = _epilogue_launch(body, out, node.id, "matmul", f"matmul-{matmul}", None, list(node.inputs), matmul,
                               None, a_t, b_t)
    else:
        lau = _epilogue_launch(body_of(node), node.attrs["output"], node.id, "fused", "fused-epilogue",
                               node.attrs["pattern"], list(node.inputs), matmul,
                               sabotage if sabotage in FUSED_SABOTAGE else None, a_t, b_t)
    lau.inputs = [_unfold(graph, i, folds)[0] for i in node.inputs]
    return lau


def transposed_products(graph, matmul, keep=(), folds=()):
    """{transposeLast2 id: matmul id} for a plain tensor-core matmul C = A.B whose only reader is a
    transposeLast2 that does not itself fold into a GEMM: the pair becomes one GEMM computing
    C^T = B^T.A^T directly -- no transpose pass over C, and when C has few rows (attention's
    [64, 256] products of a head dimension of 64) no 128-row tile half spent on padding.  Autodiff
    makes these: the gradient of K^T's reader, transposed back."""
    keep, folds = set(keep), set(folds)
    consumers = {}
    for n in graph.nodes:
        for i in n.inputs:
            consumers.setdefault(i, []).append(n.id)
    out = {}
    for T in graph.nodes:
        if T.op != "transpose" or not _is_last2_swap(T) or T.id in folds:
            continue
        M = graph.nodes[T.inputs[0]]
        if (M.op != "matmul" or M.id in keep or consumers.get(M.id) != [T.id]
                or not uses_tensor_cores(graph.nodes[M.inputs[0]].shape, matmul)):
            continue
        out[T.id] = M.id
    return out


def _transposed_product_launch(graph, T, M, matmul, folds):
    """The GEMM launch of node T = transpose(M), M = A.B: T = B^T.A^T, each operand read through its
    folded transposes with the swapped flag (the slot of B^T holds B's source, transposed when B is
    not itself a transpose, and likewise for A^T)."""
    a_src, a_t = _unfold(graph, M.inputs[0], folds)
    b_src, b_t = _unfold(graph, M.inputs[1], folds)
    sa, sb = list(graph.nodes[M.inputs[0]].shape), list(graph.nodes[M.inputs[1]].shape)
    shapes = [sb[:-2] + [sb[-1], sb[-2]], sa[:-2] + [sa[-1], sa[-2]]]
    body, out = _one_op_body("matmul", shapes, M.attrs)
    lau = _epilogue_launch(body, out, T.id, "matmul", f"matmul-{matmul}", None, [b_src, a_src], matmul, None,
                           not b_t, not a_t, cross_ba=True)
    lau.inputs = [b_src, a_src]
    lau.bytes = _bytes(graph, lau)
    return lau


def lower(graph, matmul="naive", sabotage=None, fold=False, keep=()):
    """One launch per op, no fusion (src/gpu/lower.js:68-114).  `fold`: drop transposes feeding GEMM
    operands, and compute a GEMM read only by a transpose as the transposed product."""
    folds = foldable_transposes(graph, matmul, keep) if fold else set()
    tprods = transposed_products(graph, matmul, keep, folds) if fold else {}
    tmats = set(tprods.values())
    launches = []
    for node in graph.nodes:
        if node.op in ("input", "const") or node.id in folds or node.id in tmats:
            continue
        if node.id in tprods:
            launches.append(_transposed_product_launch(graph, node, graph.nodes[tprods[node.id]], matmul, folds))
            continue
        if folds and _matmul_operands(graph, node) and set(_matmul_operands(graph, node)) & folds:
            lau = _folded_launch(graph, node, matmul, sabotage, folds)
        else:
            lau = _plain_launch(graph, node, matmul)
        lau.bytes = _bytes(graph, lau)
        launches.append(lau)
    return {"launches": launches, "folded": sorted(folds), "transposed": sorted(tprods.items())}


# ------------------------------------------------------------------ elementwise + column sum
def _elementwise_producer(node):
    if node.op == "fused":
        return node.attrs["kind"] == "elementwise"
    return node.op in _BIN or node.op in _UN


def colsum_fusions(graph, keep=()):
    """Column sums to fuse with their producer: {sum id: (producer id, write)}.

    A `sum` over axis 0 of a value with more than one column whose producer is an elementwise launch (a
    fused elementwise node or a plain elementwise op) is computed in the producer's pass over the
    tensor (tcb/colsum.cuh).  `write`: the producer's value is kept or read by another node, so the
    fused launch still stores it; otherwise it is never materialised.  The reference's pass leaves these
    sums plain (src/fusion/fuse.js:43-45)."""
    keep = set(keep)
    consumers = {}
    for n in graph.nodes:
        for i in n.inputs:
            consumers.setdefault(i, []).append(n.id)
    out, taken = {}, set()
    for S in graph.nodes:
        if S.op != "sum" or S.attrs["axis"] != 0:
            continue
        P = graph.nodes[S.inputs[0]]
        if P.id in taken or len(P.shape) < 2 or size(P.shape[1:]) <= 1 or not _elementwise_producer(P):
            continue
        out[S.id] = (P.id, P.id in keep or len(consumers[P.id]) > 1)
        taken.add(P.id)
    return out


ROWSUM_MIN_ROWS = SM_COUNT * 8   # a warp per row: fewer rows would leave the producer's pass short of warps


def rowsum_fusions(graph, keep=(), exclude=()):
    """Sums over the last axis to fuse with their producer: {sum id: (producer id, write)}.

    A `sum` over the last axis of an elementwise value (a fused elementwise node or a plain elementwise
    op) with at least ROWSUM_MIN_ROWS rows is computed in the producer's pass (tcb/rowsum.cuh); `write`
    as for column sums.  Sums and producers in `exclude` (already fused otherwise) are left alone."""
    keep, exclude = set(keep), set(exclude)
    consumers = {}
    for n in graph.nodes:
        for i in n.inputs:
            consumers.setdefault(i, []).append(n.id)
    out, taken = {}, set()
    for S in graph.nodes:
        if S.op != "sum" or S.id in exclude:
            continue
        P = graph.nodes[S.inputs[0]]
        if (len(P.shape) < 2 or S.attrs["axis"] != len(P.shape) - 1 or P.id in taken or P.id in exclude
                or size(P.shape[:-1]) < ROWSUM_MIN_ROWS or not _elementwise_producer(P)):
            continue
        out[S.id] = (P.id, P.id in keep or len(consumers[P.id]) > 1)
        taken.add(P.id)
    return out


def _rowsum_launch(graph, P, S, write):
    """One launch computing elementwise node P over [R, C] and S = its sum over the last axis
    (tcb/rowsum.cuh), in tcb_reduce_rows's order, so the sums are bitwise the unfused pair's."""
    from .fuse import body_of
    if P.op == "fused":
        body, out_id = body_of(P), P.attrs["output"]
    else:
        body, out_id = _one_op_body(P.op, [graph.nodes[i].shape for i in P.inputs], P.attrs)
    R, C = size(P.shape[:-1]), P.shape[-1]
    src = f"""// elementwise ({P.op}) + sum over the last axis of [{R}, {C}], value {'stored' if write else 'not stored'}
#include "tcb/common.cuh"
#define TCB_OUTER {R}
#define TCB_N {C}
#define TCB_INNER 1
#define TCB_SPLIT 1
#define TCB_IS_MAX 0
#define TCB_WRITE {int(write)}
{_ew_body_struct(body, out_id, R * C)}#include "tcb/rowsum.cuh"
"""
    main = KernelCall("tcb_ew_rowsum", (max(1, min(math.ceil(R * 32 / 256), SM_COUNT * 8)), 1, 1), (256, 1, 1))
    if write:
        main.ptr_params = ((14, S.id),)
    lau = Launch(P.id if write else S.id, "fused", "fused-rowsum", "elementwise+rowsum", list(P.inputs), src, [main],
                 info={"R": R, "C": C, "write": write, "producer": P.id, "sum": S.id})
    if write:
        lau.nodes = [P.id, S.id]
    nbytes = sum(size(graph.nodes[i].shape) * 4 for i in dict.fromkeys(P.inputs)) + R * 4
    lau.bytes = nbytes + (R * C * 4 if write else 0)
    return lau


def _colsum_launch(graph, P, S, write):
    """One launch computing elementwise node P over [R, C] and S = sum over axis 0 of it (tcb/colsum.cuh),
    with the plain column sum's split, so the sum is bitwise the unfused pair's."""
    from .fuse import body_of
    if P.op == "fused":
        body, out_id = body_of(P), P.attrs["output"]
    else:
        body, out_id = _one_op_body(P.op, [graph.nodes[i].shape for i in P.inputs], P.attrs)
    R, C = P.shape[0], size(P.shape[1:])
    _, (_, _, _, split) = _reduce_source("sum", list(P.shape), 0)
    # 128-bit lanes only when the split already gives every SM a full complement of threads; the plain
    # sum's split aims at one thread per column and chunk (148 x 2048), which single lanes keep
    W = 4 if C % 4 == 0 and (C // 4) * split >= SM_COUNT * 1024 else 1
    src = f"""// elementwise ({P.op}) + column sum over axis 0 of [{R}, {C}], split {split}, value {'stored' if write else 'not stored'}
#include "tcb/common.cuh"
#define TCB_OUTER 1
#define TCB_N {R}
#define TCB_INNER {C}
#define TCB_SPLIT {split}
#define TCB_IS_MAX 0
#define TCB_W {W}
#define TCB_WRITE {int(write)}
{_ew_body_struct(body, out_id, R * C)}#include "tcb/colsum.cuh"
"""
    groups = C // W
    block = min(256, max(32, -(-groups // 32) * 32))
    main = KernelCall("tcb_ew_colsum", (max(1, min(math.ceil(groups / block), SM_COUNT * 8)), split, 1), (block, 1, 1))
    calls = [main]
    if write and split == 1:
        main.ptr_params = ((14, S.id),)
    if split > 1:
        fin = KernelCall("tcb_reduce_finish", (max(1, min(math.ceil(C / 32), SM_COUNT * 8)), 1, 1), (256, 1, 1))
        if write:
            fin.out_node = S.id
        calls.append(fin)
    lau = Launch(P.id if write else S.id, "fused", "fused-colsum", "elementwise+colsum", list(P.inputs), src, calls,
                 scratch_bytes=split * C * 4 if split > 1 else 0,
                 info={"R": R, "C": C, "split": split, "write": write, "producer": P.id, "sum": S.id})
    if write:
        lau.nodes = [P.id, S.id]
    nbytes = sum(size(graph.nodes[i].shape) * 4 for i in dict.fromkeys(P.inputs)) + C * 4
    lau.bytes = nbytes + (R * C * 4 if write else 0)
    return lau


# ------------------------------------------------------------------ one pass, several elementwise outputs
MO_MAX_OPERANDS = 8


def _reads_directly(node, k):
    """Whether operand slot k of an elementwise launch's node is read only at the output's own index
    (a plain op reads every operand so; a fused body must use input a<k> only in elementwise ops)."""
    if node.op != "fused":
        return True
    from .fuse import body_of
    body = body_of(node)
    nid = next(n.id for n in body.nodes if n.op == "input" and n.attrs["name"] == f"a{k}")
    return all(n.op in _BIN or n.op in _UN for n in body.nodes if nid in n.inputs)


def mo_fusions(graph, keep=(), exclude=()):
    """Readers computed in their producer's pass: {producer id: reader id}.

    A producer is an elementwise launch (a fused elementwise node or a plain elementwise op) whose value
    must be stored (another node or the caller reads it); a reader qualifies when it is an elementwise
    launch of the same shape that reads the producer at its own index, and every other operand it has
    is a graph input, a constant or a value produced earlier, so the one launch can stand at the
    producer's place.  Each node takes part in one pair at most; together they read at most 8 operands.
    With `keep` given, a reader qualifies only if a kept value depends on it (a resident program leaves
    the other readers out altogether).  `exclude`: nodes another rewrite already owns (fused column
    sums, folded transposes)."""
    exclude = set(exclude)
    live = None
    if keep:
        live = set(keep)
        for n in reversed(graph.nodes):
            if n.id in live:
                live.update(n.inputs)
    consumers = {}
    for n in graph.nodes:
        for i in n.inputs:
            consumers.setdefault(i, []).append(n.id)
    used, out = set(exclude), {}
    for P in graph.nodes:
        if P.id in used or not _elementwise_producer(P):
            continue
        for qid in consumers.get(P.id, []):
            Q = graph.nodes[qid]
            if qid in used or not _elementwise_producer(Q) or Q.shape != P.shape or (live is not None and qid not in live):
                continue
            if any(i != P.id and not (graph.nodes[i].op in ("input", "const") or i < P.id) for i in Q.inputs):
                continue
            if not all(_reads_directly(Q, k) for k, i in enumerate(Q.inputs) if i == P.id):
                continue
            operands = list(dict.fromkeys(list(P.inputs) + [i for i in Q.inputs if i != P.id]))
            if len(operands) > MO_MAX_OPERANDS:
                continue
            out[P.id] = qid
            used.update((P.id, qid))
            break
    return out


def _body_and_output(graph, node):
    from .fuse import body_of
    if node.op == "fused":
        return body_of(node), node.attrs["output"]
    return _one_op_body(node.op, [graph.nodes[i].shape for i in node.inputs], node.attrs)


def _merged_body(graph, P, Q):
    """One body computing P and its reader Q: operands = P's operands then Q's other ones (first
    appearance order); Q's reads of P use P's value.  Returns (body, [P's output, Q's output], operands)."""
    from .ir import Graph
    operands = list(dict.fromkeys(list(P.inputs) + [i for i in Q.inputs if i != P.id]))
    g = Graph()
    slot = {nid: g.input(f"a{k}", graph.nodes[nid].shape) for k, nid in enumerate(operands)}
    outs = []
    for node, reads_p in ((P, None), (Q, P.id)):
        body, out = _body_and_output(graph, node)
        remap = {}
        for n in body.nodes:
            if n.op == "input":
                src = node.inputs[int(n.attrs["name"][1:])]
                remap[n.id] = outs[0] if src == reads_p else slot[src]
            else:
                remap[n.id] = g.emit(n.op, [remap[i] for i in n.inputs], n.attrs)
        outs.append(remap[out])
    return g, outs, operands


def _mo_source(body, out_ids, n):
    """The elementwise-with-several-outputs kernel of a merged body (tcb/elementwise_mo.cuh)."""
    T = idx_type(n)
    loads = _EwLoads("W", T)
    em = Emitter(body, loads.leaf)
    base = Ctx("i")
    outs = [em.value(o, base) for o in out_ids]
    fields = "\n    ".join(loads.fields) or "float unused_;"
    stmts = "\n    ".join(loads.stmts)
    lanes = "\n      ".join(loads.per_lane)
    per_lane = f"#pragma unroll\n    for (int l = 0; l < W; ++l) {{\n      {lanes}\n    }}" if loads.per_lane else ""
    comp = "\n      ".join(em.lines)
    stores = "\n      ".join(f"o[{k}][l] = {v};" for k, v in enumerate(outs))
    return f"""// elementwise, {len(out_ids)} outputs: generated from a body of {len(body.nodes)} nodes, {n} elements
#include "tcb/common.cuh"
#define TCB_W 4
#define TCB_NOUT {len(out_ids)}
struct Body {{
  template <int W> struct Regs {{
    {fields}
  }};
  template <int W> __device__ __forceinline__ static void load(const tcb::Args& a, u64 i0, Regs<W>& r) {{
    {stmts}
    {per_lane}
  }}
  template <int W> __device__ __forceinline__ static void compute(const Regs<W>& r, float (&o)[TCB_NOUT][W]) {{
#pragma unroll
    for (int l = 0; l < W; ++l) {{
      {comp}
      {stores}
    }}
  }}
}};
#include "tcb/elementwise_mo.cuh"
"""


def _mo_launch(graph, P, Q):
    body, out_ids, operands = _merged_body(graph, P, Q)
    n = size(P.shape)
    call = KernelCall("tcb_elementwise_mo", grid1d(n), (WG, 1, 1), 0, [n])
    call.ptr_params = ((1, Q.id),)
    lau = Launch(P.id, "fused", "fused-multi", "elementwise+reader", operands, _mo_source(body, out_ids, n), [call],
                 info={"producer": P.id, "reader": Q.id, "outputs": 2})
    lau.nodes = [P.id, Q.id]
    lau.bytes = sum(size(graph.nodes[i].shape) * 4 for i in operands) + 2 * n * 4
    return lau


def fused_kernel(node, matmul="naive", sabotage=None):
    """The launch of a fused node (src/fusion/codegen-fused.js:357-362)."""
    from .fuse import body_of
    body = body_of(node)
    out = node.attrs["output"]
    kind = node.attrs["kind"]
    sab = sabotage if sabotage in FUSED_SABOTAGE else None
    if kind == "elementwise":
        return _ew_launch(body, out, size(node.shape), "fused-elementwise", node.id, "fused", node.attrs["pattern"],
                          node.inputs, sab, tag=f"fused elementwise ({len(node.inputs)} operands)")
    if kind == "epilogue":
        return _epilogue_launch(body, out, node.id, "fused", "fused-epilogue", node.attrs["pattern"], node.inputs,
                                matmul, sab)
    if kind == "rowwise":
        return _rowwise_launch(body, out, node.id, node.attrs["pattern"], node.inputs, sab)
    raise ValueError(f"no fused kernel kind '{kind}'")


def lower_fused(graph, matmul="naive", sabotage=None, fold=False, keep=(), colfuse=False, mofuse=False):
    """A fused node to its kernel, every other node to its plain launch (src/fusion/lower-fused.js:32-45).

    `fold` (resident programs only): transposeLast2 nodes read only as tensor-core GEMM operands get no
    launch; the GEMM's operand split reads their source; a GEMM read only by a transposeLast2 computes
    the transposed product itself (transposed_products).  Their values then never exist on the device,
    so verification runs that read back every node lower without it.
    `colfuse` (resident programs only): a sum over axis 0 runs in its elementwise producer's launch
    (colsum_fusions), and so does a sum over the last axis of enough rows (rowsum_fusions); a producer
    read by nothing else is then never stored.  `keep` names the values that must exist after the
    launches.
    `mofuse` (resident programs only): an elementwise reader whose other operands already exist is
    computed in its elementwise producer's launch, both stored (mo_fusions).
    """
    folds = foldable_transposes(graph, matmul, keep) if fold else set()
    tprods = transposed_products(graph, matmul, keep, folds) if fold else {}
    tmats = set(tprods.values())
    cols = colsum_fusions(graph, keep) if colfuse else {}
    rows = rowsum_fusions(graph, keep, exclude=set(cols) | {p for p, _ in cols.values()}) if colfuse else {}
    sums = {**{sid: (p, w, _colsum_launch) for sid, (p, w) in cols.items()},
            **{sid: (p, w, _rowsum_launch) for sid, (p, w) in rows.items()}}
    producer_of = {p: (sid, w, f) for sid, (p, w, f) in sums.items()}
    mos = mo_fusions(graph, keep, exclude=set(sums) | set(producer_of) | folds | set(tprods) | tmats) if mofuse else {}
    readers = set(mos.values())
    launches = []
    for node in graph.nodes:
        if node.op in ("input", "const") or node.id in folds or node.id in readers or node.id in tmats:
            continue
        if node.id in tprods:             # a GEMM read only by a transpose: the transposed product
            launches.append(_transposed_product_launch(graph, node, graph.nodes[tprods[node.id]], matmul, folds))
            continue
        if node.id in mos:                # a producer computing its reader too
            launches.append(_mo_launch(graph, node, graph.nodes[mos[node.id]]))
            continue
        if node.id in producer_of:        # the producer of a fused column or row sum
            sid, write, make = producer_of[node.id]
            if write:
                launches.append(make(graph, node, graph.nodes[sid], True))
            continue
        if node.id in sums:               # the sum itself
            pid, write, make = sums[node.id]
            if not write:
                launches.append(make(graph, graph.nodes[pid], node, False))
            continue
        ops = _matmul_operands(graph, node) if folds else None
        if ops and set(ops) & folds:
            lau = _folded_launch(graph, node, matmul, sabotage, folds)
        elif node.op == "fused":
            lau = fused_kernel(node, matmul, sabotage)
        else:
            lau = _plain_launch(graph, node, matmul)
        lau.bytes = _bytes(graph, lau)
        launches.append(lau)
    return {"launches": launches, "folded": sorted(folds), "transposed": sorted(tprods.items())}
