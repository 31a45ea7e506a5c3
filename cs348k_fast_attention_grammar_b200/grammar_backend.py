"""B200 backend for the reference's kernel grammar.

The reference lowers a grammar ``Program`` to cuTile source with per-op rule
tables (``EMIT_RULES`` / ``REDUCE_RULES``, ``grammar/kernel_ast.py:178-223``)
and ``emit_module`` (``:1221-1287``), and its search times the emitted module
through ``fn(*inputs)`` + ``KERNEL_META`` (``grammar/optimization.py:156-303``).
This module is the same hook for the B200 kernels: ``emit_module(program)``
returns importable module source with the same ``fn`` / ``KERNEL_META``
contract, and ``lower(program)`` returns the module object directly, so the
search (or any caller) can put the hand-written sm_100a kernels among its
candidates.

How a program is lowered.  Tiling, stage boundaries, fusion, hoisting and
reduction loops change how the reference's kernels are scheduled but not what
they compute, so the backend first rebuilds, for the program's output, the
whole-tensor expression over its input tensors (intermediates substituted by
the expressions that store them; a ``ReductionLoop`` stands for its partials
over the full axis).  Every rewrite of the reference's search therefore maps to
the same expression.  ``LOWER_RULES`` then maps expression patterns to kernels:

=============  ==============================================  =================
kind           expression (c, eps: constants of the program)   kernel
=============  ==============================================  =================
attention      (e / rowsum(e)) @ V, e = exp(s - rowmax(s)),    ``fa_attn_fwd_f32``
               s = c * (Q @ KT)  (also e @ V / rowsum(e))      / ``fa_attn_fwd``
mlp_ln         LN(relu(X @ W1) @ W2 + X), LN as in             ``fa_mlp_ln_fwd``
               run_mlp_search.py:76-93
mlp            act(X @ W1) @ W2, act = relu or none            ``fa_mlp_fwd``
gemm_act       act(A @ B), act = relu or none                  ``fa_gemm_act``
layer_norm     LN(X)                                           ``fa_layernorm_rows``
=============  ==============================================  =================

A program that matches no rule (or whose shapes the kernels do not take)
raises ``UnsupportedProgram``, the way the reference's renderer rejects
unknown ops; a search maps that to ``inf`` like any other emit failure.

Numerics: operands are rounded to bf16 for the tensor cores and accumulated in
fp32 (fp32 arrays in, fp32 arrays out), as ``kernel_module.fn`` does.
"""

from __future__ import annotations

import math

from . import grammar_ir as ir

POINTWISE = {"add", "mul", "sub", "div", "relu", "exp", "sqrt", "mulc", "addc"}
ROW_REDUCE = {"rowmax", "rowsum"}


class UnsupportedProgram(ValueError):
    """The program computes something no B200 kernel implements."""


# ---------------------------------------------------------------------------
# Program structure
# ---------------------------------------------------------------------------
def _iter_stmts(stmts):
    for s in stmts:
        yield s
        if ir.kind(s) == "ReductionLoop":
            yield from _iter_stmts(s.body)


def program_io(program) -> tuple[list, list, list]:
    """(inputs, intermediates, outputs), each sorted by name: inputs are read
    and never written, outputs written and never read (the reference's
    classification, ``kernel_ast.py:665-675``, which fixes ``fn``'s argument
    order)."""
    written, read = set(), set()
    for loop in program.body:
        written.add(loop.out)
        for s in _iter_stmts(loop.body):
            if ir.kind(s) == "Load":
                read.add(s.source)
    return sorted(read - written), sorted(written & read), sorted(written - read)


def _loads_feeding(v):
    k = ir.kind(v)
    if k == "Load":
        yield v
    elif k == "Compute":
        for i in v.inputs:
            yield from _loads_feeding(i)
    elif k == "ReductionLoop":
        for p in v.partials:
            yield from _loads_feeding(p)


def _axes(v) -> list:
    """Logical axes a value spans: a Load's index; matmul drops the shared
    axis; row reductions keep their input's axes (the reduced one becomes
    size 1); elementwise ops take their broadest operand's axes."""
    k = ir.kind(v)
    if k == "Load":
        return list(v.index)
    if k == "ReductionLoop":
        return _axes(v.partial)
    if k == "Compute":
        ins = [_axes(i) for i in v.inputs]
        if v.op == "matmul":
            a0, a1 = ins
            shared = set(a0) & set(a1)
            return [x for x in a0 if x not in shared] + [x for x in a1 if x not in shared]
        if v.op in ROW_REDUCE:
            return list(ins[0])
        return max(ins, key=len)
    raise UnsupportedProgram(f"no axes for {k}")


def _extent(v, axis: str, tensors: dict) -> int:
    for ld in _loads_feeding(v):
        if axis in ld.index:
            return int(tensors[ld.source][list(ld.index).index(axis)])
    raise UnsupportedProgram(f"axis {axis!r} not found in the loads feeding a value")


def program_flops(program) -> tuple[int, bool]:
    """Logical FLOPs of a program, the reference's convention
    (``kernel_ast.py:1110-1147``): matmul 2*M*N*K with the global contraction
    extent, a row reduction one op per input element, a pointwise op one op per
    element of its stage's output tensor; ``exact`` is False if an op has no
    rule."""
    total, exact = 0, True
    for loop in program.body:
        gout = math.prod(program.tensors[loop.out])
        for s in _iter_stmts(loop.body):
            if ir.kind(s) != "Compute":
                continue
            if s.op == "matmul":
                a, b = s.inputs
                shared = [x for x in _axes(a) if x in set(_axes(b))]
                k = _extent(a, shared[0], program.tensors) if shared else 1
                total += 2 * gout * k
            elif s.op in ROW_REDUCE:
                axes = _axes(s)
                rows = 1
                for x in axes:
                    if x != s.axis:
                        rows *= _extent(s, x, program.tensors)
                total += rows * _extent(s, s.axis, program.tensors)
            elif s.op in POINTWISE:
                total += gout
            else:
                exact = False
    return total, exact


# ---------------------------------------------------------------------------
# Whole-tensor expressions
# ---------------------------------------------------------------------------
# An expression is a nested tuple: ("in", name) for an input tensor, or
# (op, const, args...) for a Compute (const is None unless op is mulc/addc).
def output_expression(program):
    """The expression of the program's single output over its inputs."""
    inputs, _inter, outputs = program_io(program)
    if len(outputs) != 1:
        raise UnsupportedProgram(f"expected one output tensor, got {outputs}")
    stored: dict = {}
    memo: dict = {}

    def ex(v):
        key = id(v)
        if key in memo:
            return memo[key]
        k = ir.kind(v)
        if k == "Load":
            if v.source in stored:
                r = stored[v.source]
            elif v.source in inputs:
                r = ("in", v.source)
            else:
                raise UnsupportedProgram(f"{v.source!r} is read before it is written")
        elif k == "ReductionLoop":
            r = ex(v.partial)
        elif k == "Compute":
            if v.op not in POINTWISE | ROW_REDUCE | {"matmul"}:
                raise UnsupportedProgram(f"op {v.op!r} has no B200 rule")
            if v.op in ROW_REDUCE:
                ax = _axes(v.inputs[0])
                if not ax or ax[-1] != v.axis:
                    raise UnsupportedProgram("row reductions must reduce the last axis")
            const = float(v.const) if v.op in ("mulc", "addc") else None
            r = (v.op, const) + tuple(ex(i) for i in v.inputs)
        else:
            raise UnsupportedProgram(f"value of type {k}")
        memo[key] = r
        return r

    for loop in program.body:
        for s in _iter_stmts(loop.body):
            if ir.kind(s) == "Store":
                stored[s.dest] = ex(s.src)
    if outputs[0] not in stored:
        raise UnsupportedProgram("the output tensor is never stored")
    return stored[outputs[0]]


def _is_in(e) -> bool:
    return isinstance(e, tuple) and e[0] == "in"


def _op(e, name: str):
    return isinstance(e, tuple) and e[0] == name


def _split_scale(e):
    """(c, x) for e = mulc(x, c); (1.0, e) otherwise."""
    if _op(e, "mulc"):
        return e[1], e[2]
    return 1.0, e


def _match_scores(s):
    """s = c * (Q @ KT) in any of the places the scale can sit -> (Q, KT, c)."""
    c, inner = _split_scale(s)
    if not _op(inner, "matmul"):
        return None
    a, b = inner[2], inner[3]
    ca, a = _split_scale(a)
    cb, b = _split_scale(b)
    if not (_is_in(a) and _is_in(b)):
        return None
    return a[1], b[1], c * ca * cb


def _match_softmax_numerator(e):
    """e = exp(s - rowmax(s)) -> s."""
    if not _op(e, "exp") or not _op(e[2], "sub"):
        return None
    s, m = e[2][2], e[2][3]
    if _op(m, "rowmax") and m[2] == s:
        return s
    return None


def match_attention(expr):
    # (e / rowsum(e)) @ V
    if _op(expr, "matmul") and _op(expr[2], "div") and _is_in(expr[3]):
        num, den = expr[2][2], expr[2][3]
        v = expr[3][1]
    # (e @ V) / rowsum(e)
    elif _op(expr, "div") and _op(expr[2], "matmul") and _is_in(expr[2][3]):
        num, den = expr[2][2], expr[3]
        v = expr[2][3][1]
    else:
        return None
    if not (_op(den, "rowsum") and den[2] == num):
        return None
    s = _match_softmax_numerator(num)
    if s is None:
        return None
    sc = _match_scores(s)
    if sc is None:
        return None
    q, kt, c = sc
    return {"q": q, "kt": kt, "v": v}, {"scale": c}


def match_layer_norm(expr):
    """(r - mean) / sqrt(mean(r*r) - mean^2 + eps), mean = rowsum(r) * (1/D)
    (run_mlp_search.py:76-93) -> (r, eps, 1/D)."""
    if not (_op(expr, "div") and _op(expr[2], "sub") and _op(expr[3], "sqrt")):
        return None
    r, mean = expr[2][2], expr[2][3]
    if not (_op(mean, "mulc") and _op(mean[2], "rowsum") and mean[2][2] == r):
        return None
    inv_d = mean[1]
    ve = expr[3][2]
    if not _op(ve, "addc"):
        return None
    eps, var = ve[1], ve[2]
    if not _op(var, "sub"):
        return None
    msq, m2 = var[2], var[3]
    if not (_op(m2, "mul") and m2[2] == mean and m2[3] == mean):
        return None
    if not (_op(msq, "mulc") and abs(msq[1] - inv_d) <= 1e-12 * abs(inv_d) and
            _op(msq[2], "rowsum") and _op(msq[2][2], "mul") and
            msq[2][2][2] == r and msq[2][2][3] == r):
        return None
    return r, eps, inv_d


def _match_act_matmul(e):
    """act(A @ B) with act in relu/none -> (A, B, act) over inputs."""
    act = "none"
    if _op(e, "relu"):
        act, e = "relu", e[2]
    if _op(e, "matmul") and _is_in(e[2]) and _is_in(e[3]):
        return e[2][1], e[3][1], act
    return None


def _match_mlp(e):
    """act(X @ W1) @ W2 -> roles, act."""
    if not _op(e, "matmul") or not _is_in(e[3]):
        return None
    inner = _match_act_matmul(e[2])
    if inner is None:
        return None
    x, w1, act = inner
    return {"x": x, "w1": w1, "w2": e[3][1]}, act


def match_program(program):
    """(kind, roles, params) for the first LOWER_RULES entry the program's
    output expression matches; raises UnsupportedProgram otherwise."""
    expr = output_expression(program)
    m = match_attention(expr)
    if m is not None:
        return "attention", m[0], m[1]
    ln = match_layer_norm(expr)
    if ln is not None:
        r, eps, inv_d = ln
        if _is_in(r):
            return "layer_norm", {"x": r[1]}, {"eps": eps, "inv_d": inv_d}
        if _op(r, "add"):
            for y, xres in ((r[2], r[3]), (r[3], r[2])):
                mm = _match_mlp(y)
                if mm is not None and mm[1] == "relu" and _is_in(xres) and \
                        xres[1] == mm[0]["x"]:
                    return "mlp_ln", mm[0], {"eps": eps, "inv_d": inv_d}
        raise UnsupportedProgram("LayerNorm of an expression no kernel computes")
    mm = _match_mlp(expr)
    if mm is not None:
        return "mlp", mm[0], {"act": mm[1]}
    g = _match_act_matmul(expr)
    if g is not None:
        return "gemm_act", {"a": g[0], "b": g[1]}, {"act": g[2]}
    raise UnsupportedProgram("the program matches no B200 kernel")


# ---------------------------------------------------------------------------
# Implementations (one per kind): positional args in fn's order -> output
# ---------------------------------------------------------------------------
def _to_torch(x):
    import torch
    return x if isinstance(x, torch.Tensor) else torch.from_dlpack(x)


def _like(result, template):
    """Return ``result`` (a torch tensor) as the array type of ``template``."""
    import torch
    if isinstance(template, torch.Tensor):
        return result
    try:
        import cupy
    except ImportError:
        return result
    return cupy.from_dlpack(result)


def _check_shapes(kind: str, roles: dict, tensors: dict, params: dict) -> None:
    shp = {r: tuple(tensors[n]) for r, n in roles.items()}
    if kind == "attention":
        (n, d), (d2, n2), (n3, d3) = shp["q"], shp["kt"], shp["v"]
        if not (d == d2 and n == n2 == n3 and d == d3):
            raise UnsupportedProgram(f"attention shapes {shp} are not Q[N,d] KT[d,N] V[N,d]")
        if not (8 <= d <= 128 and d % 8 == 0):
            raise UnsupportedProgram(f"head dim {d} (the kernels take 8 .. 128, multiples of 8)")
    elif kind in ("mlp", "mlp_ln"):
        (m, k), (k2, n), (n2, k3) = shp["x"], shp["w1"], shp["w2"]
        if not (k == k2 == k3 and n == n2) or k % 64 or n % 64:
            raise UnsupportedProgram(f"MLP shapes {shp}: need X[M,K] W1[K,N] W2[N,K], "
                                     "K and N multiples of 64")
        if kind == "mlp_ln" and (k > 8192 or abs(params["inv_d"] * k - 1.0) > 1e-6):
            raise UnsupportedProgram("LayerNorm width must be the feature dim, <= 8192")
    elif kind == "gemm_act":
        (m, k), (k2, n) = shp["a"], shp["b"]
        if k != k2 or k % 64 or n % 64:
            raise UnsupportedProgram(f"GEMM shapes {shp}: K and N multiples of 64")
    elif kind == "layer_norm":
        m, n = shp["x"]
        if n % 8 or n > 8192 or abs(params["inv_d"] * n - 1.0) > 1e-6:
            raise UnsupportedProgram(f"LayerNorm width {n}: a multiple of 8, <= 8192")


def build_impl(kind: str, roles: dict, params: dict, arg_names: list):
    """The callable behind an emitted module's ``fn``: maps positional inputs
    (in ``arg_names`` order) to the kernel's operands."""
    import torch
    from . import operators as ops

    pos = {name: i for i, name in enumerate(arg_names)}

    def pick(args, role):
        return _to_torch(args[pos[roles[role]]])

    def bf16(t):
        return t.to(torch.bfloat16).contiguous()

    def impl(*args):
        if len(args) != len(arg_names):
            raise TypeError(f"fn takes {len(arg_names)} arrays ({', '.join(arg_names)})")
        if kind == "attention":
            q, kt, v = pick(args, "q"), pick(args, "kt"), pick(args, "v")
            if q.dtype == torch.float32:
                out = ops.attention_f32(q.contiguous(), kt.contiguous(), v.contiguous(),
                                        scale=params["scale"], k_transposed=True)
            else:
                o = ops.attention(bf16(q)[None, None], bf16(kt.t())[None, None],
                                  bf16(v)[None, None], scale=params["scale"])
                out = o[0, 0].to(q.dtype)
        elif kind in ("mlp", "mlp_ln"):
            x, w1, w2 = pick(args, "x"), pick(args, "w1"), pick(args, "w2")
            if kind == "mlp":
                y = ops.mlp(bf16(x), bf16(w1), bf16(w2), act=params["act"])
            else:
                y = ops.mlp_ln(bf16(x), bf16(w1), bf16(w2), eps=params["eps"])
            out = y.to(x.dtype)
        elif kind == "gemm_act":
            a, b = pick(args, "a"), pick(args, "b")
            out = ops.gemm_act(bf16(a), bf16(b), act=params["act"]).to(a.dtype)
        elif kind == "layer_norm":
            x = pick(args, "x")
            out = ops.layer_norm_rows(bf16(x), eps=params["eps"]).to(x.dtype)
        else:
            raise UnsupportedProgram(f"unknown kind {kind!r}")
        return _like(out, args[0])

    return impl


# kind -> (shape check, kernel entry point it lowers to): the rule table a
# search consults, in the role of EMIT_RULES / REDUCE_RULES for cuTile.
LOWER_RULES = {
    "attention": "fa_attn_fwd_f32 (fp32 arrays) / fa_attn_fwd (bf16)",
    "mlp_ln": "fa_mlp_ln_fwd",
    "mlp": "fa_mlp_fwd",
    "gemm_act": "fa_gemm_act",
    "layer_norm": "fa_layernorm_rows",
}


# ---------------------------------------------------------------------------
# The hook: lower / emit_module
# ---------------------------------------------------------------------------
class LoweredModule:
    """What ``emit_module``'s source defines, as an object: ``fn``,
    ``KERNEL_META``, plus the matched ``kind`` / ``roles`` / ``params``."""

    def __init__(self, kind, roles, params, meta, arg_names, fn_name="fn"):
        self.kind, self.roles, self.params = kind, roles, params
        self.KERNEL_META = meta
        self.arg_names = arg_names
        impl = build_impl(kind, roles, params, arg_names)
        setattr(self, fn_name, impl)
        if fn_name != "fn":
            self.fn = impl


def _analyse(program):
    kind, roles, params = match_program(program)
    inputs, _inter, outputs = program_io(program)
    _check_shapes(kind, roles, program.tensors, params)
    flops, exact = program_flops(program)
    meta = {"inputs": [[t, list(program.tensors[t])] for t in inputs],
            "output": [outputs[0], list(program.tensors[outputs[0]])],
            "flops": flops, "flops_exact": exact}
    return kind, roles, params, meta, inputs


def lower(program, fn_name: str = "fn") -> LoweredModule:
    """Lower a grammar program to the B200 kernels (raises UnsupportedProgram)."""
    kind, roles, params, meta, inputs = _analyse(program)
    return LoweredModule(kind, roles, params, meta, inputs, fn_name)


def emit_module(program, fn_name: str = "fn") -> str:
    """Importable module source with ``fn(*inputs)`` (sorted input names, the
    reference's order) and ``KERNEL_META``, calling the B200 kernels -- a
    drop-in for the reference's ``emit_module`` in its search's evaluator."""
    kind, roles, params, meta, inputs = _analyse(program)
    sig = ", ".join(inputs)
    lines = [
        '"""Grammar program lowered to the B200 kernels (' + LOWER_RULES[kind] + ')."""',
        "from cs348k_fast_attention_grammar_b200.grammar_backend import build_impl as _build",
        "",
        f"_IMPL = _build({kind!r}, {roles!r}, {params!r}, {inputs!r})",
        "",
        "",
        f"def {fn_name}({sig}):",
        f"    return _IMPL({sig})",
        "",
        "",
        f"KERNEL_META = {meta!r}",
        "",
    ]
    return "\n".join(lines)
