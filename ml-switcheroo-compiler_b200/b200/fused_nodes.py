"""Execution of the node types the reference's fusion passes emit.

The reference describes fusion groups as graph nodes but evaluates none of them: no
eager backend registers a kernel for them. Their meaning is fixed by the pass that
builds each one, and that is what runs here, on the same elementwise / GEMM / conv
kernels as the unfused ops:

* ``FusedElementwise`` (``transforms/passes/operator_fusion.py:673-715``): the
  ``scalar_expr`` attribute is a C float expression over ``in0 .. inN`` written from the
  templates at ``operator_fusion.py:619-637`` (``+ - * /``, unary minus, ``fmaxf``,
  ``fminf``, ``expf``, ``logf``, ``sqrtf``, ``tanhf``, ``fabsf``, float literals). It is
  parsed into a DAG (identical subexpressions shared) and run as one register program
  over the broadcast of the inputs, evaluated in float like the C expression.
* ``<Elem><Act>`` (``operator_fusion.py:906-945``, attributes ``fused_ops`` = [elem,
  act]): act(elem(*inputs)). ``AddRelu`` from the YAML rule ``ElementwiseFusion`` is
  the same computation.
* ``Fused<Conv>Bias<Act>`` (``operator_fusion.py:851-890``, conv attributes +
  ``activation`` + ``has_bias``; YAML ``Conv2DBiasActivationFusion``, inputs x, w,
  bias): act(Conv2D(x, w) + bias).
* ``HorizontalFusedOps`` (``operator_fusion.py:992-1071``): a tuple of ``fused_ops``
  applied to the shared inputs (the siblings' attributes are not kept by the pass, so
  each op runs with its defaults), read back by ``TupleGetItem`` (attribute ``index``).
* declarative rules (``operator_fusion.py:391-482``, ``transforms/fusion_patterns.yaml``):
  the matched root node is cloned under the rule's ``fused_op`` name with the attribute
  ``fused_pattern``; only the root is matched (``targets[-1]``), so the node computes the
  root op on its own inputs and attributes.
* YAML rules (``transforms/passes/fusion_patterns/*.yaml``, ``operator_fusion.py:485-538``):
  ``FusedLogExp``, ``DotGelu``, ``DotRelu``, ``FusedMultiplyAdd``, ``Linear``,
  ``FusedLayerNorm``, ``FusedLayerNormAffine``: the pattern's computation on the
  replacement inputs.

Two YAML outputs cannot be executed because the rewrite drops an operand the pattern
needs: ``FastGelu`` (the constant c of x * sigmoid(c x) is not an input) and
``Conv2DBatchNorm`` (BatchNorm has no kernel in the reference's numpy backend); both
raise ``UnimplementedMathError``.
"""

from __future__ import annotations

import re
from typing import Any, Callable

import torch

from . import _lib as L
from .errors import UnimplementedMathError

# --------------------------------------------------------------------------------
# scalar_expr: tokenizer, parser (to a hash-consed DAG) and register-program emitter
# --------------------------------------------------------------------------------
_TOKEN = re.compile(r"\s*(?:(?P<num>(?:\d+\.\d*|\.\d+|\d+)(?:[eE][+-]?\d+)?)[fF]?|(?P<name>[A-Za-z_]\w*)|(?P<op>[-+*/(),]))")
_FUNCS = {"fmaxf": ("MAX", 2), "fminf": ("MIN", 2), "expf": ("EXP", 1), "logf": ("LOG", 1), "sqrtf": ("SQRT", 1),
          "tanhf": ("TANH", 1), "fabsf": ("ABS", 1)}
_BIN = {"+": "ADD", "-": "SUB", "*": "MUL", "/": "DIV"}


def _tokens(s: str) -> list[tuple[str, str]]:
    out, pos = [], 0
    s = s.strip()
    while pos < len(s):
        m = _TOKEN.match(s, pos)
        if not m or m.end() == pos:
            raise UnimplementedMathError(f"FusedElementwise: cannot parse scalar_expr near {s[pos:pos + 20]!r}")
        kind = m.lastgroup
        out.append((kind, m.group(kind)))
        pos = m.end()
    return out


class ExprDag:
    """Nodes are tuples: ("in", k), ("imm", float32 value), (opname, child ids...).
    Structurally identical subexpressions get one id (hash-consing)."""

    def __init__(self) -> None:
        self.nodes: list[tuple] = []
        self.index: dict[tuple, int] = {}

    def add(self, key: tuple) -> int:
        i = self.index.get(key)
        if i is None:
            i = len(self.nodes)
            self.nodes.append(key)
            self.index[key] = i
        return i


def parse_scalar_expr(expr: str, n_inputs: int) -> tuple[ExprDag, int]:
    """Parse the reference's C expression; returns (dag, root id)."""
    import numpy as np

    toks = _tokens(expr)
    dag = ExprDag()
    pos = 0

    def peek():
        return toks[pos] if pos < len(toks) else (None, None)

    def take(val=None):
        nonlocal pos
        t = peek()
        if t[0] is None or (val is not None and t[1] != val):
            raise UnimplementedMathError(f"FusedElementwise: expected {val!r} in scalar_expr {expr!r}")
        pos += 1
        return t

    def primary() -> int:
        kind, val = peek()
        if kind == "num":
            take()
            return dag.add(("imm", float(np.float32(float(val)))))
        if kind == "name":
            take()
            m = re.fullmatch(r"in_?(\d+)", val)
            if m:
                k = int(m.group(1))
                if k >= n_inputs:
                    raise UnimplementedMathError(f"FusedElementwise: {val} but the node has {n_inputs} inputs")
                return dag.add(("in", k))
            if val not in _FUNCS:
                raise UnimplementedMathError(f"FusedElementwise: function {val!r} in scalar_expr has no kernel")
            op, arity = _FUNCS[val]
            take("(")
            args = [expr_()]
            while peek()[1] == ",":
                take(",")
                args.append(expr_())
            take(")")
            if len(args) != arity:
                raise UnimplementedMathError(f"FusedElementwise: {val} takes {arity} arguments")
            return dag.add((op, *args))
        if val == "(":
            take("(")
            r = expr_()
            take(")")
            return r
        raise UnimplementedMathError(f"FusedElementwise: unexpected token {val!r} in {expr!r}")

    def unary() -> int:
        if peek()[1] == "-":
            take("-")
            return dag.add(("NEG", unary()))
        if peek()[1] == "+":
            take("+")
            return unary()
        return primary()

    def term() -> int:
        r = unary()
        while peek()[1] in ("*", "/"):
            op = _BIN[take()[1]]
            r = dag.add((op, r, unary()))
        return r

    def expr_() -> int:
        r = term()
        while peek()[1] in ("+", "-"):
            op = _BIN[take()[1]]
            r = dag.add((op, r, term()))
        return r

    root = expr_()
    if pos != len(toks):
        raise UnimplementedMathError(f"FusedElementwise: trailing tokens in scalar_expr {expr!r}")
    return dag, root


def _reachable(dag: ExprDag, root: int) -> list[int]:
    seen: set[int] = set()
    order: list[int] = []
    stack = [(root, False)]
    while stack:
        i, done = stack.pop()
        if done:
            order.append(i)
            continue
        if i in seen:
            continue
        seen.add(i)
        stack.append((i, True))
        key = dag.nodes[i]
        if key[0] not in ("in", "imm"):
            for c in reversed(key[1:]):
                if c not in seen:
                    stack.append((c, False))
    return order  # children before parents


def run_dag(dag: ExprDag, root: int, inputs: list[Any], shape: tuple) -> torch.Tensor:
    """Evaluate the DAG over ``shape`` (the broadcast of the inputs) as one register
    program when it fits the kernel's limits (inputs, registers, instructions), else one
    kernel per DAG node with fp32 temporaries. Output fp32."""
    from . import ops

    order = _reachable(dag, root)
    used_inputs = sorted({dag.nodes[i][1] for i in order if dag.nodes[i][0] == "in"})
    tens = [inputs[k] for k in used_inputs]
    if all(isinstance(t, torch.Tensor) for t in tens) and len(tens) <= L.EW_MAX_IN:
        prog = _emit(dag, root, order, used_inputs)
        if prog is not None:
            p = ops.Prog()
            p.inputs = [inputs[k] for k in used_inputs]
            p.ins, p.nreg = prog[0], prog[1]
            return p.run([(prog[2], torch.float32)], shape)[0]
    # one kernel per node
    vals: dict[int, Any] = {}
    for i in order:
        key = dag.nodes[i]
        if key[0] == "in":
            vals[i] = inputs[key[1]]
        elif key[0] == "imm":
            vals[i] = key[1]
        elif len(key) == 2:
            vals[i] = ops.ew_unary(key[0], vals[key[1]], out_dtype=torch.float32)
        else:
            vals[i] = ops.ew_binary(key[0], vals[key[1]], vals[key[2]], out_dtype=torch.float32)
    r = vals[root]
    if not isinstance(r, torch.Tensor) or tuple(r.shape) != tuple(shape):
        p = ops.Prog()
        rr = p.value(r)
        r = p.run([(rr, torch.float32)], shape)[0]
    return r


def _emit(dag: ExprDag, root: int, order: list[int], used_inputs: list[int]):
    """Instructions with register reuse (a register is freed after its last use);
    returns (instructions, registers used, result register) or None if over the limits."""
    last_use: dict[int, int] = {}
    for pos, i in enumerate(order):
        key = dag.nodes[i]
        if key[0] not in ("in", "imm"):
            for c in key[1:]:
                last_use[c] = pos
    last_use[root] = len(order)
    slot = {k: j for j, k in enumerate(used_inputs)}
    free: list[int] = []
    nreg = 0
    reg: dict[int, int] = {}
    ins = []
    for pos, i in enumerate(order):
        key = dag.nodes[i]
        kids = [] if key[0] in ("in", "imm") else list(key[1:])
        # free children whose last use is this instruction before allocating the result
        # (the kernel reads all operands before writing dst)
        for c in set(kids):
            if last_use.get(c) == pos:
                free.append(reg[c])
        if free:
            r = free.pop()
        else:
            r = nreg
            nreg += 1
            if nreg > L.EW_MAX_REG:
                return None
        reg[i] = r
        if key[0] == "in":
            ins.append((L.EW["LOAD"], r, slot[key[1]], 0, 0, 0.0))
        elif key[0] == "imm":
            ins.append((L.EW["IMM"], r, 0, 0, 0, key[1]))
        else:
            a = reg[kids[0]]
            b = reg[kids[1]] if len(kids) > 1 else 0
            ins.append((L.EW[key[0]], r, a, b, 0, 0.0))
    if len(ins) + 1 > L.EW_MAX_INS:
        return None
    return ins, nreg, reg[root]


def _bshape(xs: list[Any]) -> tuple:
    shapes = [tuple(x.shape) for x in xs if isinstance(x, torch.Tensor)]
    return tuple(torch.broadcast_shapes(*shapes)) if shapes else ()


def op_fused_elementwise(*inputs, scalar_expr: str = "0.0f", fused_ops=None, **_):
    """FusedElementwise (operator_fusion.py:673-715): the scalar_expr over the inputs."""
    dag, root = parse_scalar_expr(str(scalar_expr), len(inputs))
    return run_dag(dag, root, list(inputs), _bshape(list(inputs)))


# --------------------------------------------------------------------------------
# op-chain nodes
# --------------------------------------------------------------------------------
# ELEMENTWISE_OPS of operator_fusion.py:596-615 and the activations of :918
ELEMENTWISE_OPS = ("Add", "Sub", "Mul", "Div", "TrueDivide", "Relu", "Sigmoid", "Neg", "Abs", "Exp", "Log", "Sqrt", "Gelu",
                   "Silu", "Tanh", "Pow", "Maximum", "Minimum")
ACTIVATIONS = ("Relu", "Gelu", "Silu", "Sigmoid", "Tanh")


def _op(name: str) -> Callable:
    from . import ops

    if name == "Silu":
        return lambda x, **_: ops.op_multiply(x, ops.op_sigmoid(x))
    fn = ops.OPS.get(ops.ALIASES.get(name, name))
    if fn is None:
        raise UnimplementedMathError(f"Operation {name} is not implemented in the b200 backend.")
    return fn


def _elem_act(elem: str, act: str) -> Callable:
    def run(*inputs, fused_ops=None, activation=None, **kw):
        ops_ = list(fused_ops) if fused_ops else [elem, act]
        if len(ops_) != 2:
            raise UnimplementedMathError(f"{elem}{act} with fused_ops {ops_!r}")
        return _op(ops_[1])(_op(ops_[0])(*inputs))

    return run


def _conv_bias_act(conv: str, act: str) -> Callable:
    def run(*inputs, activation=None, has_bias=True, fused_pattern=None, **kw):
        from . import ops

        if fused_pattern is not None:  # declarative rule: the root (the activation) alone
            return _op(act)(*inputs)
        if len(inputs) != 3:
            raise UnimplementedMathError(f"Fused{conv}Bias{act} expects x, w, bias")
        x, w, b = inputs
        conv_kw = {k: v for k, v in kw.items() if k in ("stride", "strides", "padding", "groups", "dilation")}
        if "strides" in conv_kw and "stride" not in conv_kw:
            conv_kw["stride"] = conv_kw.pop("strides")
        conv_kw.pop("strides", None)
        y = ops.op_conv2d(x, w, **conv_kw)
        return _op(activation or act)(ops.op_add(y, b))

    return run


def op_horizontal_fused(*inputs, fused_ops=(), sibling_ids=(), **_):
    """HorizontalFusedOps (operator_fusion.py:992-1071): each sibling op on the shared inputs."""
    return tuple(_op(name)(*inputs) for name in fused_ops)


def op_tuple_get_item(t, index=0, **_):
    """TupleGetItem: element ``index`` of a HorizontalFusedOps result."""
    if not isinstance(t, (tuple, list)):
        raise UnimplementedMathError("TupleGetItem on a value that is not a tuple")
    return t[int(index)]


# declarative rules of transforms/fusion_patterns.yaml: fused_op name -> {rule name: root op}
DECLARATIVE_ROOTS = {
    "ScaledDotProductAttention": "Matmul",
    "ConvBNActivation": "Relu",
    "LayerNorm": "Add",
    "MatMulBiasGelu": "Gelu",
    "Conv2DBatchNormFusion": "BatchNorm",
    "Conv2DBiasActivationFusion": "Relu",
    "DotGeluFusion": "Gelu",
    "DotReluFusion": "Relu",
    "FMAFusion": "Add",
    "MultiHeadAttentionFusion": "Matmul",
}


def _declarative(default_root: str | None) -> Callable:
    def run(*inputs, fused_pattern=None, **kw):
        root = DECLARATIVE_ROOTS.get(str(fused_pattern)) if fused_pattern is not None else None
        if root is None:
            root = default_root
        if root is None:
            raise UnimplementedMathError(f"declarative fused node of rule {fused_pattern!r} has no known root op")
        return _op(root)(*inputs, **kw)

    return run


def op_fused_layer_norm(x, eps, scale=None, shift=None, **_):
    """FusedLayerNorm(x, eps) / FusedLayerNormAffine(x, scale, shift, eps)
    (fusion_patterns/LayerNormFusion.yaml): (x - mean) / sqrt(var + eps) [* scale + shift]
    over the last axis, the ReduceMean axes of the matched pattern."""
    from . import ops

    e = float(eps.item()) if isinstance(eps, torch.Tensor) else float(eps)
    return ops.op_layer_norm(x, scale, shift, eps=e, axis=-1)


def op_fused_layer_norm_affine(x, scale, shift, eps, **kw):
    return op_fused_layer_norm(x, eps, scale=scale, shift=shift)


def _unexecutable(name: str, why: str) -> Callable:
    def run(*_, **__):
        raise UnimplementedMathError(f"{name}: {why}")

    return run


def register(table: dict[str, Callable]) -> None:
    """Add every fusion node type above to the op table."""
    from . import ops

    table["FusedElementwise"] = op_fused_elementwise
    for e in ELEMENTWISE_OPS:
        for a in ACTIVATIONS:
            table.setdefault(f"{e}{a}", _elem_act(e, a))
    for conv in ("Conv2D", "Conv"):
        for a in ACTIVATIONS:
            table[f"Fused{conv}Bias{a}"] = _conv_bias_act("Conv2D", a)
    table["HorizontalFusedOps"] = op_horizontal_fused
    table["TupleGetItem"] = op_tuple_get_item
    # declarative fused_op names without a YAML rule of the same name
    for name, root in (("FusedAttention", "Matmul"), ("FusedConv2D", "Relu"), ("FusedLinearGELU", "Gelu"),
                       ("FusedConv2DBatchNorm", "BatchNorm"), ("FusedLinearGelu", "Gelu"), ("FusedLinearRelu", "Relu"),
                       ("ScaledDotProductAttention", "Matmul")):
        table[name] = _declarative(root)
    # FusedLayerNorm / FusedMultiplyAdd: YAML rule (several inputs) or declarative (root only)
    yaml_ln, yaml_fma = op_fused_layer_norm, (lambda a, b, c, **_: ops.op_add(ops.op_multiply(a, b), c))

    def fused_layer_norm(*inputs, fused_pattern=None, **kw):
        return _declarative("Add")(*inputs, fused_pattern=fused_pattern, **kw) if fused_pattern else yaml_ln(*inputs, **kw)

    def fused_multiply_add(*inputs, fused_pattern=None, **kw):
        return _declarative("Add")(*inputs, fused_pattern=fused_pattern, **kw) if fused_pattern else yaml_fma(*inputs, **kw)

    table["FusedLayerNorm"] = fused_layer_norm
    table["FusedMultiplyAdd"] = fused_multiply_add
    table["FusedLayerNormAffine"] = op_fused_layer_norm_affine
    table["FusedLogExp"] = lambda x, **_: ops.op_exp(ops.op_log(x))
    table["DotGelu"] = lambda a, b, **_: ops.op_gelu(ops.op_matmul(a, b))
    table["DotRelu"] = lambda a, b, **_: ops.op_relu(ops.op_matmul(a, b))
    table["Linear"] = lambda x, w, b, **_: ops.op_add(ops.op_matmul(x, w), b)
    table["Dot"] = lambda a, b, **_: ops.op_matmul(a, b)
    table["FastGelu"] = _unexecutable("FastGelu", "the rewrite keeps only x, not the constant c of x * sigmoid(c x)")
    table["Conv2DBatchNorm"] = _unexecutable("Conv2DBatchNorm", "BatchNorm has no kernel in the reference's numpy backend")
