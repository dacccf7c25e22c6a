"""Fusion planner: turns the live nodes of a graph into fused GPU steps.

Planning uses the exact shape and dtype of every value, recorded from one unfused
execution of the graph on the same input signature (``record_meta``). Then:

1. pattern fusions: subgraphs matched structurally (op types, edges, attributes,
   constants; Add/Multiply commutative) are replaced by one hand-written kernel each
   (``PATTERNS``). A match is accepted only if every replaced node is live, no replaced
   intermediate is needed outside the match, and the fused kernel's shape rules hold.
2. elementwise clustering (subsystem 1): maximal convex groups of elementwise nodes over
   one index space become one elementwise program (one HBM read per input, one write per
   live output), the b200 counterpart of the FusedElementwise groups of
   ``transforms/passes/operator_fusion.py:673-715``.
3. everything else is one per-op step.

Steps are then ordered by a topological sort of the condensed step graph.
"""

from __future__ import annotations

import math
from typing import Any, Callable

import torch

from . import _lib as L
from . import ops
from .executor import ALIASES, Step, node_kwargs, node_step
from .graph import Graph, Node


# ----------------------------------------------------------------------------------
# value metadata from one unfused run
# ----------------------------------------------------------------------------------
class Meta:
    __slots__ = ("shape", "dtype", "scalar")

    def __init__(self, v: Any) -> None:
        if isinstance(v, torch.Tensor):
            self.shape, self.dtype, self.scalar = tuple(v.shape), v.dtype, False
        else:
            self.shape, self.dtype, self.scalar = (), None, True


def record_meta(graph: Graph, nodes: list[Node], sample: dict[str, Any]) -> dict[str, Meta]:
    env: dict[str, Any] = dict(graph.initializers)
    env.update(sample)
    meta = {k: Meta(v) for k, v in env.items()}
    consumers: dict[str, int] = {}
    for n in nodes:
        for i in n.inputs:
            consumers[i] = consumers.get(i, 0) + 1
    for n in nodes:
        node_step(n).fn(env)
        meta[n.id] = Meta(env[n.id])
        for i in n.inputs:
            consumers[i] -= 1
            if consumers[i] == 0 and i not in sample and i not in graph.outputs:
                env.pop(i, None)
    torch.cuda.synchronize()
    return meta


# ----------------------------------------------------------------------------------
# structural pattern matcher
# ----------------------------------------------------------------------------------
COMMUTATIVE = {"Add", "Multiply"}


class Pat:
    """Base of pattern terms."""


class Var(Pat):
    def __init__(self, name: str) -> None:
        self.name = name


class Const(Pat):
    def __init__(self, value: float, rtol: float = 1e-6) -> None:
        self.value, self.rtol = value, rtol


class Op(Pat):
    def __init__(self, op: str, *args: Pat, name: str | None = None, attrs: dict | None = None) -> None:
        self.op, self.args, self.name, self.attrs = op, args, name, attrs or {}


def _op_name(n: Node) -> str:
    return ALIASES.get(n.op_type, n.op_type)


def match(p: Pat, nid: str, g: Graph, bind: dict[str, str], covered: set[str]) -> bool:
    """Match pattern ``p`` rooted at node ``nid``; extends ``bind`` and ``covered`` on success."""
    if isinstance(p, Var):
        if p.name in bind:
            return bind[p.name] == nid
        bind[p.name] = nid
        return True
    node = g.nodes.get(nid)
    if node is None:
        return False
    if isinstance(p, Const):
        if node.op_type != "Constant":
            return False
        v = node.attributes.get("value")
        if not isinstance(v, (int, float)):
            return False
        if abs(float(v) - p.value) > p.rtol * max(1.0, abs(p.value)):
            return False
        covered.add(nid)
        return True
    assert isinstance(p, Op)
    if _op_name(node) != p.op or len(node.inputs) != len(p.args):
        return False
    for k, want in p.attrs.items():
        have = node.attributes.get(k)
        if callable(want):
            if not want(have):
                return False
        elif have != want:
            return False
    if p.name is not None:
        if p.name in bind and bind[p.name] != nid:
            return False
    orders = [list(range(len(p.args)))]
    if p.op in COMMUTATIVE and len(p.args) == 2:
        orders.append([1, 0])
    for order in orders:
        b2, c2 = dict(bind), set(covered)
        if all(match(p.args[j], node.inputs[i], g, b2, c2) for i, j in enumerate(order)):
            if p.name is not None:
                b2[p.name] = nid
            c2.add(nid)
            bind.clear()
            bind.update(b2)
            covered.clear()
            covered.update(c2)
            return True
    return False


def _last_axis(ax: Any) -> bool:
    return ax == -1 or ax is None


def gelu_tanh_deriv(p: Pat) -> Pat:
    """d/dp of 0.5 p (1 + tanh(k (p + c p^3))) as the corrected Gelu VJP rule emits it:
    0.5 (1 + t) + 0.5 p (1 - t^2) k (1 + 3 c p^2)."""
    k = math.sqrt(2.0 / math.pi)
    c = 0.044715
    p2 = Op("Multiply", p, p, name="_gd_p2")
    p3 = Op("Multiply", p2, p)
    t = Op("Tanh", Op("Multiply", Op("Add", p, Op("Multiply", p3, Const(c))), Const(k)), name="_gd_t")
    left = Op("Multiply", Op("Add", t, Const(1.0)), Const(0.5))
    sech2 = Op("Subtract", Const(1.0), Op("Multiply", t, t))
    dinner = Op("Multiply", Op("Add", Op("Multiply", p2, Const(3.0 * c)), Const(1.0)), Const(k))
    right = Op("Multiply", Op("Multiply", Op("Multiply", p, sech2), dinner), Const(0.5))
    return Op("Add", left, right)


# ----------------------------------------------------------------------------------
# pattern: fused row chain  affine -> gelu -> LayerNorm -> softmax (+argmax) and its VJP
# ----------------------------------------------------------------------------------
def _rowfused_pattern():
    x, a, b, gamma, beta, cot = (Var(n) for n in ("x", "a", "b", "gamma", "beta", "cot"))
    p = Op("Add", Op("Multiply", x, a), b, name="p")
    g = Op("Gelu", p, name="g")
    n = Op("LayerNorm", g, gamma, beta, name="n")
    y = Op("Softmax", n, name="y", attrs={"axis": _last_axis})
    s = Op("ReduceSum", Op("Multiply", cot, y), attrs={"axis": _last_axis, "keepdims": True})
    dn = Op("Multiply", y, Op("Subtract", cot, s), name="dn")
    dg = Op("LayerNormInputGrad", dn, g, gamma, name="dg")
    dp = Op("Multiply", dg, gelu_tanh_deriv(p), name="dp")
    roots = {
        "dx": Op("Multiply", dp, a, name="dx"),
        "da": Op("BroadcastReduce", Op("Multiply", dp, x), a, name="da"),
        "db": Op("BroadcastReduce", dp, b, name="db"),
    }
    optional = {
        "am": Op("Argmax", y, name="am", attrs={"axis": _last_axis}),
        "dgamma": Op("LayerNormGammaGrad", dn, g, name="dgamma"),
        "dbeta": Op("LayerNormBetaGrad", dn, name="dbeta"),
    }
    return roots, optional


class Match:
    def __init__(self, kind: str, bind: dict[str, str], covered: set[str], outputs: dict[str, str]) -> None:
        self.kind, self.bind, self.covered, self.outputs = kind, bind, covered, outputs


def find_rowfused(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]]) -> list[Match]:
    roots, optional = _rowfused_pattern()
    found = []
    for nid, node in live.items():
        if _op_name(node) != "Multiply":
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if not match(roots["dx"], nid, g, bind, cov):
            continue
        ok = True
        outs = {"dx": bind["dx"]}
        for key in ("da", "db"):
            cand = [u for u in users.get(bind["dp"], []) if u in live] + [
                u for v in users.get(bind["dp"], []) for u in users.get(v, []) if u in live
            ]
            hit = False
            for c in cand:
                b2, c2 = dict(bind), set(cov)
                if match(roots[key], c, g, b2, c2):
                    bind, cov, hit = b2, c2, True
                    outs[key] = bind[key]
                    break
            ok &= hit
        if not ok:
            continue
        for key, pat in optional.items():
            anchor = bind["y"] if key == "am" else bind["dn"]
            for c in users.get(anchor, []):
                if c not in live:
                    continue
                b2, c2 = dict(bind), set(cov)
                if match(pat, c, g, b2, c2):
                    bind, cov = b2, c2
                    outs[key] = bind[key]
                    break
        # y is an output of the fused kernel too
        outs["y"] = bind["y"]
        # shape rules: x, cot [rows, C] fp32; a, b, gamma, beta [C] fp32
        mx = meta.get(bind["x"])
        if mx is None or mx.scalar or len(mx.shape) < 1 or mx.dtype != torch.float32:
            continue
        C = mx.shape[-1]
        good = meta[bind["cot"]].shape == mx.shape and meta[bind["cot"]].dtype == torch.float32
        for v in ("a", "b", "gamma", "beta"):
            m = meta.get(bind[v])
            good &= m is not None and not m.scalar and m.shape == (C,) and m.dtype == torch.float32
        good &= C <= 16384 and meta[bind["y"]].shape == mx.shape
        if not good:
            continue
        cov = {c for c in cov if c in live}
        found.append(Match("rowfused", bind, cov, outs))
    return found


def rowfused_step(m: Match, meta: dict[str, Meta], eps: float) -> Step:
    b, o = m.bind, m.outputs
    shape = meta[b["x"]].shape
    C = shape[-1]
    R = math.prod(shape[:-1])
    ins = [b[k] for k in ("x", "a", "b", "gamma", "beta", "cot")]
    lib_ws = L.lib().b200_rowfused_workspace_bytes
    ws_bytes = int(lib_ws(R, C))

    def run(env: dict) -> None:
        x, a, bb, ga, be, cot = (ops.contiguous(env[k]) for k in ins)
        dev = ops.device()
        y = torch.empty(shape, dtype=torch.float32, device=dev)
        dx = torch.empty(shape, dtype=torch.float32, device=dev)
        da = torch.empty(C, dtype=torch.float32, device=dev)
        db = torch.empty(C, dtype=torch.float32, device=dev)
        am = torch.empty(shape[:-1], dtype=torch.int64, device=dev) if "am" in o else None
        dgam = torch.empty(C, dtype=torch.float32, device=dev) if "dgamma" in o else None
        dbet = torch.empty(C, dtype=torch.float32, device=dev) if "dbeta" in o else None
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=dev)
        L.call("b200_rowfused_fwd_bwd", x.data_ptr(), a.data_ptr(), bb.data_ptr(), ga.data_ptr(), be.data_ptr(),
               cot.data_ptr(), y.data_ptr(), None if am is None else am.data_ptr(), dx.data_ptr(), da.data_ptr(),
               db.data_ptr(), None if dgam is None else dgam.data_ptr(), None if dbet is None else dbet.data_ptr(),
               R, C, float(eps), ws.data_ptr(), ws_bytes, ops.stream_ptr())
        env[o["y"]] = y
        env[o["dx"]] = dx
        env[o["da"]] = da
        env[o["db"]] = db
        if am is not None:
            env[o["am"]] = am
        if dgam is not None:
            env[o["dgamma"]] = dgam
        if dbet is not None:
            env[o["dbeta"]] = dbet

    return Step(list(o.values()), ins, run, "rowfused_fwd_bwd")


# ----------------------------------------------------------------------------------
# pattern: GEMM with fused bias + activation epilogue (+ ReLU-grad mask)
#   act(Matmul(A, B) + bias), bias a [N] vector; the backward's Greater(pre, 0) mask is
#   written by the same epilogue (one byte per element) instead of re-reading pre.
# ----------------------------------------------------------------------------------
def find_gemm_epilogue(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                       outputs: set[str]) -> list[Match]:
    found = []
    for nid, node in live.items():
        op = _op_name(node)
        if op not in ("Relu", "Gelu", "GELU", "Add"):
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if op == "Add":
            # bias epilogue without an activation: Add(Matmul(A, B), bias)
            pat = Op("Add", Op("Matmul", Var("A"), Var("B"), name="mm"), Var("bias"), name="act")
        else:
            pat = Op(op, Op("Add", Op("Matmul", Var("A"), Var("B"), name="mm"), Var("bias"), name="pre"), name="act")
        if not match(pat, nid, g, bind, cov):
            continue
        if op == "Add":
            bind["pre"] = bind["act"]
        mm = g.nodes[bind["mm"]]
        if mm.attributes.get("transpose_a") or mm.attributes.get("transpose_b"):
            continue
        N = meta[bind["mm"]].shape[-1] if not meta[bind["mm"]].scalar else 0
        mb = meta.get(bind["bias"])
        if mb is None or mb.scalar or mb.shape != (N,):
            continue
        if meta[bind["act"]].shape != meta[bind["mm"]].shape:
            continue
        outs = {"act": bind["act"]}
        # the ReLU-grad mask: Greater(pre, 0)
        if op == "Relu":
            for u in users.get(bind["pre"], []):
                un = live.get(u)
                if un is not None and _op_name(un) == "Greater" and un.inputs[0] == bind["pre"] and _const_value(g, un.inputs[1]) == 0.0:
                    outs["mask"] = u
                    cov.add(u)
                    cov.add(un.inputs[1])
        # mm must not be needed elsewhere; pre either not, or it is kept as a second output
        def leaks(v: str) -> bool:
            return v in outputs or any(u not in cov for u in users.get(v, []))

        if leaks(bind["mm"]):
            continue
        if op != "Relu" and "mask" in outs:
            continue
        kind = "gemm_bias" if op == "Add" else "gemm_" + op.lower()
        bf, f32 = gemm_use(bind["act"], live, users, outputs)
        bind["bf16"] = str(bf and not f32)
        bind["twin"] = str(bf and f32)  # fp32 result plus a bf16 copy for the GEMM consumers
        if op != "Add" and leaks(bind["pre"]):
            # the VJP reads the pre-activation (GELU): the epilogue writes pre in fp32 and,
            # when the activation only feeds bf16 GEMMs, the activation in bf16 beside it
            if bind["bf16"] != "True":
                continue
            outs["pre"] = bind["pre"]
            kind += "_dual"
        found.append(Match(kind, bind, {c for c in cov if c in live or g.nodes[c].op_type == "Constant"}, outs))
    # activation epilogues first: a plain bias match must not pre-empt the ReLU/GELU one
    found.sort(key=lambda m: m.kind == "gemm_bias")
    return found


def find_gemm_residual(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                       outputs: set[str]) -> list[Match]:
    """Add(R, Add(Matmul(A, B), bias)), either operand order of the outer Add, where the
    matmul and the bias sum feed nothing else: one GEMM whose epilogue adds the bias and
    then R (a transformer's residual connection after an output projection)."""
    found = []
    pat = Op("Add", Op("Matmul", Var("A"), Var("B"), name="mm"), Var("bias"), name="pre")
    for nid, node in live.items():
        if _op_name(node) != "Add" or len(node.inputs) != 2:
            continue
        for k in (0, 1):
            inner, rid = live.get(node.inputs[k]), node.inputs[1 - k]
            if inner is None or _op_name(inner) != "Add":
                continue
            bind: dict[str, str] = {}
            cov: set[str] = set()
            if not match(pat, inner.id, g, bind, cov):
                continue
            mm = g.nodes[bind["mm"]]
            if mm.attributes.get("transpose_a") or mm.attributes.get("transpose_b"):
                continue
            mo, mr, mbias, mB = meta.get(nid), meta.get(rid), meta.get(bind["bias"]), meta.get(bind["B"])
            if any(x is None or x.scalar for x in (mo, mr, mbias, mB)) or len(mB.shape) != 2:
                continue
            N = mo.shape[-1]
            if mbias.shape != (N,) or mr.shape != mo.shape or meta[bind["pre"]].shape != mo.shape or \
                    meta[bind["mm"]].shape != mo.shape or mr.dtype != torch.float32 or mo.dtype != torch.float32:
                continue
            cov.add(nid)
            if rid in cov or any(v in outputs or any(u not in cov for u in users.get(v, [])) for v in (bind["mm"], bind["pre"])):
                continue
            bind.update({"R": rid, "act": nid})
            found.append(Match("gemm_bias_residual", bind, {c for c in cov if c in live or g.nodes[c].op_type == "Constant"},
                               {"act": nid}))
            break
    return found


def gemm_residual_step(m: Match) -> Step:
    b = m.bind

    def run(env: dict) -> None:
        env[b["act"]] = ops.gemm(env[b["A"]], env[b["B"]], bias=env[b["bias"]], resid=env[b["R"]])

    return Step([b["act"]], [b["A"], b["B"], b["bias"], b["R"]], run, "gemm_bias_residual")


def gemm_epilogue_step(m: Match) -> Step:
    b, o = m.bind, m.outputs
    kind = m.kind.replace("_dual", "")
    epi = {"gemm_relu": L.EPI_RELU, "gemm_gelu": L.EPI_GELU}.get(kind, L.EPI_NONE)
    want_mask = "mask" in o
    dual = m.kind.endswith("_dual")
    out_dt = torch.bfloat16 if (b.get("bf16") == "True" and not dual) else torch.float32
    twin = not dual and b.get("twin") == "True" and epi == L.EPI_NONE
    ins = [b["A"], b["B"], b["bias"]]

    def run(env: dict) -> None:
        res = ops.gemm(env[b["A"]], env[b["B"]], bias=env[b["bias"]], epilogue=epi, want_mask=want_mask, out_dtype=out_dt,
                       act_bf16=dual or twin)
        if twin:
            env[o["act"]] = res[0]
            ops.register_cast(res[0], res[1])
            if want_mask:
                env[o["mask"]] = res[2]
        elif dual:
            env[o["pre"]], env[o["act"]] = res[0], res[1]
            if want_mask:
                env[o["mask"]] = res[2]
        elif want_mask:
            env[o["act"]], env[o["mask"]] = res
        else:
            env[o["act"]] = res

    label = m.kind + ("[bf16]" if out_dt == torch.bfloat16 else ("[+bf16]" if twin else ""))
    return Step(list(o.values()), ins, run, label)


# ----------------------------------------------------------------------------------
# patterns: convolution epilogues (bf16 implicit-GEMM convolutions)
#   Relu(Conv2D(x, w)) -> one kernel writing relu(.) only. The pre-activation's other
#   readers are the ReLU VJP's Greater(pre, 0) masks, and Greater(relu(pre), 0) is the
#   same mask elementwise, so the ReLU output stands in for the pre-activation there.
#   Multiply(Conv2DInputGrad(dy, w), Greater(pre, 0)) -> the input-gradient kernel
#   multiplies by (pre > 0) in its epilogue.
# ----------------------------------------------------------------------------------
def _is_zero_mask(g: Graph, n: Node | None, of: str) -> bool:
    return n is not None and _op_name(n) == "Greater" and len(n.inputs) == 2 and n.inputs[0] == of and \
        _const_value(g, n.inputs[1]) == 0.0


def _conv_attrs(n: Node) -> dict:
    return {k: n.attributes[k] for k in ("stride", "strides", "padding", "groups", "dilation", "dilations", "target_shape")
            if k in n.attributes}


def _conv_ok(kind: int, n: Node, meta: dict[str, Meta]) -> bool:
    a = n.attributes
    if int(a.get("groups", 1) or 1) != 1 or ops._stride2(a.get("dilations", a.get("dilation", 1)) or 1) != (1, 1):
        return False
    stride = a.get("strides", a.get("stride", (1, 1)))
    padding = a.get("padding", "SAME")
    mi = [meta.get(i) for i in n.inputs[:2]]
    mo = meta.get(n.id)
    if any(m is None or m.scalar or m.dtype != torch.float32 for m in mi) or mo is None or mo.scalar:
        return False
    if kind == 0:
        return ops.conv_fused_ok(0, mi[0].shape, mi[1].shape, stride, padding, out_hw=tuple(mo.shape[2:]))
    # input gradient: x shape = target_shape (= the output's), dy = inputs[0]
    return len(mo.shape) == 4 and ops.conv_fused_ok(1, mo.shape, mi[1].shape, stride, padding, out_hw=tuple(mi[0].shape[2:]))


def find_conv_relu(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                   outputs: set[str]) -> list[Match]:
    found = []
    for nid, node in live.items():
        if _op_name(node) != "Relu" or len(node.inputs) != 1:
            continue
        conv = live.get(node.inputs[0])
        if conv is None or _op_name(conv) != "Conv2D" or conv.id in outputs or len(conv.inputs) != 2:
            continue
        others = [u for u in users.get(conv.id, []) if u != nid]
        if not all(_is_zero_mask(g, live.get(u), conv.id) for u in others):
            continue
        if meta[nid].shape != meta[conv.id].shape or not _conv_ok(0, conv, meta):
            continue
        found.append(Match("conv_relu", {"x": conv.inputs[0], "w": conv.inputs[1], "conv": conv.id, "act": nid},
                           {conv.id, nid}, {"act": nid, "conv": conv.id}))
    return found


def conv_relu_step(m: Match, g: Graph) -> Step:
    b = m.bind
    kw = _conv_attrs(g.nodes[b["conv"]])
    info = {"values": [b["act"], b["conv"]], "x": b["x"], "relu": True, "fp32": True}

    def run(env: dict) -> None:
        r = ops.op_conv2d(env[b["x"]], env[b["w"]], relu=True, fp32_out=info["fp32"], **kw)
        env[b["act"]] = r
        env[b["conv"]] = r  # read only by Greater(pre, 0) masks: same mask from relu(pre)

    st = Step([b["act"], b["conv"]], [b["x"], b["w"]], run, "conv_relu")
    st.conv_copy = info
    return st


def find_conv_dgrad_mask(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                         outputs: set[str]) -> list[Match]:
    found = []
    pat = Op("Multiply", Op("Conv2DInputGrad", Var("dy"), Var("w"), name="dg"), Op("Greater", Var("pre"), Const(0.0), name="gt"),
             name="mul")
    for nid, node in live.items():
        if _op_name(node) != "Multiply":
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if not match(pat, nid, g, bind, cov):
            continue
        if any(v in outputs or any(u != nid for u in users.get(v, [])) for v in (bind["dg"], bind["gt"])):
            continue
        mp, mo = meta.get(bind["pre"]), meta.get(nid)
        if mp is None or mo is None or mp.scalar or mp.shape != mo.shape or mp.dtype != torch.float32:
            continue
        if meta[bind["dg"]].shape != mo.shape or not _conv_ok(1, g.nodes[bind["dg"]], meta):
            continue
        found.append(Match("conv_dgrad_mask", bind, {c for c in cov if c in live or g.nodes[c].op_type == "Constant"},
                           {"dx": nid}))
    return found


def conv_dgrad_mask_step(m: Match, g: Graph) -> Step:
    b = m.bind
    kw = _conv_attrs(g.nodes[b["dg"]])
    info = {"values": [b["mul"]], "dy": b["dy"], "pre": b["pre"], "relu": False, "fp32": True}

    def run(env: dict) -> None:
        env[b["mul"]] = ops.op_conv2d_input_grad(env[b["dy"]], env[b["w"]], mask=env[b["pre"]], fp32_out=info["fp32"], **kw)

    st = Step([b["mul"]], [b["dy"], b["w"], b["pre"]], run, "conv_dgrad_mask")
    st.conv_copy = info
    return st


def _reads_copy(r: Step, v: str, producer: dict, meta: dict[str, Meta], g: Graph) -> bool:
    """Whether step ``r`` reads value ``v`` only through the bf16 channels-last copy that the
    fused convolution ``producer`` writes beside it (same channel padding)."""
    mv = meta.get(v)
    if mv is None or mv.scalar or len(mv.shape) != 4:
        return False
    cp = ops._rup(mv.shape[1], 8)
    info = getattr(r, "conv_copy", None)
    if r.label == "conv_relu" and info is not None:
        return info["x"] == v  # channels_last(x, C rounded up to 8)
    if r.label == "conv_dgrad_mask" and info is not None:
        if info["pre"] == v:
            return producer["relu"]  # the mask from the ReLU output's copy (nonzero where > 0)
        return info["dy"] == v  # channels_last(dy, O rounded up to 8)
    if r.label == "Conv2DWeightGrad" and len(r.inputs) >= 2 and v in r.inputs[:2]:
        node = g.nodes.get(r.outputs[0])
        mx, mdy = meta.get(r.inputs[0]), meta.get(r.inputs[1])
        if node is None or mx is None or mdy is None or mx.scalar or mdy.scalar or len(mdy.shape) != 4:
            return False
        a = node.attributes
        ts = a.get("target_shape")
        if ts is None or len(ts) != 4:
            return False
        if not ops.conv_fused_ok(2, mx.shape, tuple(int(t) for t in ts), a.get("strides", a.get("stride", (1, 1))),
                                 a.get("padding", "SAME"), out_hw=tuple(mdy.shape[2:])):
            return False  # the staged (non-implicit) weight gradient reads fp32
        if r.inputs[1] == v and cp != ops._rup(mv.shape[1], 64):
            return False  # its dy copy has the channels padded to 64
        return True
    return False


def _conv_copy_only(steps: list[Step], outputs: set[str], meta: dict[str, Meta], g: Graph) -> None:
    """Fused convolution results that every reader takes from the channels-last bf16 copy
    of the fused epilogue (the next convolution's operand, the weight gradient's operands,
    the ReLU VJP mask of an input gradient) skip their fp32 NCHW write: the step still
    returns an fp32 tensor (the copy's cache key), left unwritten."""
    readers: dict[str, list[Step]] = {}
    for st in steps:
        for v in st.inputs:
            readers.setdefault(v, []).append(st)
    for st in steps:
        info = getattr(st, "conv_copy", None)
        if info is None or any(v in outputs for v in info["values"]):
            continue
        if all(_reads_copy(r, v, info, meta, g) for v in info["values"] for r in readers.get(v, []) if r is not st):
            info["fp32"] = False


def _perm_of(n: Node, ndim: int) -> list[int]:
    axes = n.attributes.get("axes", n.attributes.get("perm"))
    if axes is None:
        return list(reversed(range(ndim)))
    return [int(a) % ndim for a in axes]


def _contig_strides(shape: tuple) -> list[int]:
    st, acc = [], 1
    for d in reversed(shape):
        st.append(acc)
        acc *= max(1, d)
    return list(reversed(st))


def find_matmul_transpose(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                          outputs: set[str], taken: set[str]) -> list[Match]:
    """Transpose(Matmul(a, b), perm) where the Matmul feeds nothing else: the GEMM writes
    straight into the transposed (contiguous) layout, so the Transpose and any Reshape
    after it are views (attention's head merge / split of q, k, v and their gradients)."""
    found = []
    for tid, tn in live.items():
        if _op_name(tn) != "Transpose" or len(tn.inputs) != 1 or tid in taken:
            continue
        mm = tn.inputs[0]
        mn = live.get(mm)
        if mn is None or mm in taken or _op_name(mn) != "Matmul" or len(mn.inputs) != 2:
            continue
        if mm in outputs or users.get(mm) != [tid]:
            continue
        mo, to = meta.get(mm), meta.get(tid)
        if mo is None or to is None or mo.scalar or len(mo.shape) < 3 or mo.dtype != torch.float32:
            continue
        nd = len(mo.shape)
        perm = _perm_of(tn, nd)
        inv = [perm.index(i) for i in range(nd)]
        cst = [_contig_strides(to.shape)[inv[i]] for i in range(nd)]  # strides of C inside Y
        if cst[-1] == 1:
            swap = False
        elif cst[-2] == 1:
            swap = True
        else:
            continue
        bf, f32 = gemm_use(tid, live, users, outputs)
        bind = {"mm": mm, "t": tid, "a": mn.inputs[0], "b": mn.inputs[1], "perm": ",".join(map(str, perm)),
                "swap": str(swap), "bf16": str(bf), "f32": str(f32)}
        found.append(Match("matmul_transpose", bind, {mm, tid}, {"y": tid}))
    return found


def matmul_transpose_step(m: Match, meta: dict[str, Meta]) -> Step:
    b = m.bind
    mn = None
    perm = [int(x) for x in b["perm"].split(",")]
    inv = [perm.index(i) for i in range(len(perm))]
    yshape = meta[b["t"]].shape
    swap, bf, f32 = b["swap"] == "True", b["bf16"] == "True", b["f32"] == "True"
    del mn

    def run(env: dict, _kw=None) -> None:
        a, bb = env[b["a"]], env[b["b"]]
        kw = _kw or {}
        if kw.get("transpose_a"):
            a = a.transpose(-1, -2)
        if kw.get("transpose_b"):
            bb = bb.transpose(-1, -2)
        y, yb = _out_buffers(yshape, f32, bf)
        prim = y if y is not None else yb
        out = prim.permute(*inv)
        out2 = yb.permute(*inv) if (y is not None and yb is not None) else None
        if swap:
            ok = ops.gemm_out(bb.transpose(-1, -2), a.transpose(-1, -2), out.transpose(-1, -2),
                              None if out2 is None else out2.transpose(-1, -2))
        else:
            ok = ops.gemm_out(a, bb, out, out2)
        if not ok:
            res = ops.gemm(a, bb)
            yc = ops.contiguous(res.permute(*perm))
            y = yc if f32 else None
            yb = ops.cast(yc, torch.bfloat16) if bf else None
        _publish(env, b["t"], y, yb)

    return Step([b["t"]], [b["a"], b["b"]], run, "matmul_T" + ("[bf16]" if bf and not f32 else ("[+bf16]" if bf else "")))


def layernorm_step(n: Node, f32: bool) -> Step:
    """LayerNorm writing bf16 for its GEMM consumers (and fp32 only if something else
    reads it)."""
    kw = node_kwargs(n, "LayerNorm")
    eps = float(kw.get("epsilon", kw.get("eps", 1e-5)))
    axis = kw.get("axis", -1)
    ins = list(n.inputs)

    def run(env: dict) -> None:
        args = [env[i] for i in ins]
        y, yb = ops.layer_norm(args[0], args[1] if len(args) > 1 else None, args[2] if len(args) > 2 else None, eps, axis,
                               f32=f32, bf16=True)
        _publish(env, n.id, y, yb)

    return Step([n.id], ins, run, "LayerNorm" + ("" if f32 else "[bf16]"))


def matmul_step(n: Node, bf16_out: bool, shape: tuple = (), twin: bool = False) -> Step:
    """A Matmul node without a fused epilogue; its output is written in bf16 when it
    only feeds bf16 GEMMs, or in fp32 with a bf16 twin (``twin``) when both are read."""
    kw = node_kwargs(n, "Matmul")
    ta, tb = bool(kw.get("transpose_a")), bool(kw.get("transpose_b"))
    a_id, b_id = n.inputs[0], n.inputs[1]
    out_dt = torch.bfloat16 if bf16_out else torch.float32

    def run(env: dict) -> None:
        a, bb = env[a_id], env[b_id]
        if ta:
            a = a.transpose(-1, -2)
        if tb:
            bb = bb.transpose(-1, -2)
        if twin:
            y, yb = _out_buffers(shape, True, True)
            if ops.gemm_out(a, bb, y, yb):
                _publish(env, n.id, y, yb)
                return
        env[n.id] = ops.gemm(a, bb, out_dtype=out_dt)

    return Step([n.id], [a_id, b_id], run, "Matmul" + ("[bf16]" if bf16_out else ("[+bf16]" if twin else "")))


# ----------------------------------------------------------------------------------
# pattern: ReLU-with-bias backward  gp = cot * mask ; dbias = BroadcastReduce(gp, bias)
# ----------------------------------------------------------------------------------
def _only_gemm_consumers(g: Graph, v: str, live: dict[str, Node], users: dict[str, list[str]], skip: set[str]) -> bool:
    for u in users.get(v, []):
        if u in skip or u not in live:
            continue
        op = _op_name(live[u])
        if op == "Matmul":
            continue
        if op in ("Transpose", "Reshape") and _only_gemm_consumers(g, u, live, users, skip):
            continue
        return False
    return True


def find_mask_bwd(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                  outputs: set[str]) -> list[Match]:
    found = []
    for nid, node in live.items():
        if _op_name(node) != "Multiply" or len(node.inputs) != 2:
            continue
        m0, m1 = meta.get(node.inputs[0]), meta.get(node.inputs[1])
        if m0 is None or m1 is None or m0.scalar or m1.scalar:
            continue
        if m1.dtype == torch.bool and m0.dtype == torch.float32:
            cot, mask = node.inputs
        elif m0.dtype == torch.bool and m1.dtype == torch.float32:
            mask, cot = node.inputs
        else:
            continue
        mo = meta[nid]
        if mo.shape != meta[cot].shape or mo.shape != meta[mask].shape or len(mo.shape) < 1:
            continue
        C = mo.shape[-1]
        br = None
        for u in users.get(nid, []):
            un = live.get(u)
            if un is not None and _op_name(un) == "BroadcastReduce" and un.inputs[0] == nid:
                mb = meta.get(un.inputs[1])
                if mb is not None and not mb.scalar and mb.shape == (C,) and meta[u].shape == (C,):
                    br = u
                    break
        if br is None:
            continue
        bf16_only = ops.Config.matmul_dtype == "bf16" and nid not in outputs and _only_gemm_consumers(g, nid, live, users, {br})
        found.append(Match("relu_bwd_bias", {"cot": cot, "mask": mask, "gp": nid, "db": br, "bf16": str(bf16_only)},
                           {nid, br}, {"gp": nid, "db": br}))
    return found


def mask_bwd_step(m: Match, meta: dict[str, Meta]) -> Step:
    b = m.bind
    shape = meta[b["gp"]].shape
    C = shape[-1]
    R = math.prod(shape[:-1])
    bf16_only = b["bf16"] == "True"
    ws_bytes = int(L.lib().b200_mask_mul_colsum_workspace_bytes(R, C))

    def run(env: dict) -> None:
        g = ops.contiguous(env[b["cot"]])
        mk = ops.contiguous(env[b["mask"]])
        dev = ops.device()
        gp = torch.empty(shape, dtype=torch.bfloat16 if bf16_only else torch.float32, device=dev)
        db = torch.empty(C, dtype=torch.float32, device=dev)
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=dev)
        L.call("b200_mask_mul_colsum", g.data_ptr(), mk.data_ptr(), gp.data_ptr() if bf16_only else None,
               None if bf16_only else gp.data_ptr(), db.data_ptr(), R, C, ws.data_ptr(), ws_bytes, ops.stream_ptr())
        env[b["gp"]] = gp
        env[b["db"]] = db

    return Step([b["gp"], b["db"]], [b["cot"], b["mask"]], run, "relu_bwd_bias" + ("[bf16]" if bf16_only else ""))


# ----------------------------------------------------------------------------------
# pattern: LogSoftmax -> TakeAlongAxis (label pick) and the VJP chain
#   ZerosLike + ScatterAdd + (g - exp(ls) * sum(g))  ->  one kernel
# ----------------------------------------------------------------------------------
def find_xent(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
              outputs: set[str]) -> list[Match]:
    x, labels, d = Var("x"), Var("labels"), Var("d")
    ls = Op("LogSoftmax", x, name="ls", attrs={"axis": _last_axis})
    dls = Op("ScatterAdd", Op("ZerosLike", ls, name="z"), labels, d, name="dls", attrs={"dim": lambda v: v in (-1, None) or v == -1})
    s = Op("ReduceSum", dls, name="s", attrs={"axis": _last_axis, "keepdims": True})
    root = Op("Subtract", dls, Op("Multiply", Op("Exp", ls, name="e"), s, name="es"), name="dx")
    found = []
    for nid, node in live.items():
        if _op_name(node) != "Subtract":
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if not match(root, nid, g, bind, cov):
            continue
        mx, ml, md = meta.get(bind["x"]), meta.get(bind["labels"]), meta.get(bind["d"])
        if mx is None or mx.scalar or len(mx.shape) < 1 or mx.dtype not in (torch.float32, torch.bfloat16):
            continue
        R = math.prod(mx.shape[:-1])
        if ml is None or ml.dtype != torch.int64 or ml.shape != tuple(mx.shape[:-1]) + (1,):
            continue
        if md is None or md.scalar or md.shape != ml.shape or md.dtype != torch.float32:
            continue
        outs = {"dx": bind["dx"]}
        for u in users.get(bind["ls"], []):
            un = live.get(u)
            if un is not None and _op_name(un) == "TakeAlongAxis" and un.inputs == [bind["ls"], bind["labels"]] and _last_axis(un.attributes.get("axis", -1)):
                outs["picked"] = u
                cov.add(u)
        produced = set(outs.values())
        leak = [c for c in cov if c not in produced and (c in outputs or any(u not in cov for u in users.get(c, [])))]
        if leak:
            continue
        del R
        found.append(Match("xent", bind, cov, outs))
    return found


def xent_step(m: Match, meta: dict[str, Meta], bf16_dx: bool = False) -> Step:
    b, o = m.bind, m.outputs
    shape = meta[b["x"]].shape
    V = shape[-1]
    R = math.prod(shape[:-1])
    # dx straight in bf16 when it only feeds the output-projection GEMMs (fp32 logits,
    # whole 4-column groups: the register-row kernel)
    bf = bf16_dx and V % 4 == 0 and meta[b["x"]].dtype == torch.float32

    def run(env: dict) -> None:
        x = ops.contiguous(env[b["x"]])
        lab = ops.contiguous(env[b["labels"]])
        d = ops.contiguous(ops.cast(env[b["d"]], torch.float32))
        dev = ops.device()
        dx = None if bf else torch.empty(shape, dtype=torch.float32, device=dev)
        dxb = torch.empty(shape, dtype=torch.bfloat16, device=dev) if bf else None
        picked = torch.empty(tuple(shape[:-1]) + (1,), dtype=torch.float32, device=dev) if "picked" in o else None
        L.call("b200_logsoftmax_pick", ops.code(x), x.data_ptr(), lab.data_ptr(), d.data_ptr(),
               None if picked is None else picked.data_ptr(), None, None if dx is None else dx.data_ptr(),
               None if dxb is None else dxb.data_ptr(), R, V, ops.stream_ptr())
        env[o["dx"]] = dxb if bf else dx
        if picked is not None:
            env[o["picked"]] = picked

    return Step(list(o.values()), [b["x"], b["labels"], b["d"]], run, "xent_fwd_bwd" + ("[bf16]" if bf else ""))


# ----------------------------------------------------------------------------------
# pattern: GELU backward  dp = g * gelu'(p)  (+ bias gradient BroadcastReduce(dp, bias))
# ----------------------------------------------------------------------------------
def find_gelu_bwd(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                  outputs: set[str]) -> list[Match]:
    root = Op("Multiply", Var("g"), gelu_tanh_deriv(Var("p")), name="dp")
    found = []
    for nid, node in live.items():
        if _op_name(node) != "Multiply":
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if not match(root, nid, g, bind, cov):
            continue
        mg, mp, mo = meta.get(bind["g"]), meta.get(bind["p"]), meta.get(nid)
        if mg is None or mp is None or mo is None or mg.scalar or mp.scalar or len(mp.shape) < 1:
            continue
        if mg.shape != mp.shape or mo.shape != mp.shape or mg.dtype != torch.float32 or mp.dtype != torch.float32:
            continue
        cov = {c for c in cov if c in live or g.nodes[c].op_type == "Constant"}
        inner = [c for c in cov if c != nid and c in live]
        if any(c in outputs or any(u not in cov for u in users.get(c, [])) for c in inner):
            continue
        C = mp.shape[-1]
        br = None
        for u in users.get(nid, []):
            un = live.get(u)
            if un is not None and _op_name(un) == "BroadcastReduce" and un.inputs[0] == nid:
                mb = meta.get(un.inputs[1])
                if mb is not None and not mb.scalar and mb.shape == (C,) and meta[u].shape == (C,):
                    br = u
                    break
        skip = frozenset([br]) if br else frozenset()
        bf, f32 = gemm_use(nid, live, users, outputs, skip)
        bind.update({"db": br or "", "bf16": str(bf), "f32": str(f32)})
        outs = {"dp": nid}
        if br:
            outs["db"] = br
            cov.add(br)
        found.append(Match("gelu_bwd", bind, cov, outs))
    return found


def gelu_bwd_step(m: Match, meta: dict[str, Meta]) -> Step:
    b, o = m.bind, m.outputs
    shape = meta[o["dp"]].shape
    C = shape[-1]
    R = math.prod(shape[:-1])
    bf, f32 = b["bf16"] == "True", b["f32"] == "True"
    ws_bytes = int(L.lib().b200_gelu_bwd_colsum_workspace_bytes(R, C))

    def run(env: dict) -> None:
        gg = ops.contiguous(ops.cast(env[b["g"]], torch.float32))
        pp = ops.contiguous(ops.cast(env[b["p"]], torch.float32))
        dev = ops.device()
        y, yb = _out_buffers(shape, f32, bf)
        db = torch.empty(C, dtype=torch.float32, device=dev) if "db" in o else None
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=dev)
        L.call("b200_gelu_bwd_colsum", gg.data_ptr(), pp.data_ptr(), None if yb is None else yb.data_ptr(),
               None if y is None else y.data_ptr(), None if db is None else db.data_ptr(), R, C, ws.data_ptr(), ws_bytes,
               ops.stream_ptr())
        _publish(env, o["dp"], y, yb)
        if db is not None:
            env[o["db"]] = db

    label = "gelu_bwd" + ("_bias" if "db" in o else "") + ("[bf16]" if bf and not f32 else "")
    return Step(list(o.values()), [b["g"], b["p"]], run, label)


# ----------------------------------------------------------------------------------
# pattern: LayerNormInputGrad + LayerNormGammaGrad + LayerNormBetaGrad of one (dy, x)
# ----------------------------------------------------------------------------------
def find_ln_bwd(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                outputs: set[str]) -> list[Match]:
    found = []
    for nid, node in live.items():
        if _op_name(node) != "LayerNormInputGrad" or len(node.inputs) < 2:
            continue
        dy, x = node.inputs[0], node.inputs[1]
        gamma = node.inputs[2] if len(node.inputs) > 2 else ""
        mx, md = meta.get(x), meta.get(dy)
        if mx is None or md is None or mx.scalar or md.scalar or md.shape != mx.shape or len(mx.shape) < 1:
            continue
        if mx.dtype != torch.float32 or md.dtype != torch.float32 or node.attributes.get("axis", -1) not in (-1, None):
            continue
        outs, cov = {"dx": nid}, {nid}
        for u in users.get(dy, []):
            un = live.get(u)
            if un is None or u == nid or un.attributes.get("axis", -1) not in (-1, None):
                continue
            op = _op_name(un)
            if op == "LayerNormGammaGrad" and un.inputs[:2] == [dy, x] and "dgamma" not in outs:
                outs["dgamma"] = u
                cov.add(u)
            elif op == "LayerNormBetaGrad" and un.inputs[:1] == [dy] and "dbeta" not in outs:
                outs["dbeta"] = u
                cov.add(u)
        eps = float(node.attributes.get("eps", node.attributes.get("epsilon", 1e-5)))
        if "dgamma" in outs:
            ge = float(live[outs["dgamma"]].attributes.get("eps", live[outs["dgamma"]].attributes.get("epsilon", 1e-5)))
            if ge != eps:
                cov.discard(outs.pop("dgamma"))
        bind = {"dy": dy, "x": x, "gamma": gamma, "eps": repr(eps)}
        found.append(Match("ln_bwd", bind, cov, outs))
    return found


def ln_bwd_step(m: Match, meta: dict[str, Meta]) -> Step:
    b, o = m.bind, m.outputs
    shape = meta[b["x"]].shape
    C = shape[-1]
    R = math.prod(shape[:-1])
    eps = float(b["eps"])
    ws_bytes = int(L.lib().b200_layernorm_bwd_workspace_bytes(R, C))
    ins = [b["dy"], b["x"]] + ([b["gamma"]] if b["gamma"] else [])

    def run(env: dict) -> None:
        dy = ops.contiguous(ops.cast(env[b["dy"]], torch.float32))
        x = ops.contiguous(ops.cast(env[b["x"]], torch.float32))
        ga = ops.contiguous(ops.cast(env[b["gamma"]], torch.float32)) if b["gamma"] else None
        dev = ops.device()
        dx = torch.empty(shape, dtype=torch.float32, device=dev)
        dg = torch.empty(C, dtype=torch.float32, device=dev) if "dgamma" in o else None
        db = torch.empty(C, dtype=torch.float32, device=dev) if "dbeta" in o else None
        ws = torch.empty(max(1, ws_bytes), dtype=torch.uint8, device=dev)
        L.call("b200_layernorm_bwd_rows", dy.data_ptr(), x.data_ptr(), None if ga is None else ga.data_ptr(), dx.data_ptr(),
               None, None if dg is None else dg.data_ptr(), None if db is None else db.data_ptr(), R, C, eps, ws.data_ptr(),
               ws_bytes, ops.stream_ptr())
        env[o["dx"]] = dx
        if dg is not None:
            env[o["dgamma"]] = dg
        if db is not None:
            env[o["dbeta"]] = db

    return Step(list(o.values()), ins, run, "ln_bwd" + ("+params" if len(o) > 1 else ""))


# ----------------------------------------------------------------------------------
# operand dtype of values that feed the tensor cores
# ----------------------------------------------------------------------------------
def gemm_use(v: str, live: dict[str, Node], users: dict[str, list[str]], outputs: set[str],
             skip: frozenset = frozenset()) -> tuple[bool, bool]:
    """(feeds a bf16 GEMM, needed in fp32): walks the consumers of ``v`` through
    Transpose/Reshape views. A value that only feeds bf16 GEMMs is produced in bf16 by
    its kernel (the cast the GEMM would do, moved into the producer's store)."""
    if ops.Config.matmul_dtype != "bf16":
        return False, True
    gemm = other = False
    stack, seen = [v], set()
    while stack:
        x = stack.pop()
        if x in seen:
            continue
        seen.add(x)
        if x in outputs:
            other = True
        for u in users.get(x, []):
            if u in skip or u not in live:
                continue
            op = _op_name(live[u])
            if op == "Matmul":
                gemm = True
            elif op in ("Transpose", "Reshape"):
                stack.append(u)
            else:
                other = True
    return gemm, other or not gemm


def _out_buffers(shape: tuple, f32: bool, bf16: bool) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    dev = ops.device()
    y = torch.empty(shape, dtype=torch.float32, device=dev) if f32 else None
    yb = torch.empty(shape, dtype=torch.bfloat16, device=dev) if bf16 else None
    return y, yb


def _publish(env: dict, key: str, y: torch.Tensor | None, yb: torch.Tensor | None) -> None:
    """fp32 value in the environment with its bf16 twin registered for GEMM operands,
    or the bf16 value alone when nothing needs fp32."""
    if y is not None:
        env[key] = y
        if yb is not None:
            ops.register_cast(y, yb)
    else:
        env[key] = yb


def _scalar_tensor(m: Meta | None) -> bool:
    return m is not None and not m.scalar and math.prod(m.shape) == 1 and m.dtype == torch.float32


# ----------------------------------------------------------------------------------
# pattern: [Multiply(x, s) ->] Softmax / LogSoftmax over the last axis, s a device scalar
# ----------------------------------------------------------------------------------
def find_softmax(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                 outputs: set[str]) -> list[Match]:
    found = []
    for nid, node in live.items():
        op = _op_name(node)
        if op not in ("Softmax", "LogSoftmax") or len(node.inputs) != 1:
            continue
        x = node.inputs[0]
        mx, my = meta.get(x), meta.get(nid)
        if mx is None or mx.scalar or mx.dtype != torch.float32 or len(mx.shape) < 1 or my is None or my.shape != mx.shape:
            continue
        ax = node.attributes.get("axis", -1)
        if not (ax is None or int(ax) % len(mx.shape) == len(mx.shape) - 1):
            continue
        cov, src, scale = {nid}, x, ""
        xn = live.get(x)
        if xn is not None and _op_name(xn) == "Multiply" and x not in outputs and users.get(x) == [nid]:
            a, b = xn.inputs
            for big, sm in ((a, b), (b, a)):
                mb = meta.get(big)
                if mb is not None and not mb.scalar and mb.shape == mx.shape and mb.dtype == torch.float32 and _scalar_tensor(meta.get(sm)):
                    src, scale = big, sm
                    cov.add(x)
                    break
        bf, f32 = gemm_use(nid, live, users, outputs)
        bind = {"x": src, "scale": scale, "y": nid, "log": str(op == "LogSoftmax"), "bf16": str(bf), "f32": str(f32)}
        found.append(Match("softmax", bind, cov, {"y": nid}))
    return found


def softmax_step(m: Match, meta: dict[str, Meta]) -> Step:
    b = m.bind
    shape = meta[b["y"]].shape
    cols = shape[-1]
    rows = math.prod(shape[:-1])
    log, bf, f32 = b["log"] == "True", b["bf16"] == "True", b["f32"] == "True"
    ins = [b["x"]] + ([b["scale"]] if b["scale"] else [])

    def run(env: dict) -> None:
        x = ops.contiguous(ops.cast(env[b["x"]], torch.float32))
        sc = ops.contiguous(ops.cast(env[b["scale"]], torch.float32)) if b["scale"] else None
        y, yb = _out_buffers(shape, f32, bf)
        L.call("b200_softmax_rows", x.data_ptr(), None if sc is None else sc.data_ptr(), None if y is None else y.data_ptr(),
               None if yb is None else yb.data_ptr(), rows, cols, 1 if log else 0, ops.stream_ptr())
        _publish(env, b["y"], y, yb)

    label = ("scaled_" if b["scale"] else "") + ("log_softmax" if log else "softmax") + ("[bf16]" if bf and not f32 else "")
    return Step([b["y"]], ins, run, label)


# ----------------------------------------------------------------------------------
# pattern: softmax VJP  y * (g - ReduceSum(g * y, -1, keepdims)) [* s]
# ----------------------------------------------------------------------------------
def find_softmax_bwd(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                     outputs: set[str]) -> list[Match]:
    y, gv = Var("y"), Var("g")
    s = Op("ReduceSum", Op("Multiply", gv, y, name="gy"), name="s", attrs={"axis": _last_axis, "keepdims": True})
    inner = Op("Multiply", y, Op("Subtract", gv, s, name="d"), name="dx")
    scaled = Op("Multiply", inner, Var("scale"), name="out")
    cands = []
    for nid, node in live.items():
        if _op_name(node) != "Multiply":
            continue
        bind: dict[str, str] = {}
        cov: set[str] = set()
        if match(scaled, nid, g, bind, cov) and _scalar_tensor(meta.get(bind["scale"])):
            cands.append((0, bind, cov, bind["out"]))
            continue
        bind, cov = {}, set()
        if match(inner, nid, g, bind, cov):
            bind["scale"] = ""
            cands.append((1, bind, cov, bind["dx"]))
    # a scaled match wins over the unscaled one nested inside it
    cands.sort(key=lambda c: c[0])
    found, claimed = [], set()
    for _, bind, cov, out in cands:
        if cov & claimed:
            continue
        my, mg = meta.get(bind["y"]), meta.get(bind["g"])
        if my is None or mg is None or my.scalar or mg.scalar or my.shape != mg.shape or len(my.shape) < 1:
            continue
        if my.dtype != torch.float32 or mg.dtype != torch.float32 or meta[out].shape != my.shape:
            continue
        cov = {c for c in cov if c in live}
        leak = [c for c in cov if c != out and (c in outputs or any(u not in cov for u in users.get(c, [])))]
        if leak:
            continue
        bf, f32 = gemm_use(out, live, users, outputs)
        bind.update({"outv": out, "bf16": str(bf), "f32": str(f32)})
        found.append(Match("softmax_bwd", bind, cov, {"dx": out}))
        claimed |= cov
    return found


def softmax_bwd_step(m: Match, meta: dict[str, Meta]) -> Step:
    b = m.bind
    shape = meta[b["outv"]].shape
    cols = shape[-1]
    rows = math.prod(shape[:-1])
    bf, f32 = b["bf16"] == "True", b["f32"] == "True"
    ins = [b["y"], b["g"]] + ([b["scale"]] if b["scale"] else [])

    def run(env: dict) -> None:
        y = ops.contiguous(ops.cast(env[b["y"]], torch.float32))
        gg = ops.contiguous(ops.cast(env[b["g"]], torch.float32))
        sc = ops.contiguous(ops.cast(env[b["scale"]], torch.float32)) if b["scale"] else None
        dx, dxb = _out_buffers(shape, f32, bf)
        L.call("b200_softmax_bwd_rows", y.data_ptr(), gg.data_ptr(), None if sc is None else sc.data_ptr(),
               None if dx is None else dx.data_ptr(), None if dxb is None else dxb.data_ptr(), rows, cols, ops.stream_ptr())
        _publish(env, b["outv"], dx, dxb)

    label = "softmax_bwd" + ("_scaled" if b["scale"] else "") + ("[bf16]" if bf and not f32 else "")
    return Step([b["outv"]], ins, run, label)


# ----------------------------------------------------------------------------------
# patterns: attention score rows. A Matmul whose only consumer is a (scaled) Softmax, or
# the softmax VJP, runs as one tcgen05 kernel with the row reduction in its epilogue, so
# the fp32 scores (or their gradient) never go to HBM.
# ----------------------------------------------------------------------------------
ATTN_MAX_N, ATTN_MAX_K = 512, 128


def _attn_matmul(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]], outputs: set[str],
                 vid: str, allowed: set[str]) -> Node | None:
    """The Matmul producing ``vid`` when it qualifies: bf16 GEMM policy, rows of at most
    512 columns, K <= 128, and every consumer of ``vid`` inside ``allowed``."""
    mm = live.get(vid)
    if mm is None or _op_name(mm) not in ("Matmul", "BatchMatMul") or len(mm.inputs) != 2 or vid in outputs:
        return None
    if ops.Config.matmul_dtype != "bf16" or any(u not in allowed for u in users.get(vid, [])):
        return None
    mo, ma = meta.get(vid), meta.get(mm.inputs[0])
    if mo is None or ma is None or mo.scalar or ma.scalar or len(mo.shape) < 2 or len(ma.shape) < 2:
        return None
    kw = node_kwargs(mm, "Matmul")
    K = ma.shape[-2] if kw.get("transpose_a") else ma.shape[-1]
    if mo.shape[-1] > ATTN_MAX_N or K > ATTN_MAX_K:
        return None
    return mm


def _mm_operands(mm: Node, env: dict) -> tuple[torch.Tensor, torch.Tensor]:
    kw = node_kwargs(mm, "Matmul")
    a, b = env[mm.inputs[0]], env[mm.inputs[1]]
    if kw.get("transpose_a"):
        a = a.transpose(-1, -2)
    if kw.get("transpose_b"):
        b = b.transpose(-1, -2)
    return a, b


def find_attn_softmax(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                      outputs: set[str]) -> list[Match]:
    found = []
    for m in find_softmax(g, live, meta, users, outputs):
        if m.bind["log"] == "True":
            continue
        mm = _attn_matmul(g, live, meta, users, outputs, m.bind["x"], set(m.covered))
        if mm is None:
            continue
        bind = dict(m.bind)
        bind["mm"] = mm.id
        found.append(Match("attn_softmax", bind, set(m.covered) | {mm.id}, {"y": bind["y"]}))
    return found


def attn_softmax_step(m: Match) -> Step:
    b = m.bind
    mm_id = b["mm"]
    f32, bf = b["f32"] == "True", b["bf16"] == "True"
    ins = list(dict.fromkeys(m.extra_inputs + ([b["scale"]] if b["scale"] else [])))

    def run(env: dict) -> None:
        a, bb = _mm_operands(m.mm_node, env)
        y, yb = ops.gemm_softmax_rows(a, bb, env[b["scale"]] if b["scale"] else None, f32, bf)
        _publish(env, b["y"], y, yb)

    return Step([b["y"]], ins, run, ("scaled_" if b["scale"] else "") + "scores_softmax" + ("[bf16]" if bf and not f32 else ""))


def find_attn_softmax_bwd(g: Graph, live: dict[str, Node], meta: dict[str, Meta], users: dict[str, list[str]],
                          outputs: set[str]) -> list[Match]:
    found = []
    for m in find_softmax_bwd(g, live, meta, users, outputs):
        mm = _attn_matmul(g, live, meta, users, outputs, m.bind["g"], set(m.covered))
        if mm is None:
            continue
        bind = dict(m.bind)
        bind["mm"] = mm.id
        found.append(Match("attn_softmax_bwd", bind, set(m.covered) | {mm.id}, {"dx": bind["outv"]}))
    return found


def attn_softmax_bwd_step(m: Match) -> Step:
    b = m.bind
    f32, bf = b["f32"] == "True", b["bf16"] == "True"
    ins = list(dict.fromkeys(m.extra_inputs + [b["y"]] + ([b["scale"]] if b["scale"] else [])))

    def run(env: dict) -> None:
        a, bb = _mm_operands(m.mm_node, env)
        dx, dxb = ops.gemm_softmax_bwd_rows(a, bb, env[b["y"]], env[b["scale"]] if b["scale"] else None, f32, bf)
        _publish(env, b["outv"], dx, dxb)

    return Step([b["outv"]], ins, run, "scores_softmax_bwd" + ("_scaled" if b["scale"] else "") + ("[bf16]" if bf and not f32 else ""))


# ----------------------------------------------------------------------------------
# elementwise clustering (subsystem 1)
# ----------------------------------------------------------------------------------
EW_UNARY = {"Negative": "NEG", "Exp": "EXP", "Log": "LOG", "Tanh": "TANH", "Sqrt": "SQRT", "Relu": "RELU", "Gelu": "GELU",
            "GELU": "GELU", "Abs": "ABS", "Sigmoid": "SIGMOID", "Erf": "ERF"}
EW_BINARY = {"Add": "ADD", "Subtract": "SUB", "Multiply": "MUL", "TrueDivide": "DIV", "Power": "POW", "Maximum": "MAX",
             "Minimum": "MIN", "Greater": "GT", "GreaterEqual": "GE", "Less": "LT", "Equal": "EQ"}
EW_BOOL_OUT = {"Greater", "GreaterEqual", "Less", "Equal"}


def _is_ew(n: Node) -> bool:
    op = _op_name(n)
    return op in EW_UNARY or op in EW_BINARY or op == "Where"


def _const_value(g: Graph, nid: str) -> float | None:
    n = g.nodes.get(nid)
    if n is not None and n.op_type == "Constant" and isinstance(n.attributes.get("value"), (int, float)):
        return float(n.attributes["value"])
    return None


def cluster_elementwise(g: Graph, order: list[Node], meta: dict[str, Meta], taken: set[str],
                        users: dict[str, list[str]], outputs: set[str]) -> list[list[Node]]:
    """Greedy convex clusters of elementwise nodes that share one output shape."""
    clusters: list[list[Node]] = []
    cid: dict[str, int] = {}
    # anc[c] = set of cluster ids this cluster transitively depends on through non-members
    for n in order:
        if n.id in taken or not _is_ew(n):
            continue
        m = meta.get(n.id)
        if m is None or m.scalar or m.dtype not in (torch.float32, torch.bool):
            continue
        # candidate clusters: those of elementwise producers with the same shape
        cands = []
        for i in n.inputs:
            c = cid.get(i)
            if c is not None and meta[clusters[c][-1].id].shape == m.shape and c not in cands:
                cands.append(c)
        placed = False
        for c in cands:
            members = {x.id for x in clusters[c]}
            # convexity: no input of n may depend on the cluster through a non-member
            if any(_depends_via_outside(g, i, members, taken_meta=meta) for i in n.inputs if i not in members):
                continue
            trial = clusters[c] + [n]
            if _fits(g, trial, meta, users, outputs):
                clusters[c].append(n)
                cid[n.id] = c
                placed = True
                break
        if not placed:
            clusters.append([n])
            cid[n.id] = len(clusters) - 1
    return clusters


def _depends_via_outside(g: Graph, start: str, members: set[str], taken_meta: dict, limit: int = 4096) -> bool:
    """Does value ``start`` (not a member) depend on any member of ``members``?"""
    stack, seen = [start], set()
    while stack and len(seen) < limit:
        v = stack.pop()
        if v in seen:
            continue
        seen.add(v)
        node = g.nodes.get(v)
        if node is None:
            continue
        for i in node.inputs:
            if i in members:
                return True
            stack.append(i)
    return False


def _cluster_io(g: Graph, nodes: list[Node], users: dict[str, list[str]], outputs: set[str]):
    ids = {n.id for n in nodes}
    ext_in: list[str] = []
    for n in nodes:
        for i in n.inputs:
            if i not in ids and _const_value(g, i) is None and i not in ext_in:
                ext_in.append(i)
    outs = [n.id for n in nodes if n.id in outputs or any(u not in ids for u in users.get(n.id, []))]
    return ext_in, outs


def _fits(g: Graph, nodes: list[Node], meta: dict[str, Meta], users, outputs) -> bool:
    ext_in, outs = _cluster_io(g, nodes, users, outputs)
    if len(ext_in) > L.EW_MAX_IN or len(outs) > L.EW_MAX_OUT:
        return False
    n_ins = len(ext_in) + sum(1 + sum(1 for i in n.inputs if _const_value(g, i) is not None) for n in nodes) + len(outs)
    if n_ins > L.EW_MAX_INS:
        return False
    return _alloc_registers(g, nodes, ext_in, outs) is not None


def _alloc_registers(g: Graph, nodes: list[Node], ext_in: list[str], outs: list[str]):
    """Linear-scan register allocation of the program; None if it needs > 16 registers."""
    ids = [n.id for n in nodes]
    last_use: dict[str, int] = {}
    for k, n in enumerate(nodes):
        for i in n.inputs:
            last_use[i] = k
    for o in outs:
        last_use[o] = len(nodes)
    free = list(range(L.EW_MAX_REG))
    reg: dict[str, int] = {}
    prog: list[tuple] = []

    def get(v: str, k: int):
        if v in reg:
            return reg[v]
        cv = _const_value(g, v)
        if not free:
            return None
        r = free.pop(0)
        if cv is not None:
            prog.append(("IMM", r, 0, 0, 0, cv))
            # constants are re-materialised per use; release right away after this node
            return ("tmp", r)
        prog.append(("LOAD", r, ext_in.index(v), 0, 0, 0.0))
        reg[v] = r
        return r

    for k, n in enumerate(nodes):
        srcs = []
        tmps = []
        for i in n.inputs:
            r = get(i, k)
            if r is None:
                return None
            if isinstance(r, tuple):
                tmps.append(r[1])
                r = r[1]
            srcs.append(r)
        # release inputs whose last use is this node (and temporaries)
        for i in set(n.inputs):
            if i in reg and last_use.get(i, -1) <= k and i not in outs:
                free.insert(0, reg.pop(i))
        for t in tmps:
            free.insert(0, t)
        if not free:
            return None
        d = free.pop(0)
        reg[n.id] = d
        op = _op_name(n)
        if op in EW_UNARY:
            prog.append((EW_UNARY[op], d, srcs[0], 0, 0, 0.0))
        elif op in EW_BINARY:
            prog.append((EW_BINARY[op], d, srcs[0], srcs[1], 0, 0.0))
        else:  # Where
            prog.append(("WHERE", d, srcs[0], srcs[1], srcs[2], 0.0))
        if last_use.get(n.id, -1) <= k and n.id not in outs:
            free.insert(0, reg.pop(n.id))
    return prog, {o: reg[o] for o in outs}


def ew_cluster_step(g: Graph, nodes: list[Node], meta: dict[str, Meta], users, outputs, live=None) -> Step:
    ext_in, outs = _cluster_io(g, nodes, users, outputs)
    prog, out_reg = _alloc_registers(g, nodes, ext_in, outs)
    shape = meta[nodes[-1].id].shape
    out_dtypes = [meta[o].dtype for o in outs]
    # float outputs that feed bf16 GEMMs: stored in bf16 (alone, or as a registered twin)
    twins: list[str] = []
    if live is not None:
        for i, o in enumerate(outs):
            if out_dtypes[i] != torch.float32 or len(meta[o].shape) < 2:
                continue
            bf, f32 = gemm_use(o, live, users, outputs)
            if bf and not f32:
                out_dtypes[i] = torch.bfloat16
            elif bf and len(outs) + len(twins) < L.EW_MAX_OUT:
                twins.append(o)
    ops_seq = [(L.EW[name], d, a, b, c, imm) for (name, d, a, b, c, imm) in prog]
    label = "ew[" + ",".join(_op_name(n) for n in nodes) + "]"
    if any(dt == torch.bfloat16 for dt in out_dtypes) or twins:
        label += "[bf16]"

    def run(env: dict) -> None:
        p = ops.Prog()
        vals = []
        for v in ext_in:
            x = env[v]
            if not isinstance(x, torch.Tensor):
                x = ops.full((), float(x))
            vals.append(x)
        p.inputs = vals
        p.ins = list(ops_seq)
        p.nreg = L.EW_MAX_REG
        specs = [(out_reg[o], dt) for o, dt in zip(outs, out_dtypes)] + [(out_reg[o], torch.bfloat16) for o in twins]
        res = p.run(specs, shape)
        for o, r in zip(outs, res):
            env[o] = r
        for o, r in zip(twins, res[len(outs):]):
            ops.register_cast(env[o], r)

    return Step(outs, list(ext_in), run, label)


# ----------------------------------------------------------------------------------
# shape-only operands: BroadcastLike's target, ZerosLike/OnesLike/Numel's operand are
# read for their shape only. With shapes fixed per plan, these edges are not data
# dependencies (dropping them lets e.g. the loss cotangent be computed before the fused
# cross-entropy kernel that produces the forward value it takes the shape of).
# ----------------------------------------------------------------------------------
SHAPE_ONLY = {"BroadcastLike": (1,), "ZerosLike": (0,), "OnesLike": (0,), "Numel": (0,)}


def data_inputs(n: Node) -> list[str]:
    so = SHAPE_ONLY.get(_op_name(n), ())
    return [i for k, i in enumerate(n.inputs) if k not in so]


def shape_only_step(n: Node, meta: dict[str, Meta]) -> Step:
    op = _op_name(n)
    nid = n.id
    if op == "BroadcastLike":
        src = n.inputs[0]
        shape = meta[n.inputs[1]].shape

        def run(env: dict) -> None:
            v = env[src]
            if not isinstance(v, torch.Tensor):
                env[nid] = ops.full(shape, float(v))
            else:
                env[nid] = v if tuple(v.shape) == tuple(shape) else v.expand(shape)

        return Step([nid], [src], run, "BroadcastLike")
    if op in ("ZerosLike", "OnesLike"):
        shape, dtype = meta[n.inputs[0]].shape, meta[n.inputs[0]].dtype
        val = 0.0 if op == "ZerosLike" else 1.0

        def run(env: dict) -> None:
            env[nid] = ops.full(shape, val, dtype)

        return Step([nid], [], run, op)
    numel = float(math.prod(meta[n.inputs[0]].shape)) if not meta[n.inputs[0]].scalar else 1.0

    def run_numel(env: dict) -> None:
        env[nid] = numel

    return Step([nid], [], run_numel, "Numel")


# ----------------------------------------------------------------------------------
# planning
# ----------------------------------------------------------------------------------
def plan_steps(graph: Graph, nodes: list[Node], sample: dict[str, Any]) -> list[Step]:
    meta = record_meta(graph, nodes, sample)
    live = {n.id: n for n in nodes}
    users: dict[str, list[str]] = {}
    for n in nodes:
        for i in data_inputs(n):
            users.setdefault(i, []).append(n.id)
    outputs = set(graph.outputs)
    taken: set[str] = set()
    groups: list[tuple[list[str], Step]] = []

    # 1. patterns
    for m in find_rowfused(graph, live, meta, users):
        if m.covered & taken:
            continue
        produced = set(m.outputs.values())
        leak = [c for c in m.covered if c not in produced and (c in outputs or any(u not in m.covered for u in users.get(c, [])))]
        if leak:
            continue
        eps = float(graph.nodes[m.bind["n"]].attributes.get("eps", graph.nodes[m.bind["n"]].attributes.get("epsilon", 1e-5)))
        groups.append((sorted(m.covered), rowfused_step(m, meta, eps)))
        taken |= m.covered

    # attention score rows: GEMM + (scaled) softmax, GEMM + softmax VJP
    for finder, stepper in ((find_attn_softmax, attn_softmax_step), (find_attn_softmax_bwd, attn_softmax_bwd_step)):
        for m in finder(graph, live, meta, users, outputs):
            if m.covered & taken:
                continue
            m.mm_node = graph.nodes[m.bind["mm"]]
            m.extra_inputs = list(m.mm_node.inputs)
            groups.append((sorted(m.covered), stepper(m)))
            taken |= m.covered

    for m in find_gemm_residual(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), gemm_residual_step(m)))
        taken |= m.covered

    for m in find_gemm_epilogue(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), gemm_epilogue_step(m)))
        taken |= m.covered

    for m in find_conv_relu(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), conv_relu_step(m, graph)))
        taken |= m.covered

    for m in find_conv_dgrad_mask(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), conv_dgrad_mask_step(m, graph)))
        taken |= m.covered

    for m in find_xent(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        bf, f32 = gemm_use(m.outputs["dx"], live, users, outputs)
        groups.append((sorted(m.covered), xent_step(m, meta, bf and not f32)))
        taken |= m.covered

    for m in find_mask_bwd(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), mask_bwd_step(m, meta)))
        taken |= m.covered

    for m in find_ln_bwd(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), ln_bwd_step(m, meta)))
        taken |= m.covered

    for m in find_gelu_bwd(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), gelu_bwd_step(m, meta)))
        taken |= m.covered

    for m in find_softmax_bwd(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), softmax_bwd_step(m, meta)))
        taken |= m.covered

    for m in find_softmax(graph, live, meta, users, outputs):
        if m.covered & taken:
            continue
        groups.append((sorted(m.covered), softmax_step(m, meta)))
        taken |= m.covered

    # GEMMs that write straight into a transposed layout
    for m in find_matmul_transpose(graph, live, meta, users, outputs, taken):
        if m.covered & taken:
            continue
        mm = graph.nodes[m.bind["mm"]]
        st = matmul_transpose_step(m, meta)
        kw = node_kwargs(mm, "Matmul")
        if kw.get("transpose_a") or kw.get("transpose_b"):
            fn = st.fn
            st.fn = lambda env, _fn=fn, _kw=dict(kw): _fn(env, _kw)
        groups.append((sorted(m.covered), st))
        taken |= m.covered

    # LayerNorms whose output feeds bf16 GEMMs also write (or only write) bf16
    for n in nodes:
        if n.id in taken or _op_name(n) != "LayerNorm":
            continue
        mo = meta.get(n.id)
        if mo is None or mo.scalar:
            continue
        bf, f32 = gemm_use(n.id, live, users, outputs)
        if bf:
            groups.append(([n.id], layernorm_step(n, f32)))
            taken.add(n.id)

    # plain matmuls whose result only feeds bf16 GEMMs store bf16
    for n in nodes:
        if n.id in taken or _op_name(n) != "Matmul" or len(n.inputs) != 2:
            continue
        mo = meta.get(n.id)
        if mo is None or mo.scalar or len(mo.shape) < 2:
            continue
        bf, f32 = gemm_use(n.id, live, users, outputs)
        if bf:
            groups.append(([n.id], matmul_step(n, not f32, mo.shape, twin=f32)))
            taken.add(n.id)

    # 2. elementwise clusters
    rest = [n for n in nodes if n.id not in taken]
    for cl in cluster_elementwise(graph, rest, meta, taken, users, outputs):
        if len(cl) == 1:
            mo = meta.get(cl[0].id)
            if mo is None or mo.scalar or mo.dtype != torch.float32 or len(mo.shape) < 2:
                continue
            if not gemm_use(cl[0].id, live, users, outputs)[0]:
                continue
        groups.append(([n.id for n in cl], ew_cluster_step(graph, cl, meta, users, outputs, live)))
        taken |= {n.id for n in cl}

    # constants feeding only fused steps are folded into the programs
    # 3. the rest, one step per node
    for n in nodes:
        if n.id not in taken:
            if n.op_type == "Constant" and all(u in taken for u in users.get(n.id, [])) and n.id not in outputs:
                continue
            if _op_name(n) in SHAPE_ONLY:
                groups.append(([n.id], shape_only_step(n, meta)))
            else:
                groups.append(([n.id], node_step(n)))
    steps = _schedule(groups)
    _conv_copy_only(steps, outputs, meta, graph)
    return steps


def _schedule(groups: list[tuple[list[str], Step]]) -> list[Step]:
    """Topological order of the condensed step graph."""
    owner: dict[str, int] = {}
    for k, (members, st) in enumerate(groups):
        for v in members:
            owner[v] = k
        for v in st.outputs:
            owner[v] = k
    deps = []
    for k, (_, st) in enumerate(groups):
        deps.append({owner[i] for i in st.inputs if i in owner and owner[i] != k})
    order, state = [], [0] * len(groups)
    for root in range(len(groups)):
        if state[root]:
            continue
        stack = [(root, iter(sorted(deps[root])))]
        state[root] = 1
        while stack:
            k, it = stack[-1]
            nxt = next(it, None)
            if nxt is None:
                stack.pop()
                state[k] = 2
                order.append(groups[k][1])
            elif state[nxt] == 0:
                state[nxt] = 1
                stack.append((nxt, iter(sorted(deps[nxt]))))
            elif state[nxt] == 1:
                raise RuntimeError("fusion produced a cyclic step graph")
    return order
