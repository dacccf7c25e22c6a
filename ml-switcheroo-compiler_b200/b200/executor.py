"""Whole-graph execution for ``execute_graph`` / ``compile_graph``.

A ``Plan`` is built once per (graph, input shapes/dtypes):
  1. dependency order of all nodes (``Graph.topo_order``, the same order contract as
     ``interpreter/evaluator.py:293``);
  2. dead-node pruning: only nodes that reach a graph output run (the reference
     interpreter evaluates every node, ``evaluator.py:296-297``; dead gradients such as
     dX of the first layer are skipped here);
  3. fusion: ``fusion.plan_steps`` groups nodes into fused GPU steps (whole-row
     kernels, GEMM epilogues, elementwise programs); every other node is one step;
  4. liveness: each intermediate is released after its last consumer step.

``Plan.run`` launches the steps on the current CUDA stream. ``CompiledGraph`` wraps a
plan with static input/output buffers and replays it as one captured CUDA graph.
"""

from __future__ import annotations

from typing import Any, Callable

import torch

from . import ops
from .errors import UnimplementedMathError
from .graph import Graph, Node, coerce

ALIASES = ops.ALIASES


def node_kwargs(node: Node, target: str) -> dict[str, Any]:
    """Attribute -> kwargs rules of ``_prepare_node_kwargs`` (evaluator.py:793-832)."""
    kw = {k: v for k, v in node.attributes.items() if k not in ("var_name", "is_parameter", "param_name")}
    if target == "Checkpoint":
        return {}
    conv_like = {"Conv", "Conv1D", "Conv2D", "Conv3D", "ConvTranspose", "ConvTranspose2D", "MaxPool2D", "AvgPool2D", "StridedSlice"}
    if "strides" in kw and target not in conv_like:
        kw.pop("strides")
    if node.shape_metadata:
        mt = tuple(int(d) if isinstance(d, int) else str(d) for d in node.shape_metadata)
        if target in ("Expand", "BroadcastTo", "ConstantOfShape", "Zeros", "Ones", "Full") and "shape" not in kw:
            kw["shape"] = mt
        if target == "Reshape" and "newshape" not in kw:
            kw["newshape"] = mt
    return kw


class Step:
    """A unit of GPU work producing one or more environment values."""

    def __init__(self, outputs: list[str], inputs: list[str], fn: Callable[[dict], None], label: str) -> None:
        self.outputs = outputs
        self.inputs = inputs
        self.fn = fn
        self.label = label

    def __repr__(self) -> str:  # pragma: no cover
        return f"Step({self.label} -> {len(self.outputs)} values)"


def node_step(node: Node) -> Step:
    """One graph node evaluated by its per-op kernel (the ``execute_op`` path)."""
    op = node.op_type
    nid = node.id
    if op == "Constant":
        val = node.attributes["value"]

        def run_const(env: dict) -> None:
            env[nid] = val if isinstance(val, (int, float)) else ops.to_device(val)

        return Step([nid], [], run_const, "Constant")
    if op == "Output":
        ins = list(node.inputs)

        def run_out(env: dict) -> None:
            vals = [env[i] for i in ins if i]
            env[nid] = vals[0] if len(vals) == 1 else tuple(vals)

        return Step([nid], ins, run_out, "Output")
    if op == "Identity":
        ins = list(node.inputs)

        def run_id(env: dict) -> None:
            env[nid] = env[ins[0]] if ins else None

        return Step([nid], ins, run_id, "Identity")
    if op == "Recompute":
        # _evaluate_recompute_node (evaluator.py:720-735): the original op with its attributes
        orig = ALIASES.get(str(node.attributes.get("original_op", op)), str(node.attributes.get("original_op", op)))
        oa = node.attributes.get("original_attrs", {})
        resolved = Node(nid, orig, list(node.inputs), dict(oa) if isinstance(oa, dict) else {}, node.shape_metadata)
        st = node_step(resolved)
        st.label = f"Recompute({st.label})"
        return st
    target = ALIASES.get(op, op)
    ins = list(node.inputs)
    if target in ("Slice", "GetItem", "IndexPut", "SetItem"):
        return _indexing_step(node, target)
    if target == "Checkpoint":
        return _checkpoint_step(node)
    fn = ops.OPS.get(target)
    if fn is None:
        raise UnimplementedMathError(f"Operation {op} is not implemented in the b200 backend.")
    kwargs = node_kwargs(node, target)

    def run_op(env: dict) -> None:
        env[nid] = fn(*[env[i] for i in ins], **kwargs)

    return Step([nid], ins, run_op, target)


def _indexing_step(node: Node, target: str) -> Step:
    """Slice / GetItem / IndexPut / SetItem (evaluator.py:428-508) on device values."""
    from . import indexing

    nid, ins = node.id, list(node.inputs)
    kwargs = node_kwargs(node, target)
    cache: dict = {}  # device index arrays of the key, uploaded on the first (eager) run
    if target == "Slice":

        def run(env: dict) -> None:
            env[nid] = indexing.slice_node(env[ins[0]], kwargs, cache)

    elif target == "GetItem":
        key = indexing.parse_key(kwargs.get("key"))

        def run(env: dict) -> None:
            env[nid] = indexing.get_item(env[ins[0]], key, cache)

    else:
        key = indexing.parse_key(kwargs.get("key", kwargs.get("index", 0)))

        def run(env: dict) -> None:
            env[nid] = indexing.index_put(env[ins[0]], key, env[ins[1]])

    return Step([nid], ins, run, target)


def _subgraph_of(node: Node) -> Any:
    sg = None
    subs = getattr(node, "subgraphs", None) or {}
    if isinstance(subs, dict):
        sg = subs.get("body") or subs.get("subgraph")
    return sg if sg is not None else node.attributes.get("subgraph")


def _checkpoint_step(node: Node) -> Step:
    """_handle_checkpoint (evaluator.py:511-545): the node's forward subgraph evaluated on
    its inputs by a nested plan (fused like any graph); one output, or a tuple."""
    raw = _subgraph_of(node)
    if raw is None or not hasattr(raw, "inputs") and not (isinstance(raw, dict) and "inputs" in raw):
        raise AttributeError("Checkpoint node is missing a valid subgraph")
    sub = coerce(raw)
    runner = GraphRunner(sub)
    nid, ins = node.id, list(node.inputs)
    sg_in = list(sub.inputs)

    def run(env: dict) -> None:
        res = runner(dict(zip(sg_in, [env[i] for i in ins])))
        env[nid] = res[sub.outputs[0]] if len(sub.outputs) == 1 else tuple(res[o] for o in sub.outputs)

    return Step([nid], ins, run, "Checkpoint")


class Plan:
    def __init__(self, graph: Graph, sample: dict[str, Any], fuse: bool = True) -> None:
        self.graph = graph
        order = graph.topo_order()
        outs = set(graph.outputs)
        needed: set[str] = set()
        stack = list(outs)
        while stack:
            nid = stack.pop()
            if nid in needed or nid not in graph.nodes:
                continue
            needed.add(nid)
            stack.extend(graph.nodes[nid].inputs)
        self.live_nodes = [n for n in order if n.id in needed and n.op_type != "Input"]
        self.input_ids = [n.id for n in order if n.op_type == "Input" and n.id in needed]
        if fuse:
            from .fusion import plan_steps

            self.steps = plan_steps(graph, self.live_nodes, sample)
        else:
            self.steps = [node_step(n) for n in self.live_nodes]
        # release each value after its last consumer step (graph outputs are kept)
        last: dict[str, int] = {}
        for i, st in enumerate(self.steps):
            for v in st.inputs:
                last[v] = i
        self.free_after: list[list[str]] = [[] for _ in self.steps]
        for v, i in last.items():
            if v not in outs and v not in self.input_ids:
                self.free_after[i].append(v)

    def begin(self, inputs: dict[str, Any]) -> dict[str, Any]:
        """The environment of one run: initializers and inputs (missing inputs raise)."""
        env: dict[str, Any] = dict(self.graph.initializers)
        env.update(inputs)
        for i in self.input_ids:
            if i not in env:
                raise ValueError(f"Missing input value for node '{i}'")  # environment.py:33-48
        ops.clear_cast_cache()
        return env

    def run_steps(self, env: dict[str, Any], lo: int, hi: int, capture: dict | None = None) -> None:
        """Steps [lo, hi) of a run begun with ``begin``; values die after their last use.
        ``capture`` (id -> None) receives the values of those ids as they are produced."""
        for st, dead in zip(self.steps[lo:hi], self.free_after[lo:hi]):
            st.fn(env)
            if capture is not None:
                for o in st.outputs:
                    if o in capture and o in env:
                        capture[o] = env[o]
            for v in dead:
                env.pop(v, None)

    def finish(self, env: dict[str, Any]) -> dict[str, Any]:
        ops.clear_cast_cache()
        res = {}
        for oid in self.graph.outputs:
            if oid not in env:
                raise RuntimeError(f"Output node '{oid}' was never evaluated.")  # evaluator.py:301-303
            res[oid] = env[oid]
        return res

    def run(self, inputs: dict[str, Any], capture: dict | None = None) -> dict[str, Any]:
        env = self.begin(inputs)
        try:
            self.run_steps(env, 0, len(self.steps), capture)
        finally:
            ops.clear_cast_cache()
        return self.finish(env)

    def last_use(self) -> dict[str, int]:
        """Index of the last step that produces or reads each value."""
        last: dict[str, int] = {}
        for i, st in enumerate(self.steps):
            for v in list(st.outputs) + list(st.inputs):
                last[v] = i
        return last

    def describe(self) -> list[str]:
        return [s.label for s in self.steps]


def _signature(inputs: dict[str, Any]) -> tuple:
    sig = []
    for k in sorted(inputs):
        v = inputs[k]
        if isinstance(v, torch.Tensor):
            sig.append((k, tuple(v.shape), str(v.dtype)))
        else:
            sig.append((k, type(v).__name__))
    return tuple(sig)


class GraphRunner:
    """Caches one Plan per input signature for a graph."""

    def __init__(self, graph: Any, fuse: bool = True) -> None:
        self.graph = coerce(graph)
        self.fuse = fuse
        self.plans: dict[tuple, Plan] = {}

    def device_inputs(self, inputs: dict[str, Any]) -> dict[str, Any]:
        return {k: (ops.to_device(v) if not isinstance(v, (int, float)) else v) for k, v in inputs.items()}

    def plan_for(self, dinputs: dict[str, Any]) -> Plan:
        sig = _signature(dinputs)
        p = self.plans.get(sig)
        if p is None:
            p = Plan(self.graph, dinputs, fuse=self.fuse)
            self.plans[sig] = p
        return p

    def __call__(self, inputs: dict[str, Any]) -> dict[str, Any]:
        d = self.device_inputs(inputs)
        return self.plan_for(d).run(d)


class CompiledGraph:
    """Static-buffer executable: inputs are copied into fixed device buffers and the
    whole plan replays as one CUDA graph (launch overhead paid once per step)."""

    def __init__(self, graph: Any, fuse: bool = True, use_cuda_graph: bool = True) -> None:
        self.runner = GraphRunner(graph, fuse=fuse)
        self.use_cuda_graph = use_cuda_graph
        self.static_in: dict[str, torch.Tensor] | None = None
        self.static_out: dict[str, Any] | None = None
        self.cuda_graph: torch.cuda.CUDAGraph | None = None
        self.sig: tuple | None = None

    def _capture(self, d: dict[str, Any]) -> None:
        plan = self.runner.plan_for(d)
        self.static_in = {k: (ops.copy(v) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
        # warm up on a side stream (allocations settle, one-time attribute calls happen)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            plan.run(self.static_in)
        torch.cuda.current_stream().wait_stream(s)
        if self.use_cuda_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.static_out = plan.run(self.static_in)
            self.cuda_graph = g
        self.sig = _signature(d)

    def __call__(self, inputs: dict[str, Any]) -> dict[str, Any]:
        if self.static_in is not None and self.sig == _signature(inputs):
            # the captured signature: host tensors (pinned: asynchronous H2D) and device
            # tensors go straight into the static buffers, with no intermediate copy
            for k, v in inputs.items():
                dst = self.static_in[k]
                if isinstance(dst, torch.Tensor) and v is not dst:
                    dst.copy_(v, non_blocking=True)
            if self.cuda_graph is not None:
                self.cuda_graph.replay()
                return self.static_out
            return self.runner.plan_for(self.static_in).run(self.static_in)
        d = self.runner.device_inputs(inputs)
        if self.sig != _signature(d):
            self._capture(d)
        for k, v in d.items():
            dst = self.static_in[k]
            # callers that fill the static buffers in place (inputs already resident)
            # pass them back unchanged: nothing to copy
            if isinstance(dst, torch.Tensor) and v is not dst:
                dst.copy_(v, non_blocking=True)  # device-to-device copy engine transfer
        if self.cuda_graph is not None:
            self.cuda_graph.replay()
            return self.static_out
        return self.runner.plan_for(self.static_in).run(self.static_in)
