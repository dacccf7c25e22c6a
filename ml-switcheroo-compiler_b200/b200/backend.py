"""The ``b200`` backend class: the drop-in boundary of the reference's backend plugin API.

Registered under the name ``"b200"`` with the reference's ``register_backend``
(``backends/registry.py:426-448``). Members mirror what the interpreter and the grad
API call on a backend:

* ``execute_op(op_type, *args, **kwargs)`` - one op (``interpreter/evaluator.py:593``);
* ``array`` / ``asarray`` / ``zeros`` / ``item`` / ``get_module``
  (``backends/generator_mixins.py:107-188``);
* ``execute_graph(graph, inputs)`` and ``compile_graph(graph)`` - the optional
  whole-graph hooks (``grad/api.py:38-68``, used at ``grad/api.py:207-211`` and
  ``grad/jvp_vjp.py:524-528``).

Values are ``torch.Tensor`` on the current CUDA device (they provide ``.shape``,
``__getitem__``, ``__setitem__`` and ``.item()``, which the interpreter uses directly).
Unknown ops raise ``UnimplementedMathError``; there is no CPU fallback.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any, Callable, Mapping

import torch

from . import ops
from .executor import CompiledGraph, GraphRunner
from .graph import coerce, content_key


class B200Backend:
    """Backend plugin for NVIDIA B200 (sm_100a)."""

    name = "b200"
    # runners (one plan per input signature each) keyed by the graph's content: node ids,
    # op types, inputs, attributes, shape metadata, graph inputs / outputs. The reference
    # builds a new LogicalGraph object per backward() call and its graphs are unhashable,
    # so identity keys would miss every time and could alias a dead graph's plan to a new
    # graph that reuses its address; content keys do neither. Least recently used first
    # out beyond MAX_RUNNERS.
    MAX_RUNNERS = 16
    _runners: "OrderedDict[str, GraphRunner]" = OrderedDict()

    # ---- per-op path -------------------------------------------------------------
    @classmethod
    def execute_op(cls, op_type: str, *args: Any, **kwargs: Any) -> Any:
        return ops.execute_op(op_type, *args, **kwargs)

    @classmethod
    def array(cls, data: Any, dtype: Any = None) -> Any:
        if isinstance(data, (int, float, bool)) and dtype is None:
            return ops.to_device(torch.tensor(float(data), dtype=torch.float32))
        return ops.to_device(data)

    @classmethod
    def asarray(cls, data: Any) -> Any:
        return data if isinstance(data, torch.Tensor) and data.is_cuda else ops.to_device(data)

    @classmethod
    def zeros(cls, shape: tuple[int, ...]) -> Any:
        return ops.full(tuple(shape), 0.0)

    @classmethod
    def item(cls, data: Any) -> float:
        return float(data.item()) if isinstance(data, torch.Tensor) else float(data)

    @classmethod
    def get_module(cls) -> Any:
        return ops

    # ---- weight I/O hooks of the reference's format classes -------------------------
    @classmethod
    def from_buffer(cls, buffer: bytes, dtype: str, shape: Any) -> Any:
        """serialization/formats/safetensors.py:118-129: one tensor's bytes -> HBM."""
        from . import weights

        return weights.from_buffer(buffer, dtype, shape)

    @classmethod
    def load_npz(cls, filepath: str) -> Any:
        """serialization/formats/npz.py:84-93: the archive's arrays -> HBM."""
        from . import weights

        return weights.load_npz(filepath)

    @classmethod
    def save_npz(cls, weights_np: Any, filepath: str) -> None:
        """serialization/formats/npz.py:105-108: device tensors -> the reference's npz layout."""
        from . import weights

        weights.save_npz(weights_np, filepath)

    # ---- whole-graph hooks -----------------------------------------------------------
    @classmethod
    def _runner(cls, graph: Any) -> GraphRunner:
        g = coerce(graph)
        key = content_key(g)
        r = cls._runners.get(key)
        if r is None:
            r = GraphRunner(g)
            cls._runners[key] = r
            while len(cls._runners) > cls.MAX_RUNNERS:
                cls._runners.popitem(last=False)
        else:
            cls._runners.move_to_end(key)
        return r

    @classmethod
    def execute_graph(cls, graph: Any, inputs: Mapping[str, Any]) -> dict[str, Any]:
        """Run a whole fwd+bwd graph: fused kernels, dead nodes pruned. The returned
        tensors are fresh per call (the caller owns them)."""
        return cls._runner(graph)(dict(inputs))

    @classmethod
    def compile_graph(cls, graph: Any, alias_outputs: bool = False) -> Callable[[Mapping[str, Any]], Mapping[str, Any]]:
        """A replayable executable: static input buffers plus one captured CUDA graph per
        input signature. Host inputs (pinned: asynchronous) are copied straight into the
        static buffers.

        Each call returns fresh output tensors (device copies of the graph's static
        outputs), so results held from an earlier call are never overwritten, as with
        ``execute_graph``. ``alias_outputs=True`` skips that copy: every call then returns
        the same static output tensors, which the next call overwrites in place."""
        cg = CompiledGraph(graph)
        if alias_outputs:
            return lambda inputs: cg(dict(inputs))

        def run(inputs: Mapping[str, Any]) -> dict[str, Any]:
            out = cg(dict(inputs))
            return {k: (ops.copy(v) if isinstance(v, torch.Tensor) else v) for k, v in out.items()}

        return run


def register() -> type[B200Backend]:
    """Register ``B200Backend`` as backend ``"b200"`` with the reference registry
    (call once, before ``config.backend = "b200"``)."""
    from ml_switcheroo_compiler.backends.registry import register_backend

    register_backend("b200")(B200Backend)
    return B200Backend
