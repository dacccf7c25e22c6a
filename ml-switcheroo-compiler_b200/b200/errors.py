"""Exception types of the backend boundary.

When the reference package is importable, its own classes are used
(``core/errors.py:86`` UnimplementedMathError, ``:106`` CompilationError,
``:122`` BackendNotSupportedError), so callers of the plugin catch exactly what they
catch for the numpy backend. Otherwise same-named local classes stand in.
"""

from __future__ import annotations

try:  # pragma: no cover - depends on the environment
    from ml_switcheroo_compiler.core.errors import (  # type: ignore
        BackendNotSupportedError,
        CompilationError,
        UnimplementedMathError,
    )
except Exception:  # noqa: BLE001

    class UnimplementedMathError(NotImplementedError):
        """An op without a b200 kernel (the reference raises this for unknown ops)."""

    class CompilationError(RuntimeError):
        """Malformed graph (e.g. a cycle)."""

    class BackendNotSupportedError(RuntimeError):
        """A dtype / feature combination the backend does not support."""


__all__ = ["BackendNotSupportedError", "CompilationError", "UnimplementedMathError"]
