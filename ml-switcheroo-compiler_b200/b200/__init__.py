"""b200: B200-native (sm_100a) execution backend for ml-switcheroo-compiler fwd+bwd graphs.

``B200Backend`` is the plugin class (``register()`` adds it to the reference's backend
registry as ``"b200"``). Kernels live in ``libb200.so`` (C ABI: ``include/b200.h``),
loaded through ``b200._lib``; there is no CPU fallback.
"""

from .backend import B200Backend, register
from .errors import BackendNotSupportedError, CompilationError, UnimplementedMathError

__all__ = ["B200Backend", "BackendNotSupportedError", "CompilationError", "UnimplementedMathError", "register"]
