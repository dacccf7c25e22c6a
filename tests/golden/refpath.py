"""Locate the reference's source tree for the fixture generators in this folder.

The generators import the reference package (``ml_switcheroo_compiler``) read-only. Its
``src`` directory comes from ``--reference-src PATH`` on the command line or the
``ML_SWITCHEROO_REFERENCE_SRC`` environment variable; nothing is assumed about where the
reference is checked out. The usage-derived ``ml_switcheroo_ir`` stand-in under
``oracle/standin`` goes on ``sys.path`` ahead of it.
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
ENV = "ML_SWITCHEROO_REFERENCE_SRC"


def reference_src(argv: list[str] | None = None) -> str:
    """The reference ``src`` directory: ``--reference-src PATH`` (removed from ``argv``)
    or ``$ML_SWITCHEROO_REFERENCE_SRC``."""
    argv = sys.argv if argv is None else argv
    path = None
    if "--reference-src" in argv:
        i = argv.index("--reference-src")
        if i + 1 >= len(argv):
            raise SystemExit("--reference-src needs a path")
        path = argv[i + 1]
        del argv[i : i + 2]
    path = path or os.environ.get(ENV)
    if not path:
        raise SystemExit(f"give the reference's src directory with --reference-src PATH or ${ENV}")
    if not os.path.isdir(os.path.join(path, "ml_switcheroo_compiler")):
        raise SystemExit(f"{path} does not contain the ml_switcheroo_compiler package")
    os.environ[ENV] = path  # later imports in this process (one generator importing another) find it
    return path


def add_reference_to_path(argv: list[str] | None = None) -> str:
    """Put the stand-in and the reference source on ``sys.path``; returns the source path."""
    src = reference_src(argv)
    for p in (src, os.path.join(REPO, "oracle", "standin")):
        if p not in sys.path:
            sys.path.insert(0, p)
    return src
