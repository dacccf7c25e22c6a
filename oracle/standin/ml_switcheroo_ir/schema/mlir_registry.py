"""Stand-in ``ml_switcheroo_ir.schema.mlir_registry`` (usage-derived)."""

MLIR_REGISTRY: dict = {}
