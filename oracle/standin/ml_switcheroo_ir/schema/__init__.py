"""Stand-in ``ml_switcheroo_ir.schema`` (usage-derived)."""
