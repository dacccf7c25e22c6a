"""Stand-in ``ml_switcheroo_ir.schema.ghost`` (usage-derived)."""

from pydantic import BaseModel, ConfigDict


class ExtendedGhostRef(BaseModel):
    """Opaque reference record (not on the execution path)."""

    model_config = ConfigDict(extra="allow")
