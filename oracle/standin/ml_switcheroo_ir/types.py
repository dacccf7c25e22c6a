"""Stand-in ``ml_switcheroo_ir.types`` (usage-derived; see package docstring)."""

from __future__ import annotations

import typing
from enum import Enum

from pydantic import BaseModel, ConfigDict


class DType(str, Enum):
    """Canonical dtype names read by ``core/dtype.py:93-121``."""

    float64 = "float64"
    float32 = "float32"
    float16 = "float16"
    bfloat16 = "bfloat16"
    float8_e4m3b11fnuz = "float8_e4m3b11fnuz"
    float8_e4m3fn = "float8_e4m3fn"
    fp8_e4m3fnuz = "float8_e4m3fnuz"
    float8_e5m2 = "float8_e5m2"
    fp8_e5m2fnuz = "float8_e5m2fnuz"
    complex64 = "complex64"
    complex128 = "complex128"
    int64 = "int64"
    int32 = "int32"
    int16 = "int16"
    int8 = "int8"
    int4 = "int4"
    uint64 = "uint64"
    uint32 = "uint32"
    uint16 = "uint16"
    uint8 = "uint8"
    uint4 = "uint4"
    bool = "bool"
    string = "string"
    object = "object"


class TensorSpec(BaseModel):
    """Shape + dtype of a graph input."""

    model_config = ConfigDict(extra="allow", arbitrary_types_allowed=True)
    shape: typing.Any = None
    dtype: typing.Any = None
