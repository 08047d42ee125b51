"""Typed metadata filters pushed down to the device.

``MetadataFilter`` is the filter language of crates/proxima-server/src/filter.rs
(a conjunction of per-field conditions: a bare scalar is equality; operators
eq, ne, gt, gte, lt, lte, in, exists; no type coercion). ``parse`` follows
filter.rs:122-200 and ``accepts`` filter.rs:216-256 (the host form, what the
reference evaluates per candidate). ``compile`` turns it into the
``pxc_condition`` list the native library evaluates per slot over
``DeviceColumns`` (typed device columns of the fields the filters read), so a
filtered batch search needs no per-slot host pass.
"""
from __future__ import annotations

import ctypes as C
import math
import struct

import numpy as np

from . import _native as N
from .errors import Configuration

VALUE_ABSENT, VALUE_TEXT, VALUE_INT, VALUE_FLOAT, VALUE_BOOL = 0, 1, 2, 3, 4
EQ, NE, GT, GE, LT, LE, IN, EXISTS = range(8)
_OPS = {"eq": EQ, "ne": NE, "gt": GT, "gte": GE, "lt": LT, "lte": LE}


def metadata_value(v):
    """A Python metadata value as MetadataValue (crates/proxima-core/src/metadata.rs:21-31):
    (tag, payload) with no coercion; None is absent."""
    if v is None:
        return VALUE_ABSENT, None
    if isinstance(v, bool):
        return VALUE_BOOL, bool(v)
    if isinstance(v, (int, np.integer)):
        return VALUE_INT, int(v)
    if isinstance(v, (float, np.floating)):
        return VALUE_FLOAT, float(v)
    if isinstance(v, str):
        return VALUE_TEXT, v
    raise TypeError(f"unsupported metadata value {v!r}")


def _json_number(v):
    """A JSON number as filter.rs reads it: integral and below 9.007e15 in magnitude -> Int, else Float."""
    f = float(v)
    if math.isfinite(f) and f == math.floor(f) and abs(f) < 9.007e15:
        return VALUE_INT, int(f)
    return VALUE_FLOAT, f


def _scalar(field, v):
    """filter.rs scalar_value."""
    if isinstance(v, bool):
        return VALUE_BOOL, v
    if isinstance(v, str):
        return VALUE_TEXT, v
    if isinstance(v, (int, float, np.integer, np.floating)):
        return _json_number(v)
    raise Configuration("filter", field, f"filter on '{field}' needs a string, number or boolean")


def _number(field, v):
    """filter.rs number."""
    if isinstance(v, bool) or not isinstance(v, (int, float, np.integer, np.floating)):
        raise Configuration("filter", field, f"range filter on '{field}' needs a number")
    return _json_number(v)


def _total_key(f: float) -> int:
    b = struct.unpack("<q", struct.pack("<d", f))[0]
    return b ^ ((b >> 63) & 0x7FFFFFFFFFFFFFFF)


def _compare(bound, value):
    """Number::compare (filter.rs:81-97): -1 / 0 / 1, or None when the pairing is not comparable."""
    bt, bv = bound
    vt, vv = value
    if bt == VALUE_INT and vt == VALUE_INT:
        return (vv > bv) - (vv < bv)
    if vt == VALUE_FLOAT and bt in (VALUE_FLOAT, VALUE_INT):
        a, b = _total_key(vv), _total_key(float(bv))
        return (a > b) - (a < b)
    return None


def _equal(a, b) -> bool:
    return a[0] == b[0] and a[1] == b[1]


class MetadataFilter:
    """A compiled conjunction of (field, operator, operand) conditions, sorted by field."""

    def __init__(self, conditions):
        self.conditions = conditions

    @classmethod
    def parse(cls, obj: dict) -> "MetadataFilter":
        """MetadataFilter::parse (filter.rs:122-200) from the JSON object as a Python dict."""
        if not isinstance(obj, dict):
            raise Configuration("filter", 0, "filter must be an object")
        conds = []
        for field, cond in obj.items():
            if isinstance(cond, dict):
                if not cond:
                    raise Configuration("filter", field, f"filter on '{field}' has no operators")
                for op, operand in cond.items():
                    if op in ("eq", "ne"):
                        conds.append((field, _OPS[op], _scalar(field, operand)))
                    elif op in ("gt", "gte", "lt", "lte"):
                        conds.append((field, _OPS[op], _number(field, operand)))
                    elif op == "in":
                        if not isinstance(operand, (list, tuple)):
                            raise Configuration("filter", field, f"'in' on '{field}' needs an array")
                        if not operand:
                            raise Configuration("filter", field, f"'in' on '{field}' has an empty list")
                        conds.append((field, IN, [_scalar(field, x) for x in operand]))
                    elif op == "exists":
                        if not isinstance(operand, bool):
                            raise Configuration("filter", field, f"'exists' on '{field}' needs true or false")
                        conds.append((field, EXISTS, operand))
                    else:
                        raise Configuration("filter", field, f"unknown operator '{op}' on '{field}'")
            else:
                conds.append((field, EQ, _scalar(field, cond)))
        conds.sort(key=lambda c: c[0])
        return cls(conds)

    def fields(self) -> list[str]:
        return sorted({c[0] for c in self.conditions})

    def is_empty(self) -> bool:
        return not self.conditions

    def accepts(self, _id: int, metadata: dict) -> bool:
        """Filter::accepts (filter.rs:216-256)."""
        for field, op, operand in self.conditions:
            raw = metadata.get(field) if metadata else None
            value = metadata_value(raw)
            if op == EXISTS:
                held = (value[0] != VALUE_ABSENT) == operand
            elif value[0] == VALUE_ABSENT:
                held = False
            elif op == EQ:
                held = _equal(value, operand)
            elif op == NE:
                held = not _equal(value, operand)
            elif op == IN:
                held = any(_equal(value, o) for o in operand)
            else:
                o = _compare(operand, value)
                held = o is not None and ((op == GT and o == 1) or (op == GE and o >= 0) or
                                          (op == LT and o == -1) or (op == LE and o <= 0))
            if not held:
                return False
        return True

    __call__ = accepts

    def compile(self, cols: "DeviceColumns"):
        """The pxc_condition / pxc_operand arrays of this filter over `cols`."""
        conds = (N.PxcCondition * max(1, len(self.conditions)))()
        operands = []
        for i, (field, op, operand) in enumerate(self.conditions):
            c = conds[i]
            c.column = cols.column(field)
            c.op = op
            if op == EXISTS:
                c.tag, c.value = 0, int(operand)
            elif op == IN:
                c.tag, c.count, c.value = 0, len(operand), len(operands)
                operands.extend(cols.payload(o) for o in operand)
            else:
                c.tag, c.value = cols.payload(operand)
        ops = (N.PxcOperand * max(1, len(operands)))()
        for j, (t, v) in enumerate(operands):
            ops[j].tag, ops[j].value = t, v
        return conds, len(self.conditions), ops, len(operands)


class DeviceColumns:
    """Typed device columns (pxc_columns): one MetadataValue per slot per field.
    Text values are coded through a per-instance dictionary (equal strings, equal codes)."""

    UNSEEN_TEXT = -1  # the code of a filter string no slot holds

    def __init__(self, ctx):
        self.ctx = ctx
        self.lib = N.load()
        h = N.vp()
        N.call("pxc_columns_create", ctx.handle, C.byref(h))
        self.handle = h
        self._fields: dict[str, int] = {}
        self._codes: dict[str, int] = {}

    def column(self, field: str) -> int:
        if field not in self._fields:
            self._fields[field] = len(self._fields)
        return self._fields[field]

    def payload(self, tv, assign: bool = False):
        tag, v = tv
        if tag == VALUE_TEXT:
            if v not in self._codes:
                if not assign:
                    return tag, self.UNSEEN_TEXT
                self._codes[v] = len(self._codes)
            return tag, self._codes[v]
        if tag == VALUE_FLOAT:
            return tag, struct.unpack("<q", struct.pack("<d", v))[0]
        if tag == VALUE_BOOL:
            return tag, int(v)
        if tag == VALUE_ABSENT:
            return tag, 0
        return tag, int(v)

    def set_values(self, field: str, values, slot_begin: int = 0) -> None:
        """Slots slot_begin.. of `field`: Python metadata values (None = absent)."""
        n = len(values)
        tags = np.zeros(n, np.uint8)
        pay = np.zeros(n, np.int64)
        for i, v in enumerate(values):
            tags[i], pay[i] = self.payload(metadata_value(v), assign=True)
        N.call("pxc_columns_set", self.handle, self.column(field), N.ptr(tags), N.ptr(pay), slot_begin, n)

    def truncate(self, nslots: int) -> None:
        N.call("pxc_columns_truncate", self.handle, nslots)

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.pxc_columns_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
