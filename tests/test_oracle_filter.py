"""The metadata filter language (crates/proxima-server/src/filter.rs) on the host:
the product's MetadataFilter (parse + accepts, the form compiled to the device)
and the oracle's restatement, both pinned by the reference's own filter tests
(filter.rs:268-445) and agreeing with each other on randomised metadata."""
import math
import random

import pytest

from oracle import pxo
from proxima_b200.errors import Configuration
from proxima_b200.filters import MetadataFilter

KATS = [  # (filter, metadata, expected) from filter.rs's tests
    ({}, {}, True),
    ({"lang": "en", "year": 2024, "public": True}, {"lang": "en", "year": 2024, "public": True}, True),
    ({"lang": "en", "year": 2024, "public": True}, {"lang": "fr", "year": 2024, "public": True}, False),
    ({"a": 1, "b": 2}, {"a": 1}, False),
    ({"a": 1, "b": 2}, {"a": 1, "b": 2}, True),
    ({"year": {"gte": 2020, "lt": 2025}}, {"year": 2019}, False),
    ({"year": {"gte": 2020, "lt": 2025}}, {"year": 2020}, True),
    ({"year": {"gte": 2020, "lt": 2025}}, {"year": 2024}, True),
    ({"year": {"gte": 2020, "lt": 2025}}, {"year": 2025}, False),
    ({"score": {"gt": 0.5}}, {"score": 0.9}, True),
    ({"score": {"gt": 0.5}}, {"score": 9}, False),
    ({"score": {"gte": 1}}, {"score": 1.5}, True),
    ({"score": {"gte": 1}}, {"score": 0.5}, False),
    ({"status": {"in": ["a", "b"]}, "draft": {"ne": True}}, {"status": "a", "draft": False}, True),
    ({"status": {"in": ["a", "b"]}, "draft": {"ne": True}}, {"status": "c", "draft": False}, False),
    ({"status": {"in": ["a", "b"]}, "draft": {"ne": True}}, {"status": "a", "draft": True}, False),
    ({"x": 1}, {}, False),
    ({"x": {"ne": 1}}, {}, False),
    ({"x": {"gt": 0}}, {}, False),
    ({"x": {"in": [1, 2]}}, {}, False),
    ({"x": {"exists": True}}, {}, False),
    ({"x": {"exists": False}}, {}, True),
]


@pytest.mark.parametrize("flt,meta,expected", KATS)
def test_reference_filter_known_answers(flt, meta, expected):
    assert MetadataFilter.parse(flt).accepts(1, meta) is expected
    assert pxo.metadata_filter_accepts(flt, meta) is expected


def test_compilation_errors():
    for bad in ([], {"a": {}}, {"a": {"between": 1}}, {"a": {"gt": "x"}}, {"a": {"in": []}}, {"a": {"in": 5}},
                {"a": {"exists": 1}}, {"a": None}):
        with pytest.raises(Configuration):
            MetadataFilter.parse(bad)


def test_conditions_are_ordered_by_field():
    assert MetadataFilter.parse({"b": 1, "a": 2}).conditions == MetadataFilter.parse({"a": 2, "b": 1}).conditions


VALUES = [None, 0, 1, -5, 2024, 2**40, 0.0, -0.0, 0.5, 1.0, 2024.0, -3.25, math.inf, -math.inf, math.nan,
          True, False, "a", "b", "en", ""]


def random_filter(rng):
    flt = {}
    for field in rng.sample(["x", "y", "z"], rng.randint(1, 3)):
        kind = rng.randrange(6)
        if kind == 0:
            flt[field] = rng.choice([v for v in VALUES if v is not None and not (isinstance(v, float) and
                                                                                 math.isnan(v))])
        elif kind == 1:
            op = rng.choice(["gt", "gte", "lt", "lte"])
            flt[field] = {op: rng.choice([0, 1, -5, 2024, 0.5, -3.25, 1.0, 1e300])}
        elif kind == 2:
            flt[field] = {"in": rng.sample(["a", "b", 1, 0.5, True, 2024], rng.randint(1, 3))}
        elif kind == 3:
            flt[field] = {"exists": rng.random() < 0.5}
        elif kind == 4:
            flt[field] = {"ne": rng.choice(["a", 1, 0.5, False])}
        else:
            flt[field] = {"gte": rng.choice([-5, 0]), "lt": rng.choice([1, 2024, 0.75])}
    return flt


def random_metadata(rng):
    meta = {}
    for field in ("x", "y", "z"):
        v = rng.choice(VALUES)
        if v is not None:
            meta[field] = v
    return meta


def test_product_and_oracle_agree_on_random_filters():
    rng = random.Random(7)
    for _ in range(3000):
        flt, meta = random_filter(rng), random_metadata(rng)
        assert MetadataFilter.parse(flt).accepts(1, meta) == pxo.metadata_filter_accepts(flt, meta), (flt, meta)
