"""Pin the CPU oracle to the reference's documented known answers
(tests/golden/semantics_kat.json, derived case by case from the cited
reference documentation and code)."""
import pytest

import oracle
from kat_cases import build, load_cases

CASES = load_cases()


@pytest.mark.parametrize("case", CASES, ids=[f"{i}-{c['kind']}" for i, c in enumerate(CASES)])
def test_oracle_matches_documented_answer(case):
    kind, rec, ins, check = build(case)
    outs = oracle.elementwise(rec, ins) if kind == "elementwise" else oracle.reduce(rec, ins)
    assert check(outs), f"{case} -> {outs}"


def test_fixture_covers_every_semantic_family():
    kinds = {c["kind"] for c in CASES}
    assert {"int_op", "cast", "cast_bits", "bf16_nan", "maximum", "minimum", "compare", "arg", "reduce",
            "float_op"} <= kinds
    assert all(c["source"] for c in CASES)
