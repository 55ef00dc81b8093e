"""The oracle's restated F.* compositions reproduce the committed fixtures,
which were produced by executing the reference's own functional.py on the
oracle's engine (tests/golden/make_golden.py)."""

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
import make_golden  # noqa: E402

from parity import assert_bitexact  # noqa: E402

CASES = make_golden.cases()


@pytest.mark.parametrize("name,build", CASES, ids=[c[0] for c in CASES])
def test_oracle_reproduces_fixture(oracle, golden, name, build):
    got = build(oracle)
    for k, v in got.items():
        assert_bitexact(v, golden[f"{name}.{k}"], what=f"{name}.{k}")
