"""The CPU oracle against the reference's own known-answer tests.

Every case in tests/golden/reference_cases.json is a testthat case of the
reference (file:line in the case) with the base-R expected value; the oracle
must reproduce them before it is trusted as the checker of the CUDA path.
"""
import re

import numpy as np
import pytest

from golden_runner import expected_of, run_oracle
from helpers import assert_rel, golden_cases

CASES = golden_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_oracle_matches_reference_case(case):
    if "error" in case:
        with pytest.raises(ValueError) as ei:
            run_oracle(case)
        assert re.search(case["error"], str(ei.value))
        return
    got = np.asarray(run_oracle(case), dtype=np.float64)
    exp = expected_of(case)
    if exp.size == 1:
        got = got.reshape(-1)[:1].reshape(exp.shape) if got.size == 1 else got
    assert got.size == exp.size, (case["id"], got.shape, exp.shape)
    got = got.reshape(exp.shape, order="F") if got.shape != exp.shape else got
    # f32 inputs: the reference compares at tolerance 1e-6 (tests/testthat/helper-tensor-eq.R:13-15)
    assert_rel(got, exp, 1e-6, case["id"], atol=1e-7)
