"""The reference's known-answer cases through the CUDA path (acediar mirror)."""
import re

import numpy as np
import pytest

from golden_runner import expected_of, run_gpu, run_oracle
from helpers import assert_rel, golden_cases

CASES = golden_cases()
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", CASES, ids=[c["id"] for c in CASES])
def test_cuda_matches_reference_case(acd, case):
    if "error" in case:
        with pytest.raises(ValueError) as ei:
            run_gpu(acd, case)
        assert re.search(case["error"], str(ei.value))
        return
    got = np.asarray(run_gpu(acd, case), dtype=np.float64)
    exp = expected_of(case)
    assert got.size == exp.size, (case["id"], got.shape, exp.shape)
    if got.shape != exp.shape:
        assert got.size == 1 and exp.size == 1
        got = got.reshape(exp.shape)
    assert_rel(got, exp, 1e-6, case["id"], atol=1e-7)
    # and against the oracle on the same inputs
    orc = np.asarray(run_oracle(case), dtype=np.float64).reshape(got.shape, order="F")
    assert_rel(got, orc, 1e-6, case["id"] + " vs oracle", atol=1e-7)
