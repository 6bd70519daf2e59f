"""Float parity gates that record what they measured.

`gate(value, limit)` asserts value < limit (a rel-L2 or an absolute error
against the oracle or another kernel) and records the measured value with
the test that took it; conftest.py prints every recorded gate at the end of
the run, tightest margin first, so a drift toward a limit shows before a
test fails."""
import os

RECORDS = []


def gate(value, limit, what=""):
    test = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    RECORDS.append((test, what, float(value), float(limit)))
    assert value < limit, f"{what or 'error'} {value:.3e} not below {limit:.1e}"
    return value
