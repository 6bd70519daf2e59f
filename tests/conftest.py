import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "sam3d.cpp_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built libs3dsp.so")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Every float gate the run checked (tests/gates.py), tightest first."""
    from gates import RECORDS

    if not RECORDS:
        return
    rows = sorted(RECORDS, key=lambda r: -r[2] / r[3])
    tr = terminalreporter
    tr.section("float parity gates (measured / limit, tightest first)")
    for test, what, value, limit in rows[:60]:
        tr.write_line(f"{value:10.3e} / {limit:8.1e}  ({100 * value / limit:5.1f} %)  {test} {what}".rstrip())
    if len(rows) > 60:
        tr.write_line(f"... {len(rows) - 60} more, all further from their limits")
