import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# lines of measured parity figures, printed at the end of the run
_PARITY_LINES = []


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture
def parity_report():
    """A list a test appends one line of measured parity figures to; the lines
    are printed in the run's terminal summary."""
    return _PARITY_LINES


def pytest_terminal_summary(terminalreporter):
    if _PARITY_LINES:
        terminalreporter.write_sep("-", "measured parity (relative L2)")
        for line in _PARITY_LINES:
            terminalreporter.write_line(line)
