import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

_PARITY_LINES = []


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Prints the per-config parity statistics the full-size tests recorded (rows checked,
    near-tie disagreements, largest probability error), so they show in a -q run's tail."""
    if _PARITY_LINES:
        terminalreporter.write_sep("-", "full-size parity against the oracle")
        for line in _PARITY_LINES:
            terminalreporter.write_line(line)


@pytest.fixture(scope="session")
def parity_log():
    return _PARITY_LINES


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.lib()
    return o
