import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_terminal_summary(terminalreporter):
    from tests.helpers import PARITY_REPORT
    if PARITY_REPORT:
        terminalreporter.section("parity at the workloads' full sizes")
        for line in PARITY_REPORT:
            terminalreporter.write_line(line)
