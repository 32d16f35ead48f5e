"""Shared pytest setup: the ``gpu`` marker, the repo root on sys.path, and the
parity-margin report (worst error / tolerance bound per test, printed in the
terminal summary so every run shows how close each kernel came to its bar)."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

_MARGINS: dict = {}


def record_margin(worst: float, name: str | None = None) -> None:
    """Record a worst normalised error (error / bound, 1.0 = at the bound)
    for the running test; the summary keeps the largest per test."""
    if name is None:
        name = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    _MARGINS[name] = max(_MARGINS.get(name, 0.0), float(worst))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_terminal_summary(terminalreporter):
    if not _MARGINS:
        return
    terminalreporter.write_sep("-", "parity margins (worst error / tolerance bound)")
    for name in sorted(_MARGINS):
        terminalreporter.write_line(f"{_MARGINS[name]:.4f}  {name}")
    terminalreporter.write_line(f"max {max(_MARGINS.values()):.4f} over {len(_MARGINS)} tests")
