import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Lists, on every run, the parity keys that met the bf16 bar only relative
    to the reference's own CUDA path (flash-linear-attention's recorded errors
    on the same inputs) rather than the absolute rtol 2e-2 / atol 2e-3 bar."""
    try:
        from kda_cuda_runner import RELATIVE_ONLY
    except Exception:  # noqa: BLE001 -- CPU-only runs never import the runner
        return
    if not RELATIVE_ONLY:
        return
    tr = terminalreporter
    tr.section("keys passing only relative to flash-linear-attention's errors")
    for case in sorted(RELATIVE_ONLY):
        keys = ", ".join(f"{k} (viol {v:.2f}, rel {r:.1e})" for k, (v, r) in sorted(RELATIVE_ONLY[case].items()))
        tr.write_line(f"{case}: {keys}")
