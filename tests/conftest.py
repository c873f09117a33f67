import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


def pytest_terminal_summary(terminalreporter):
    """Parity figures of every oracle check made in this session (bit-identical fraction and
    error over tolerance, under the asserted sqrt(K) bound and the worst-case K bound)."""
    try:
        from oracle import oracle as O
    except Exception:
        return
    if not O.REPORTS:
        return
    tr = terminalreporter
    tr.section("parity figures (GPU result vs oracle, per check)")
    for tid, r in O.REPORTS:
        tr.write_line(f"{tid or '-'} K={r.get('K')}: {O.format_report(r)}")
    n = sum(r["elements"] for _, r in O.REPORTS)
    bad = sum(r["mismatches"] for _, r in O.REPORTS)
    bit = sum(r["bit_identical_frac"] * r["elements"] for _, r in O.REPORTS) / max(n, 1)
    worst = max(r["max_err_over_tol"] for _, r in O.REPORTS)
    tr.write_line(f"parity summary: {len(O.REPORTS)} checks, {n} elements, {bad} outside tolerance, "
                  f"bit-identical {bit:.6f}, max err/tol {worst:.3g}")
