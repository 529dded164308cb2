import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(autouse=True)
def _skip_gpu_without_cuda(request):
    if request.node.get_closest_marker("gpu") and not cuda_ok():
        pytest.skip("no CUDA device")


def pytest_terminal_summary(terminalreporter):
    """Parity summary: for every test that compared a CUDA result with the
    oracle, the bar's worst |x-r|/(|r|+rms) next to the plain max relative
    error |x-r|/|r| and the share of elements within rtol*|r|."""
    try:
        import oracle
    except Exception:
        return
    log = oracle.PARITY_LOG
    if not log:
        return
    per = {}
    for tid, rtol, worst, plain, within, n in log:
        w = per.setdefault(tid, [rtol, 0.0, 0.0, 1.0, 0])
        w[1], w[2], w[3], w[4] = max(w[1], worst), max(w[2], plain), min(w[3], within), w[4] + n
    tr = terminalreporter
    tr.write_sep("-", f"parity vs oracle: {len(per)} tests")
    tr.write_line(f"{'rtol':>7} {'worst(|r|+rms)':>14} {'plain max rel':>13} {'within rtol|r|':>14} {'elems':>9}  test")
    for tid, (rtol, worst, plain, within, n) in sorted(per.items()):
        tr.write_line(f"{rtol:7.0e} {worst:14.3e} {plain:13.3e} {within:14.6f} {n:9d}  {tid}")
