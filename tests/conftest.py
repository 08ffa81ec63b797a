"""Test configuration: puts the repository root on sys.path and registers
the ``gpu`` marker (tests that need a B200)."""
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def pytest_terminal_summary(terminalreporter):
    """Reports the largest backward-gradient errors the GPU tests measured
    (relative to each gradient's largest entry), per dtype."""
    mod = sys.modules.get("test_attention_bwd_gpu")
    worst = getattr(mod, "WORST", None) if mod else None
    if worst:
        terminalreporter.write_line("backward worst error / max|grad|: " +
                                    ", ".join(f"{k} {v:.3e}" for k, v in sorted(worst.items())))
