"""pytest setup: the `gpu` marker, import paths, and readers for the golden fixtures."""
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "moe-stream-mac_b200"
for p in (str(REPO), str(PKG), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs on the GPU box with -m gpu)")
