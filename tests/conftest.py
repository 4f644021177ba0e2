import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PACKAGE = os.path.join(ROOT, "fast-transformer_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for path in (ROOT, PACKAGE, GOLDEN):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device; run with -m gpu")
