import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# A checkout of the reference project, for the CPU tests that compare with
# its own code: $H4B_REFERENCE_ROOT, else a sibling directory `reference`
# next to this repository. Tests that need it skip when it is absent.
REFERENCE_ROOT = Path(os.environ.get("H4B_REFERENCE_ROOT", ROOT.parent / "reference"))


def reference_available() -> bool:
    return (REFERENCE_ROOT / "cpu_lightspark.py").is_file() and (REFERENCE_ROOT / "inference_runtime.py").is_file()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
