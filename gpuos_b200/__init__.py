"""gpuos_b200 — B200-native aggregated small-op executor.

`gpuos_b200.gpuos_ext` is a drop-in for the reference's `gpuos_ext` module
(init / submit_* / flush / register_* / shutdown); `gpuos_b200.scheduler`
mirrors the reference's TorchDispatch scheduler.  The compute path is the
CUDA code in `libgpuos_b200.so`; there is no CPU fallback: if the native
library is missing, `load()` (and `from gpuos_b200 import gpuos_ext`) fails.
"""
import importlib
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libgpuos_b200.so"


def load():
    """Import and return the native `gpuos_ext` module, failing loudly."""
    try:
        return importlib.import_module(".gpuos_ext", __name__)
    except ImportError as e:  # the native module is the product
        raise ImportError(
            "gpuos_b200 native extension is not built; run `python -m gpuos_b200._build` "
            f"(nvcc for sm_100a). Original error: {e}") from e
