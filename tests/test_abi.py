"""The C ABI library loads and exports every function that include/hardshell_b200.h declares
(no GPU needed: nothing here launches a kernel)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "hardshell_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:int|void|uint32_t|uint64_t)\s+(hs_\w+)\s*\(", text, flags=re.M)


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ["hs_open", "hs_model_load", "hs_batch_new", "hs_batch_set_overlap", "hs_batch_reset",
                     "hs_batch_position", "hs_batch_run_coded", "hs_batch_run_weights", "hs_last_error",
                     "hs_mem_info", "hs_model_free", "hs_batch_free", "hs_dev_free"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    from taco_b200 import build

    lib_path = build.build()
    lib = ctypes.CDLL(str(lib_path))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_open_without_a_gpu_reports_no_device():
    """CudaDevice::open on a machine without a device gives NoDevice (the reference's
    crates/hardshell-cuda/tests/no_device.rs). Skipped where a GPU is visible."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from taco_b200 import backend as B

    with pytest.raises(B.HardShellError) as e:
        B.CudaDevice(0)
    assert e.value.code == B.HS_NO_DEVICE
