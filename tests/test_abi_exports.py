"""The C-ABI library loads without a GPU and exports what include/tgs_abi.h declares."""
import ctypes
import subprocess

from tinygs_b200 import _abi


def test_header_declares_the_boundary():
    syms = _abi.header_symbols()
    for name in ("tgs_raster_create", "tgs_raster_forward", "tgs_raster_backward", "tgs_loss_l1_ssim",
                 "tgs_adam_step", "tgs_status_string"):
        assert name in syms
    # every declared function has a ctypes prototype and vice versa
    assert set(syms) == set(_abi.PROTOTYPES)


def test_library_loads_and_exports_every_symbol():
    lib = _abi.load_library()
    for name in _abi.header_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_abi.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(_abi.header_symbols()) <= exported
    # nothing but the ABI leaks out of the library
    assert {s for s in exported if not s.startswith("tgs_")} <= {"_init", "_fini"}


def test_status_strings_and_version_need_no_gpu():
    lib = _abi.load_library()
    assert lib.tgs_version().decode().startswith("tinygs-b200")
    assert lib.tgs_status_string(_abi.TGS_OK) == b"ok"
    assert lib.tgs_status_string(_abi.TGS_ERR_CAPACITY) == b"capacity exceeded"
    assert lib.tgs_status_string(12345) == b"unknown status"


def test_argument_validation_runs_before_any_device_work():
    lib = _abi.load_library()
    h = ctypes.c_void_p()
    assert lib.tgs_raster_create(None, ctypes.byref(h)) == _abi.TGS_ERR_INVALID_ARGUMENT
    bad = _abi.TgsRasterCaps(10, 0, 10, 0)
    assert lib.tgs_raster_create(ctypes.byref(bad), ctypes.byref(h)) == _abi.TGS_ERR_INVALID_ARGUMENT
    huge = _abi.TgsRasterCaps(10, 100000, 100000, 0)
    assert lib.tgs_raster_create(ctypes.byref(huge), ctypes.byref(h)) == _abi.TGS_ERR_UNSUPPORTED
    assert lib.tgs_raster_forward(None, None, None, 0, None, None, None, None) == _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_loss_l1(7, 8, 8, None, None, None, None, 1.0, None) == _abi.TGS_ERR_INVALID_ARGUMENT
    assert lib.tgs_adam_step(None, None, None, None, None, 1, 1.0, 0, None) == _abi.TGS_ERR_INVALID_ARGUMENT
