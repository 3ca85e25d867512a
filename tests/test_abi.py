"""The C-ABI library loads without a GPU and exports every symbol its headers declare."""

import ctypes
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(stratum_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("stratum_nf4_quantize", "stratum_nf4_dequantize", "stratum_nf4_dequantize_dq",
                 "stratum_nf4_quantize_absmax_dq", "stratum_last_error", "stratum_abi_version"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from stratum_b200 import _lib

    lib = _lib.lib()  # loads (and builds if needed) without touching a GPU
    exported = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                              check=True).stdout
    exported = set(re.findall(r"\bT (stratum_\w+)", exported))
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in declared_symbols():
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)
    # the Python binding types every declared function
    assert declared_symbols() <= set(_lib.SIGNATURES)
    assert lib.stratum_abi_version() == _lib.ABI_VERSION


def test_invalid_arguments_are_reported_without_a_gpu():
    from stratum_b200 import _lib

    lib = _lib.lib()
    # blocksize outside the supported set is rejected before any CUDA call
    rc = lib.stratum_nf4_dequantize(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 128, 48,
                                    ctypes.c_void_p(16), 1, None)
    assert rc == _lib.STRATUM_ERR_UNSUPPORTED
    assert b"blocksize" in lib.stratum_last_error()
    rc = lib.stratum_nf4_quantize(None, 1, 64, 64, None, None, None, None)
    assert rc == _lib.STRATUM_ERR_INVALID
    assert lib.stratum_nf4_quantize(None, 1, 0, 64, None, None, None, None) == _lib.STRATUM_OK  # empty input


def test_package_exports_exist():
    import stratum_b200

    missing = [n for n in stratum_b200.__all__ if not hasattr(stratum_b200, n)]
    assert missing == []
    # the reference's hot-path names are all present (stratum/__init__.py:51-54, stratum/upload.py)
    for name in ("NF4Linear", "NF4Prefetch", "prefetch_weights", "ensure_prefetched_weights", "prepare_nf4",
                 "ensure_weights", "free_weights", "DeviceStage", "assign_layers_to_devices", "NF4_ATTR"):
        assert name in stratum_b200.__all__
    assert stratum_b200.NF4_ATTR == "roundpipe_nf4_payload"
