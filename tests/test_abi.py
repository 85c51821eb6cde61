"""The C ABI: the library builds, loads without a GPU, exports every function include/bpt_b200.h declares, and
the ctypes binding covers exactly those functions. No kernel is called here."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "bpt_b200.h"


def declared() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(bpt_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def library():
    from bpt_b200 import _lib

    if not _lib.LIB_PATH.exists():
        import importlib.util

        spec = importlib.util.spec_from_file_location("bpt_build", ROOT / "bytes-per-token_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return ctypes.CDLL(str(_lib.LIB_PATH))


def test_header_declares_the_entry_points():
    names = declared()
    assert {"bpt_w4a16_linear", "bpt_paged_attend", "bpt_paged_kv_write", "bpt_kivi_decode_partials"} <= names


def test_library_exports_every_declared_symbol(library):
    missing = [name for name in sorted(declared()) if not hasattr(library, name)]
    assert not missing, f"declared in {HEADER.name} but not exported: {missing}"


def test_binding_covers_the_header(library):
    from bpt_b200 import _lib

    assert set(_lib.SIGNATURES) == declared()


def test_abi_version_and_error_string_need_no_gpu(library):
    from bpt_b200 import _lib

    assert _lib.lib().bpt_abi_version() == 1
    assert isinstance(_lib.lib().bpt_last_error(), bytes)


def test_host_side_validation_runs_before_any_launch(library):
    """A bad argument is refused by the C entry point itself, with a status and a message, on any machine."""
    from bpt_b200 import _lib

    L = _lib.lib()
    st = L.bpt_w4a16_linear(None, 0, None, None, None, None, 0, 1, 1, 1, 128, 0, None)
    assert st == _lib.ERR_INVALID and b"null" in L.bpt_last_error()
    st = L.bpt_paged_kv_write(1, 1, 2, 0, 0, 0, 1, 1, 1, 96, 1, 1, 1, 1, 1, 1.0, 1.0, None, None, 16, 1, None)
    assert st == _lib.ERR_UNSUPPORTED and b"D=96" in L.bpt_last_error()
    assert L.bpt_paged_attend_workspace_bytes(32, 16, 128, 8) >= 32 * 8 * 16 * 128 * 4
    # rms_norm_int8: x_out without delta, and a row stride shorter than the row
    assert L.bpt_rms_norm_int8(None, 2, 64, None, 2, None, None, None, None, 0, 64, 1e-6, 0, None) == _lib.OK  # empty
    st = L.bpt_rms_norm_int8(1, 2, 64, 1, 2, None, 1, 1, 1, 4, 64, 1e-6, 0, None)
    assert st == _lib.ERR_INVALID and b"needs delta" in L.bpt_last_error()
    st = L.bpt_rms_norm_int8(1, 2, 32, 1, 2, None, None, 1, 1, 4, 64, 1e-6, 0, None)
    assert st == _lib.ERR_INVALID and b"row stride" in L.bpt_last_error()
