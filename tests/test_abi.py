"""CPU checks of the C ABI: the library loads, exports every symbol the
header declares, and fails loudly (no CPU fallback) without a GPU."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "jammi_b200.h")


def header_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(jb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = header_symbols()
    for s in ("jb_model_load", "jb_encode_text", "jb_encode_image", "jb_op_linear", "jb_op_linear_s8"):
        assert s in syms


def test_library_exports_every_header_symbol():
    from jammi_b200 import _lib
    lib = _lib.lib()
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # the ctypes table covers every declared entry point
    assert set(header_symbols()) <= set(_lib.exported_symbols())


def test_load_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from jammi_b200 import _lib
    h = ctypes.c_void_p()
    st = _lib.lib().jb_model_load(b"/nonexistent.safetensors", b"{}", 0, _lib.FMT_BF16, ctypes.byref(h))
    assert st == _lib.ERR_NO_DEVICE
    assert b"device" in _lib.lib().jb_last_error().lower()
    assert not h.value


def test_missing_library_raises(monkeypatch, tmp_path):
    import jammi_b200._lib as L
    monkeypatch.setattr(L, "LIB_PATH", str(tmp_path / "absent.so"))
    monkeypatch.setattr(L, "_lib", None)
    with pytest.raises(ImportError):
        L.lib()
    # monkeypatch restores LIB_PATH and the loaded handle afterwards


def test_mask_to_lengths_rejects_holes():
    import numpy as np
    from jammi_b200.encoders import mask_to_lengths
    assert list(mask_to_lengths(np.array([[1, 1, 0], [0, 0, 0], [1, 1, 1]]))) == [2, 0, 3]
    with pytest.raises(ValueError):
        mask_to_lengths(np.array([[1, 0, 1]]))


def test_ctypes_structs_match_the_header(tmp_path):
    """The Python mirrors of the header's structs have the C compiler's size
    and field offsets (a layout drift would silently misread fields)."""
    import shutil
    import subprocess
    from jammi_b200 import _lib
    from jammi_b200.driver import GenerateOpts, GenerateStats
    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    src = tmp_path / "sizes.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "jammi_b200.h"\n'
        "int main(void) {\n"
        '  printf("%zu %zu %zu %zu %zu\\n", sizeof(jb_model_info),\n'
        "         offsetof(jb_model_info, weight_bytes), offsetof(jb_model_info, preprocess_std),\n"
        "         sizeof(jb_generate_opts), sizeof(jb_generate_stats));\n"
        "  return 0;\n}\n")
    exe = tmp_path / "sizes"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    want = [ctypes.sizeof(_lib.ModelInfo), _lib.ModelInfo.weight_bytes.offset,
            _lib.ModelInfo.preprocess_std.offset, ctypes.sizeof(GenerateOpts),
            ctypes.sizeof(GenerateStats)]
    assert got == want, (got, want)


def test_sidecar_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from jammi_b200._lib import JbError, ERR_NO_DEVICE, ERR_INVALID, lib
    from jammi_b200.sidecar import SidecarIndex
    with pytest.raises(JbError) as e:
        SidecarIndex(64, "binary")
    assert e.value.status == ERR_NO_DEVICE
    with pytest.raises(ValueError):
        SidecarIndex(64, "int8")  # quantised inside the graph library: not a device sidecar
    h = ctypes.c_void_p()
    assert lib().jb_sidecar_create(0, 64, 1, ctypes.byref(h)) == ERR_INVALID  # F16: refused before any device call
    assert lib().jb_sidecar_create(0, 0, 3, ctypes.byref(h)) == ERR_INVALID
    assert lib().jb_sidecar_len(None) == -1
    assert lib().jb_sidecar_add(None, None, None, 0, None, None) == ERR_INVALID
    lib().jb_sidecar_free(None)
