"""C-ABI library checks that need no GPU: it loads, exports every function include/minicpm5_mk.h
declares, and reports errors as status codes (no compute calls)."""
import ctypes
import os
import re

import pytest

from minicpm5_mk import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "minicpm5_mk.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mk_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_binding_list():
    assert _declared() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in _declared():
        assert hasattr(L, name), name


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.mk_status_string(0) == b"ok"
    assert L.mk_status_string(1) == b"unsupported shape"
    assert L.mk_version() >= 100
    assert L.mk_lm_head_parts() > 0


def test_bad_arguments_are_status_codes():
    L = _lib.lib()
    h = ctypes.c_void_p()
    assert L.mk_create(None, 0, ctypes.byref(h)) == 5  # MK_ERR_BAD_ARG
    c = _lib.MkConfigC(2, 384, 512, 4, 2, 80, 1000, 1024, 1e-6, 1e4, 1.0, 1.0, 1.0)
    assert L.mk_create(ctypes.byref(c), 0, ctypes.byref(h)) == 1  # head_dim 80: MK_ERR_BAD_SHAPE
    assert L.mk_forward(None, None, 1, 128, None, 0, None, None, None, None) == 5
    assert L.mk_launches_per_forward(None, 1, 128) == 0
    # shape checks run before any device work
    assert L.mk_gemm_w8a16(8, 128, 100, 128, 8, 8, 256, 0, 8, 1.0, 8, 256, None, 0, None) == 1  # K % 64
    assert L.mk_attention_prefill(8, 1, 100, 16, 2, 96, 1920, 0, 1536, 1728, 1.0, 8, 1536, None) == 1  # seq % 128


def test_header_is_plain_c_and_links(tmp_path):
    """A C host (the language of a cgo / JNI / N-API shim) includes the header as C99, links against the
    library and calls it: the boundary has no C++ types."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not installed")
    src = tmp_path / "host.c"
    src.write_text('''#include <stdio.h>
#include "minicpm5_mk.h"
int main(void) {
  mk_handle* h = NULL;
  mk_stage_times t;
  (void)t;
  if (mk_create(NULL, 0, &h) != MK_ERR_BAD_ARG) return 1;
  if (mk_sp_block(NULL, 8192, 2) != 0) return 2;
  printf("%d %s\\n", (int)mk_version(), mk_status_string(MK_ERR_WORKSPACE));
  return 0;
}
''')
    libdir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "host"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe),
                    "-L", libdir, "-l:" + os.path.basename(_lib.LIB_PATH), "-Wl,-rpath," + libdir],
                   check=True, capture_output=True, timeout=120)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=60).stdout
    assert out.split(None, 1)[1].strip() == "workspace too small"
