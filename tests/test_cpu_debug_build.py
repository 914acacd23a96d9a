"""The bounds-checked build (R2S_DEBUG, csrc/r2s_debug.cuh) builds and loads
without a GPU, exports the same C ABI as the release library and identifies
itself; its flag query rejects a null pointer without touching CUDA."""
import ctypes
import importlib.util
import os

import pytest

from _helpers import ROOT
from test_cpu_abi import declared_functions


def _build_module():
    spec = importlib.util.spec_from_file_location(
        "r2s_build", os.path.join(ROOT, "bt-3dgs_b200", "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def libs():
    from r2splat.cuda._backend import load_library

    b = _build_module()
    return load_library(b.build()), load_library(b.build(debug=True))


def test_debug_build_exports_the_release_abi(libs):
    release, debug = libs
    for name in declared_functions():
        assert hasattr(release, name) and hasattr(debug, name), name
    assert release.r2s_debug_build() == 0
    assert debug.r2s_debug_build() == 1
    assert b"bounds-checked" in debug.r2s_version()
    assert b"bounds-checked" not in release.r2s_version()


def test_debug_flag_query_rejects_null(libs):
    for lib in libs:
        assert lib.r2s_debug_flags(None, 0) == 1  # R2S_ERR_ARG
        buf = ctypes.create_string_buffer(256)
        lib.r2s_last_error(buf, 256)
        assert b"flags is null" in buf.value
