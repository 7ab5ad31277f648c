"""libb200ops.so: loads without a GPU and exports every function that
include/b200ops.h declares (CPU only, no compute calls)."""
import ctypes
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    with open(os.path.join(REPO, "include", "b200ops.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    from src import b200
    lib = b200.load_library()
    names = header_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_the_header():
    from src import b200
    assert set(b200.exported_symbols()) == set(header_functions())


def test_version_and_error_string():
    from src import b200
    lib = b200.load_library()
    assert lib.b200_version() == 1
    assert isinstance(lib.b200_last_error(), bytes)


def test_invalid_arguments_fail_before_any_launch():
    """Shape / alignment validation happens on the host: no CUDA call needed."""
    from src import b200
    lib = b200.load_library()
    # K not a multiple of 8
    rc = lib.b200_linear(ctypes.c_void_p(16), 12, ctypes.c_void_p(16), 12, None,
                         ctypes.c_void_p(16), 16, 4, 16, 12, None, 0, None)
    assert rc == -1
    assert b"multiples of 8" in lib.b200_last_error()
    # rms_norm dim not a multiple of 8
    rc = lib.b200_rms_norm(ctypes.c_void_p(16), 12, None, ctypes.c_void_p(16), ctypes.c_void_p(16),
                           12, None, 1, 12, 1e-6, None)
    assert rc == -2
