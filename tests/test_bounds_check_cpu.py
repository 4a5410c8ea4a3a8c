"""Host side of the bounds-checked build: the variant's name, folder and define, the
environment switch, and that every kernel file with checked indices has its error word read by
the bindings (and only those)."""

import os
import re

from b200serve.ops import build as B

CSRC = os.path.join(os.path.dirname(B.__file__), "csrc")


def test_variant_paths_and_flags():
    rel, chk = B.built_library_path(False), B.built_library_path(True)
    assert rel.endswith(os.path.join("_build", "b200_ops.so"))
    assert chk.endswith(os.path.join("_build_checked", "b200_ops_checked.so"))
    assert B.CHECK_DEFINE == "-DB200_BOUNDS_CHECK" and B.CHECK_DEFINE not in B.NVCC_FLAGS


def test_env_switch_selects_variant(monkeypatch):
    from b200serve import ops
    monkeypatch.setenv("B200_BOUNDS_CHECK", "1")
    assert ops.extension_path() == B.built_library_path(True)
    monkeypatch.setenv("B200_BOUNDS_CHECK", "0")
    assert ops.extension_path() == B.built_library_path(False)


def test_every_checked_unit_is_read():
    units, guarded = set(), set()
    for f in os.listdir(CSRC):
        if not f.endswith(".cu"):
            continue
        src = open(os.path.join(CSRC, f)).read()
        units |= set(re.findall(r"^B200_BOUNDS_ACCESSOR\((\w+)\)", src, re.M))
        if re.search(r"B200_IN_RANGE\(|table_block\(", src):
            guarded.add(f[:-3])
    bind = open(os.path.join(CSRC, "bindings.cpp")).read()
    listed = re.search(r"#define B200_BOUNDS_UNITS\(X\)(.*?)\n\n", bind, re.S).group(1)
    read = set(re.findall(r"X\((\w+)\)", listed))
    assert units == read, (units ^ read)
    assert guarded <= units, guarded - units
    # the error codes are distinct per site
    codes = re.findall(r"(?:B200_IN_RANGE\([^;]*?,\s*|table_block\([^;]*?,\s*)(0x[0-9a-f]+)\)",
                       "".join(open(os.path.join(CSRC, f)).read() for f in os.listdir(CSRC) if f.endswith(".cu")))
    assert len(codes) >= 12
