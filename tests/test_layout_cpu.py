"""Invariants of the product's layout, on CPU: the library never reaches
the test oracle, and it loads its CUDA path or fails loudly."""

import ast
import os

import hessboost_b200 as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hessboost_b200")


def _package_files():
    for base, _, files in os.walk(PKG):
        if "_lib" in base.split(os.sep) or "__pycache__" in base:
            continue
        for name in files:
            if name.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                yield os.path.join(base, name)


def test_package_never_reaches_the_oracle():
    # the oracle is test infrastructure: no import, path or library name of
    # it anywhere in the shipped package
    for path in _package_files():
        text = open(path, encoding="utf-8").read()
        for needle in ("oracle_lib", "liboracle", "orc_", os.sep + "oracle" + os.sep, "tests" + os.sep):
            assert needle not in text, f"{os.path.relpath(path, ROOT)} names {needle!r}"
        if path.endswith(".py"):
            for node in ast.walk(ast.parse(text)):
                if isinstance(node, (ast.Import, ast.ImportFrom)):
                    names = [a.name for a in node.names] + [getattr(node, "module", None) or ""]
                    assert not any("oracle" in n or n.startswith("tests") for n in names), path


def test_library_is_the_in_tree_build():
    # the ctypes library is the one built in the package tree, not a copy
    # found elsewhere
    assert os.path.dirname(H._build.LIB) == os.path.join(PKG, "_lib")
    assert H.lib()._name == H._build.LIB


def test_every_source_is_built():
    # every CUDA and C++ source of the package is in the library's build
    csrc = os.path.join(PKG, "csrc")
    sources = sorted(f for f in os.listdir(csrc) if f.endswith((".cu", ".cpp")))
    assert sorted(H._build.SOURCES) == sources
