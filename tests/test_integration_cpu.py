"""CPU: the reference-side code in INTEGRATION.md stays true to the C ABI.

- Every drop-in shim block (the ones that define the reference's functions over libacb) compiles
  with g++ -fsyntax-only against include/acb.h and include/acb_models.h, with the one
  reference-side type the shims name (DebugDumper) declared as a stub. This catches a shim whose
  call no longer matches a signature or passes an argument of the wrong type.
- Every acb_* function or type a block uses -- the call-site fragments included -- is declared in
  include/."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.join(os.path.dirname(__file__), "..")
DOC = os.path.join(ROOT, "INTEGRATION.md")

PRELUDE = """#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>
#include "acb.h"
#include "acb_models.h"
struct DebugDumper;  // the reference's debug dumper: the shims take it and ignore it
"""


def _blocks():
    with open(DOC) as f:
        return re.findall(r"```cpp\n(.*?)```", f.read(), re.S)


def _is_shim(block):
    """A shim block defines functions or types at namespace scope; a fragment is statements."""
    return any(re.match(r"(static |struct |#pragma once|#include )", ln) for ln in block.splitlines())


def test_integration_has_shims_and_fragments():
    blocks = _blocks()
    assert sum(_is_shim(b) for b in blocks) >= 4
    assert any(not _is_shim(b) for b in blocks)


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_integration_shims_compile(tmp_path):
    src = PRELUDE + "\n".join(b.replace("#pragma once", "") for b in _blocks() if _is_shim(b))
    path = tmp_path / "shims.cpp"
    path.write_text(src)
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wno-unused-function", "-I",
                        os.path.join(ROOT, "include"), str(path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


def test_integration_names_are_declared():
    decl = ""
    for h in ("acb.h", "acb_models.h"):
        with open(os.path.join(ROOT, "include", h)) as f:
            decl += f.read()
    declared = set(re.findall(r"\b(acb_\w+)\s*\(", decl)) | set(re.findall(r"\b(acb_\w+)\b", decl))
    used = set()
    for b in _blocks():
        used |= set(re.findall(r"\b(acb_\w+)\b", b))
    missing = sorted(u for u in used if u not in declared)
    assert not missing, missing
