"""The drop-in boundary is plain C: laya-zig's host binds it with
`@cImport`, which parses the headers as C. Both headers must compile as C99
on their own, warnings as errors, and a C program that takes the address of
every declared entry point must link against the built library."""
import os
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

INC = os.path.join(ROOT, "include")
LIB = os.path.join(ROOT, "laya_zig_b200")
needs_cc = pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")


def _entry_points(header):
    text = open(os.path.join(INC, header)).read()
    return sorted(set(re.findall(r"\b(laya_(?:gpu|tok)_\w+)\s*\(", text)))


@needs_cc
@pytest.mark.parametrize("header", ["laya_gpu.h", "laya_tok.h"])
def test_header_is_c99(header, tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "%s"\nint main(void) { return 0; }\n' % header)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", INC, "-c", str(src),
                        "-o", str(tmp_path / "h.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@needs_cc
def test_c_program_links_every_entry_point(tmp_path):
    names = _entry_points("laya_gpu.h") + _entry_points("laya_tok.h")
    assert len(names) >= 19
    body = "\n".join("    p[%d] = (void (*)(void))&%s;" % (i, n) for i, n in enumerate(names))
    src = tmp_path / "link.c"
    src.write_text('#include "laya_gpu.h"\n#include "laya_tok.h"\n#include <stdio.h>\n'
                   "int main(void) {\n    void (*p[%d])(void);\n%s\n    printf(\"%%p\\n\", (void*)p[0]);\n"
                   "    return 0;\n}\n" % (len(names), body))
    exe = tmp_path / "link"
    r = subprocess.run(["gcc", "-std=c99", "-I", INC, str(src), "-o", str(exe), "-L", LIB, "-llaya_gpu",
                        "-Wl,-rpath," + LIB], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
