"""include/godwit_cuda.h is a valid C11 header (what Swift's Clang importer
reads through swift/CGodwitCUDA/module.modulemap) and a C program links every
declared entry point from libgodwit_cuda.so.  Runs on the CPU: the program
only calls entry points that need no device."""
import os
import re
import shutil
import subprocess

import pytest

from godwit_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "godwit_cuda.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^GW_API\s+[\w\s\*]+?\b(gw_\w+)\s*\(", text, flags=re.M)))


PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "godwit_cuda.h"

/* every declared entry point, so the link fails if one is missing */
static void (*const every_entry[])(void) = {
ENTRIES
};

int main(void) {
    gw_bank_desc d;
    if (gw_version() <= 0) return 1;
    if (strlen(gw_last_error()) != 0) return 2;
    /* GPT-OSS-120B: the reference installer's 13,287,424-byte expert stride */
    if (gw_layout_default(2880, 2880, 128, 36, 4, GW_ACT_GPTOSS_CLAMPED, &d) != GW_OK) return 3;
    if (d.expert_stride != 13287424 || d.section_offset[GW_SEC_DOWN_BLOCKS] % 16384) return 4;
    if (gw_layout_default(100, 2880, 128, 36, 4, GW_ACT_SILU, &d) != GW_E_ARG) return 5;
    if (strlen(gw_last_error()) == 0) return 6;
    printf("%d entry points linked\n", (int)(sizeof every_entry / sizeof every_entry[0]));
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_header_compiles_as_c11_and_links(tmp_path):
    names = declared()
    assert names
    src = tmp_path / "abi_check.c"
    src.write_text(PROGRAM.replace("ENTRIES", ",\n".join(f"    (void (*)(void)){n}" for n in names)))
    exe = tmp_path / "abi_check"
    libdir = os.path.dirname(_abi.LIB_PATH)
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic-errors",
           "-Wno-error=pedantic", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
           "-L", libdir, "-lgodwit_cuda", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert f"{len(names)} entry points linked" in run.stdout


def test_swift_module_map_points_at_the_header():
    mm = open(os.path.join(ROOT, "swift", "CGodwitCUDA", "module.modulemap")).read()
    m = re.search(r'header\s+"([^"]+)"', mm)
    assert m and os.path.normpath(os.path.join(ROOT, "swift", "CGodwitCUDA", m.group(1))) == HEADER
    assert 'link "godwit_cuda"' in mm
    shim = open(os.path.join(ROOT, "swift", "GodwitCUDA", "ExpertRunnerCUDA.swift")).read()
    # the shim only calls entry points the header declares
    called = set(re.findall(r"\b(gw_[a-z_0-9]+)\(", shim)) - {"gw_bank_desc"}  # a struct
    assert called and called <= set(declared()), called - set(declared())
