"""include/exl3_b200.h is plain C: a C99 program includes it, links libexl3b200.so
and calls entry points that answer without a GPU (version, status strings, argument
validation, the host-memory checkpoint reader)."""

import os
import shutil
import subprocess

import pytest

from exl3_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SOURCE = r"""
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <unistd.h>
#include "exl3_b200.h"

int main(int argc, char** argv)
{
    if (exl3b200_abi_version() != EXL3B200_ABI_VERSION) return 1;
    if (strcmp(exl3b200_status_string(EXL3B200_OK), "ok") != 0) return 2;
    /* validation happens before any CUDA call */
    if (exl3b200_dequant(NULL, 8, 8, 4, 0, NULL, NULL, NULL, 0, NULL) != EXL3B200_ENULL) return 3;
    if (exl3b200_gemv_state_size(4096) == 0 || exl3b200_gemv_scratch_size(1, 4096) == 0) return 4;
    exl3b200_linear lin = {0};
    lin.k = 128;
    (void) lin;
    /* the checkpoint reader into host memory: bytes 3..10 of this program's own file */
    int fd = open(argv[0], O_RDONLY);
    if (fd < 0) return 5;
    unsigned char buf[8], ref[8];
    long long off = 3, size = 8;
    void* dst = buf;
    if (exl3b200_read_ranges(fd, &off, &size, &dst, 1, 0, NULL, 0, 2, 0, NULL) != EXL3B200_OK) return 6;
    if (pread(fd, ref, 8, 3) != 8 || memcmp(buf, ref, 8) != 0) return 7;
    close(fd);
    printf("ok\n");
    return 0;
}
"""


def test_header_compiles_as_c_and_links(tmp_path):
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    src = tmp_path / "abi.c"
    src.write_text(C_SOURCE)
    exe = tmp_path / "abi"
    libdir = os.path.dirname(_lib.LIB_PATH)
    cmd = ["gcc", "-std=c99", "-D_XOPEN_SOURCE=700", "-Wall", "-Werror", f"-I{os.path.join(ROOT, 'include')}",
           str(src), "-o", str(exe), f"-L{libdir}", f"-Wl,-rpath,{libdir}", "-l:libexl3b200.so"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", (run.returncode, run.stdout, run.stderr)
