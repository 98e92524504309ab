"""include/pf_b200.h is a C header: a C99 program that includes it compiles
without warnings, links against the shared library and gets a status back
from it (no GPU needed: a call with a bad argument is refused either way)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <stdio.h>
#include "pf_b200.h"

int main(void) {
    int8_t q[4];
    float x[4] = {1.0f, -2.0f, 0.5f, 0.0f}, s[1];
    pf_status bad = pf_quantize_activation_rows(x, q, s, -1, 4, NULL);  /* M < 0 */
    const char* msg = pf_last_error();
    printf("devices %d\nstatus %d\nmessage %s\n", (int)pf_device_count(), (int)bad, msg ? msg : "");
    return (bad == PF_ERR_NO_DEVICE || bad == PF_ERR_INVALID) ? 0 : 1;
}
"""


def test_header_compiles_as_c_and_links(tmp_path):
    lib = os.path.join(ROOT, "pocketforge_b200", "libpf_b200.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I" + os.path.join(ROOT, "include"),
                    str(src), "-o", str(exe), "-L" + os.path.dirname(lib), "-l:libpf_b200.so",
                    "-Wl,-rpath," + os.path.dirname(lib)], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "status" in out.stdout and "message" in out.stdout
