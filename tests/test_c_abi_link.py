"""The drop-in boundary from a C caller's side: the public headers compile as C99 and as C++17,
and a C program built against them links with libpyxis_cuda.so and calls it (the ABI version,
the no-device answer of pyxis_cuda_init, the host-side argument checks).  Runs without a GPU."""
import glob
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
LIBDIR = os.path.join(ROOT, "pyxis_b200")
HEADERS = sorted(glob.glob(os.path.join(INC, "*.h")))

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "pyxis_cuda.h"
#include "pyxis_decode.h"
#include "pyxis_synth.h"

int main(void) {
    if ((pyxis_cuda_abi_version() >> 16) != 1) return 10;
    pyxis_cuda_ctx *ctx = NULL;
    int rc = pyxis_cuda_init(0, &ctx);
    if (rc == PYXIS_OK) {            /* a B200 is visible: the context must be usable */
        if (!ctx || pyxis_cuda_destroy(ctx) != PYXIS_OK) return 11;
    } else if (rc != PYXIS_ENODEV || ctx != NULL || strlen(pyxis_cuda_last_error()) == 0) {
        return 12;                   /* no device: ENODEV and a message, nothing allocated */
    }
    if (pyxis_cuda_matmul(NULL, NULL, NULL, 1, 1, NULL) != PYXIS_EINVAL) return 13;
    if (pyxis_cuda_weights_free(NULL) != PYXIS_OK) return 14;
    float v[4] = {0, 0, 0, 0};
    pyxis_synth_normal_f32(7, 4, 1.0f, v);
    if (v[0] == 0.0f && v[1] == 0.0f) return 15;
    printf("c-abi ok %d\n", rc);
    return 0;
}
"""


def _compiler(name):
    path = shutil.which(name)
    if not path:
        pytest.skip(f"{name} not available")
    return path


@pytest.mark.parametrize("header", [os.path.basename(h) for h in HEADERS])
@pytest.mark.parametrize("lang", ["c", "c++"])
def test_header_compiles(header, lang):
    cc = _compiler("gcc" if lang == "c" else "g++")
    std = ["-std=c99", "-pedantic"] if lang == "c" else ["-std=c++17"]
    r = subprocess.run([cc, *std, "-Wall", "-Wextra", "-Werror", "-fsyntax-only", "-x", lang,
                        os.path.join(INC, header)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_c_program_links_and_runs():
    cc = _compiler("gcc")
    lib = os.path.join(LIBDIR, "libpyxis_cuda.so")
    if not os.path.exists(lib):
        pytest.skip("libpyxis_cuda.so not built")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "caller.c"), os.path.join(d, "caller")
        with open(src, "w") as f:
            f.write(PROGRAM)
        r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", INC, src, "-o", exe, "-L", LIBDIR,
                            "-lpyxis_cuda", f"-Wl,-rpath,{LIBDIR}"], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and "c-abi ok" in r.stdout, (r.returncode, r.stdout, r.stderr)
