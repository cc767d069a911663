"""include/qmm.h from plain C: a C99 program that includes only the header,
compiled with -Wall -Werror -pedantic and linked against libqmm_b200.so, calls
the host-side entry points the way a Zig @cImport / cgo caller would - spec
inference on the reference's own shape cases (src/weights.zig:493-541), the
mode strings, argument resolution, an error through the latch, and the
stateless operator's validation.  No GPU is used."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "mlx-runner_b200", "_build")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "qmm.h"

static int spec_of(const char* wname, int wdtype, int64_t w0, int64_t w1,
                   const char* sname, int sdtype, int64_t s0, int64_t s1, qmm_quant_spec* out) {
    const int64_t wshape[2] = {w0, w1}, sshape[2] = {s0, s1};
    qmm_tensor_info infos[2];
    infos[0].name = wname; infos[0].dtype = wdtype; infos[0].ndim = 2; infos[0].shape = wshape;
    infos[1].name = sname; infos[1].dtype = sdtype; infos[1].ndim = 2; infos[1].shape = sshape;
    return qmm_infer_quant_spec(infos, sname ? 2 : 1, out);
}

int main(void) {
    qmm_quant_spec spec;
    char msg[256];
    qmm_optional_int none = {0, false}, g16 = {16, true};
    int rc;
    printf("abi %d\n", qmm_abi_version());
    rc = spec_of("l.q.weight", QMM_DTYPE_U32, 8, 8, "l.q.scales", QMM_DTYPE_U8, 8, 4, &spec);
    printf("nvfp4 %d %s %d %d\n", rc, qmm_mode_str(spec), spec.group_size, spec.bits);
    rc = spec_of("l.q.weight", QMM_DTYPE_U32, 8, 32, "l.q.scales", QMM_DTYPE_U8, 8, 4, &spec);
    printf("mxfp8 %d %s %d %d\n", rc, qmm_mode_str(spec), spec.group_size, spec.bits);
    rc = spec_of("l.q.weight", QMM_DTYPE_U32, 8, 32, "l.q.scales", QMM_DTYPE_BF16, 8, 2, &spec);
    printf("affine %d\n", rc);
    rc = spec_of("l.q.weight", QMM_DTYPE_U32, 8, 32, NULL, 0, 0, 0, &spec);
    printf("orphan %d\n", rc);
    rc = qmm_spec_from_args(g16, none, "nvfp4", &spec);
    printf("args %d %d %d\n", rc, spec.group_size, spec.bits);
    rc = qmm_spec_from_args(none, none, "affine", &spec);
    printf("badmode %d pending %d\n", rc, qmm_error_pending());
    rc = qmm_last_error(msg, sizeof msg);
    printf("latched %d %d cleared %d\n", rc, (int)(strlen(msg) > 0), qmm_error_pending());
    rc = qmm_quantized_matmul((void*)0x100000, 8, (const void*)0x100000, 1, 32, 32, (const uint32_t*)0x100000,
                              8, 8, (const uint8_t*)0x100000, 8, 1, NULL, false, none, none, "mxfp8", NULL);
    printf("transpose %d\n", rc);
    qmm_last_error(msg, sizeof msg);
    return 0;
}
"""


def test_header_compiles_as_c99_and_links():
    cc = shutil.which("gcc")
    lib = os.path.join(LIBDIR, "libqmm_b200.so")
    if cc is None or not os.path.exists(lib):
        pytest.skip("gcc or the built library is missing")
    d = tempfile.mkdtemp(prefix="qmm_c_")
    try:
        src, exe = os.path.join(d, "prog.c"), os.path.join(d, "prog")
        with open(src, "w") as f:
            f.write(PROGRAM)
        subprocess.check_call([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                               f"-I{os.path.join(ROOT, 'include')}", src, "-o", exe, f"-L{LIBDIR}", "-lqmm_b200",
                               f"-Wl,-rpath,{LIBDIR}"])
        out = subprocess.run([exe], capture_output=True, text=True, timeout=120, check=True).stdout.split("\n")
    finally:
        shutil.rmtree(d, ignore_errors=True)
    assert out[0] == "abi 1"
    assert out[1] == "nvfp4 0 nvfp4 16 4"
    assert out[2] == "mxfp8 0 mxfp8 32 8"
    assert out[3] == "affine 4"            # QMM_ERR_AFFINE_UNSUPPORTED
    assert out[4] == "orphan 2"            # QMM_ERR_NONSTANDARD_QUANT
    assert out[5] == "args 0 16 4"
    assert out[6] == "badmode 6 pending 1"
    assert out[7] == "latched 4 1 cleared 0"  # the first failure since the last read wins
    assert out[8] == "transpose 7"         # QMM_ERR_BAD_ARGUMENT
