"""include/tecoops.h from a plain C99 translation unit.

The reference's header (teco/interface/include/tecoops.h) is a C header; a C
program must be able to include this drop-in and link libteco_ops.so.  The test
compiles tests/c_api/handle_desc.c with gcc -std=c99 -Wall -Werror, twice: alone
(also -pedantic), and after <cuda_runtime.h> (the header's own cudaStream_t
typedef must not clash with the runtime's; CUDA's headers are not pedantic C99), links it against the library and runs it (host-only
calls: handle, stream, descriptors and the operators' argument checks).
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "teco-ops_b200", "tecoops")
SRC = os.path.join(ROOT, "tests", "c_api", "handle_desc.c")


@pytest.mark.parametrize("cuda_first", [False, True])
def test_c99_client_compiles_links_and_runs(tmp_path, cuda_first):
    if not os.path.exists(os.path.join(LIBDIR, "libteco_ops.so")):
        pytest.skip("libteco_ops.so not built")
    src = SRC
    if cuda_first:
        src = str(tmp_path / "cuda_first.c")
        with open(src, "w") as f:
            f.write("#include <cuda_runtime.h>\n")
            f.write(open(SRC).read())
    exe = str(tmp_path / "client")
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror"] + ([] if cuda_first else ["-pedantic"])
    cmd += ["-I" + os.path.join(ROOT, "include"),
           "-I/usr/local/cuda/include", src, "-o", exe, "-L" + LIBDIR, "-lteco_ops",
           "-Wl,-rpath," + LIBDIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "c99 client OK" in r.stdout


def _build_decode_step(tmp_path):
    exe = str(tmp_path / "decode_step")
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-O1", "-I" + os.path.join(ROOT, "include"),
           "-I/usr/local/cuda/include", os.path.join(ROOT, "tests", "c_api", "decode_step.c"),
           "-o", exe, "-L" + LIBDIR, "-lteco_ops", "-L/usr/local/cuda/lib64", "-lcudart", "-lm",
           "-Wl,-rpath," + LIBDIR, "-Wl,-rpath,/usr/local/cuda/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c99_gpu_client_compiles(tmp_path):
    """The GPU decode-step client below compiles and links as C99 (no GPU needed)."""
    if not os.path.exists(os.path.join(LIBDIR, "libteco_ops.so")):
        pytest.skip("libteco_ops.so not built")
    _build_decode_step(tmp_path)


@pytest.mark.gpu
def test_c99_gpu_client_runs_a_decode_step(tmp_path):
    """tests/c_api/decode_step.c: reshape_and_cache + flash_attention from plain C on the
    GPU, checked on the host against an fp32 loop within the attention tolerances."""
    exe = _build_decode_step(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "c99 gpu client OK" in r.stdout
