"""The static archive as a non-Python host links it: tests/host_link/d1_host.c binds the C ABI of
include/d1kernels.h the way the reference's Rust host binds its kernels (src/cuda.rs:102-175, linked as
build.rs:11-40 links the archive it builds), with the CUDA runtime and libstdc++ only: no Python, torch or cuBLAS.

* CPU: it compiles and links against libd1kernels.a, and the executable needs no library beyond the CUDA runtime
  and the C/C++ runtimes.
* GPU: it runs one attention layer's chain (RMSNorm -> tuned QKV GEMM -> d1_flash_attn with the reference's
  64-row work list) and checks each step on the host in double precision.
"""
import shutil
import subprocess
from pathlib import Path

import pytest

from conftest import PKG_DIR, ROOT

SRC = ROOT / "tests" / "host_link" / "d1_host.c"
ARCHIVE = PKG_DIR / "libd1kernels.a"
CUDA = Path("/usr/local/cuda")
ALLOWED = ("libcudart.so", "libstdc++.so", "libm.so", "libgcc_s.so", "libc.so", "ld-linux", "libdl.so",
           "libpthread.so", "librt.so")


def _build(out_dir):
    if not ARCHIVE.exists():
        pytest.skip("libd1kernels.a not built (python fast-d1-omni_b200/build.py)")
    cc = shutil.which("gcc")
    if cc is None or not (CUDA / "include" / "cuda_runtime_api.h").exists():
        pytest.skip("gcc or the CUDA headers are missing")
    exe = Path(out_dir) / "d1_host"
    cmd = [cc, "-std=c11", "-O2", "-Wall", "-Werror", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", str(SRC),
           str(ARCHIVE), f"-L{CUDA / 'lib64'}", "-lcudart", "-lstdc++", "-ldl", "-lm", "-lpthread", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_archive_links_into_a_c_host(tmp_path):
    exe = _build(tmp_path)
    needed = subprocess.run(["readelf", "-d", str(exe)], capture_output=True, text=True).stdout
    libs = [ln.split("[")[1].rstrip("]") for ln in needed.splitlines() if "(NEEDED)" in ln]
    assert libs and all(any(lib.startswith(a) for a in ALLOWED) for lib in libs), libs


@pytest.mark.gpu
def test_c_host_runs_the_attention_chain(tmp_path, gpu_lib):
    exe = _build(tmp_path)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
