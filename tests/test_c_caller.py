"""A plain C program calls libvrs through include/vrs.h only (no Python in
between): the binding the reference's Rust crate would add is an extern "C"
block over the same declarations. The CPU test compiles it and runs the
checks that need no GPU; the GPU test runs create/search/destroy and a
k-means fit as well."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_caller", "caller.c")


def _nccl_dir():
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        p = os.path.join(list(spec.submodule_search_locations)[0], "lib")
        if os.path.exists(os.path.join(p, "libnccl.so.2")):
            return p
    return None


@pytest.fixture(scope="module")
def caller(vc, tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    exe = str(tmp_path_factory.mktemp("c_caller") / "caller")
    libdir = os.path.dirname(vc.LIB_PATH)
    subprocess.run([cc, "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
                    "-o", exe, "-L", libdir, "-lvrs", "-lm", f"-Wl,-rpath,{libdir}"], check=True)
    env = dict(os.environ)
    nd = _nccl_dir()
    if nd:
        env["LD_LIBRARY_PATH"] = nd + os.pathsep + env.get("LD_LIBRARY_PATH", "")
    return exe, env


def test_c_caller_without_gpu(caller):
    exe, env = caller
    r = subprocess.run([exe], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ok cpu" in r.stdout


@pytest.mark.gpu
def test_c_caller_on_gpu(caller, gpu):
    exe, env = caller
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("ok gpu") == 2
