"""The drop-in C++ boundary: code written against the reference's bag::cuda
API (include/bag/cuda/*.cuh) compiles with a host compiler and with nvcc,
links against libbag_b200.so, builds through the CMake bagConfig package, and
(on a GPU) computes C <- AB + C correctly."""

from __future__ import annotations

import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
SRC = os.path.join(ROOT, "tests", "cpp", "dropin_consumer.cpp")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
EXE = os.path.join(OUT_DIR, "dropin_consumer")


def build_consumer(lib_path: str) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    lib_dir = os.path.dirname(lib_path)
    subprocess.check_call(["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"),
                           "-I", os.path.join(CUDA, "include"), SRC, "-o", EXE,
                           "-L", lib_dir, "-lbag_b200", "-Wl,-rpath," + lib_dir,
                           "-L", os.path.join(CUDA, "lib64"), "-lcudart"])
    return EXE


def test_consumer_builds_with_host_compiler(built_lib):
    assert os.path.exists(build_consumer(built_lib))


def test_headers_compile_under_nvcc():
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "use.cu")
        with open(src, "w") as f:
            f.write('#include <bag/cuda/bag.cuh>\n'
                    'void use(const float* a, const float* b, float* c, cudaStream_t s) {\n'
                    '  bag_cuda::Workspace ws(64, 2, bag_cuda::Basis::Full);\n'
                    '  bag_cuda::matmul(a, b, c, 64, s, ws);\n'
                    '  strassen_cuda::primitive<-1, 0, -1, -1, true>(\n'
                    '      strassen_cuda::Backend::ColumnTile8, a, a, b, b, c, c, 32, 64, s);\n'
                    '  static_assert(sizeof(PrimBatchedPairArgs) == 12 * sizeof(void*), "");\n'
                    '}\n')
        subprocess.check_call([os.path.join(CUDA, "bin", "nvcc"), "-std=c++17", "-gencode",
                               "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "include"),
                               "-c", src, "-o", os.path.join(tmp, "use.o")])


@pytest.mark.skipif(shutil.which("cmake") is None, reason="cmake not installed")
def test_cmake_package_builds_a_downstream_consumer():
    """Build and install the package, then find_package(bag) from a new project."""
    with tempfile.TemporaryDirectory() as tmp:
        build, prefix = os.path.join(tmp, "build"), os.path.join(tmp, "prefix")
        gen = ["-G", "Ninja"] if shutil.which("ninja") else []
        subprocess.check_call(["cmake", "-S", ROOT, "-B", build, *gen, "-DBAG_BUILD_TESTS=OFF",
                               "-DCMAKE_BUILD_TYPE=Release"], stdout=subprocess.DEVNULL)
        subprocess.check_call(["cmake", "--build", build], stdout=subprocess.DEVNULL)
        subprocess.check_call(["cmake", "--install", build, "--prefix", prefix],
                              stdout=subprocess.DEVNULL)
        proj = os.path.join(tmp, "downstream")
        os.makedirs(proj)
        shutil.copy(SRC, os.path.join(proj, "main.cpp"))
        with open(os.path.join(proj, "CMakeLists.txt"), "w") as f:
            f.write("cmake_minimum_required(VERSION 3.24)\nproject(downstream LANGUAGES CXX)\n"
                    "find_package(bag 0.2 REQUIRED)\nadd_executable(app main.cpp)\n"
                    "target_link_libraries(app PRIVATE bag::cuda)\n")
        subprocess.check_call(["cmake", "-S", proj, "-B", os.path.join(proj, "b"), *gen,
                               f"-DCMAKE_PREFIX_PATH={prefix}"], stdout=subprocess.DEVNULL)
        subprocess.check_call(["cmake", "--build", os.path.join(proj, "b")],
                              stdout=subprocess.DEVNULL)
        assert os.path.exists(os.path.join(proj, "b", "app"))


@pytest.mark.gpu
def test_consumer_runs_on_gpu(built_lib, cuda):
    exe = build_consumer(built_lib)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "DROPIN OK" in out.stdout


@pytest.mark.gpu
def test_consumer_takes_tensor_leaves_from_environment(built_lib, cuda):
    """BAG_B200_MATH=3xtf32 switches a program that only calls the reference's
    API: at n = 2048 its depth-1 leaves (K = 1024) run on the tensor cores, its
    depth-2 leaves (K = 512) stay on FFMA, and every result passes the check."""
    exe = build_consumer(built_lib)
    env = dict(os.environ, BAG_B200_MATH="3xtf32")
    out = subprocess.run([exe, "2048"], capture_output=True, text=True, timeout=300, env=env)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "DROPIN OK" in out.stdout
    paths = [line.split() for line in out.stdout.splitlines() if line.startswith("depth=")]
    assert sorted(paths) == [["depth=1", "leaf_path=3xtf32"]] * 2 + [["depth=2", "leaf_path=ffma"]] * 2
    plain = subprocess.run([exe, "2048"], capture_output=True, text=True, timeout=300,
                           env={k: v for k, v in os.environ.items() if k != "BAG_B200_MATH"})
    assert plain.returncode == 0, plain.stdout + plain.stderr
    assert "leaf_path=3xtf32" not in plain.stdout
