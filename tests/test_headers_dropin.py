"""The C++ headers under include/ as a drop-in for the reference's: its own
unit tests (tests/*.cpp of the reference tree, asserts on) compile against
include/ alone -- the reference's header names forward to include/aut/ --
and pass.  Needs the reference tree (read in place, nothing copied); skipped
where it is absent."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

REF = os.environ.get("AUT_REFERENCE_TREE", "/root/reference")
TESTS = ["storage_formats_test", "memory_accessor_test", "decoder_strategy_core_test",
         "bitwidth_benchmark_core_test", "lns_benchmark_core_test"]


@pytest.mark.parametrize("name", TESTS)
def test_reference_unit_test_compiles_and_passes_against_include(name, tmp_path):
    src = os.path.join(REF, "tests", name + ".cpp")
    if not os.path.exists(src):
        pytest.skip("reference tree not available on this machine")
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path / name)
    build = subprocess.run(["g++", "-O2", "-std=c++17", "-UNDEBUG", "-Wall",
                            "-I", os.path.join(ROOT, "include"), src, "-o", exe],
                           capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-4000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, (run.stdout[-2000:], run.stderr[-2000:])


def test_reference_inspector_reproduces_the_golden_csv(tmp_path):
    """The reference's own dataset inspector (tools/inspect_dot_dataset.cpp)
    built against include/dot_dataset.hpp prints the golden CSV that the
    reference's build of it printed."""
    src = os.path.join(REF, "tools", "inspect_dot_dataset.cpp")
    if not os.path.exists(src):
        pytest.skip("reference tree not available on this machine")
    exe = str(tmp_path / "inspect")
    build = subprocess.run(["g++", "-O3", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                            src, "-o", exe], capture_output=True, text=True)
    assert build.returncode == 0, build.stderr[-4000:]
    out = subprocess.run([exe, "1024", "65536", "1048576"], capture_output=True, text=True,
                         timeout=300).stdout
    with open(os.path.join(ROOT, "tests", "golden", "dot_v1_inspect.csv")) as f:
        assert out == f.read()


def test_headers_compile_for_the_device():
    """The same headers inside a CUDA translation unit for sm_100a."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    code = r'''
#include "storage_formats.hpp"
#include "memory_accessor.hpp"
#include "decoder_strategy_core.hpp"
#include "bitwidth_benchmark_core.hpp"
#include "lns_benchmark_core.hpp"
#include "dot_dataset.hpp"
namespace bw = aut::bitwidth;
__global__ void k(const unsigned *in, double *out, float *out32) {
  const unsigned r = in[threadIdx.x];
  out[threadIdx.x] = bw::decode_raw<aut::storage::e5m11, bw::compute_kind::fp64,
                                    bw::decoder_kind::direct_masked>(r) +
                     aut::lns::multiply_fused<aut::lns::lns16_r11, double>(r, r);
  out32[threadIdx.x] = bw::decode_raw<aut::storage::e8m5, bw::compute_kind::fp32,
                                      bw::decoder_kind::direct_branchy>(r);
}
'''
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "k.cu")
        with open(src, "w") as f:
            f.write(code)
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17",
                            "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
                            "-c", src, "-o", os.path.join(d, "k.o")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-4000:]
