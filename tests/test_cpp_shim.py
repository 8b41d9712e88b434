"""The C++ shim (include/wginfer_b200_nvidia.hpp) has the reference's
ops::nvidia signatures, links against the library and maps a bad call to the
reference's exception type. Runs without a GPU: the calls fail their argument
checks before any device work."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SRC = r'''
#include <cstdio>
#include <stdexcept>
#include "wginfer_b200_nvidia.hpp"
int main() {
    namespace nv = wginfer::ops::nvidia;
    int caught = 0;
    try { nv::linear(nullptr, nullptr, nullptr, nullptr, WGINFER_DTYPE_BF16, 1, 4, 4); }
    catch (const std::invalid_argument &) { caught++; }
    try { nv::rope(nullptr, nullptr, nullptr, WGINFER_DTYPE_BF16, 1, 1, 3, 1e4f); }
    catch (const std::invalid_argument &) { caught++; }
    std::byte *p = reinterpret_cast<std::byte *>(16);  // never dereferenced: the dtype check fails first
    try { nv::add(p, p, p, WGINFER_DTYPE_I64, 4); }
    catch (const std::runtime_error &) { caught++; }
    nv::swiglu(nullptr, nullptr, nullptr, WGINFER_DTYPE_BF16, 0);  // empty: a no-op
    std::printf("%d\n", caught);
    return caught == 3 ? 0 : 1;
}
'''


def test_cpp_shim_compiles_links_and_throws(tmp_path):
    lib = os.path.join(ROOT, "wginfer_b200", "libwginfer_b200.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    src = tmp_path / "shim.cpp"
    src.write_text(SRC)
    exe = tmp_path / "shim"
    subprocess.check_call(["g++", "-std=c++17", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                           lib, f"-Wl,-rpath,{os.path.dirname(lib)}"])
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip() == "3"
