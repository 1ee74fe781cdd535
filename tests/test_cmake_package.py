"""The CMake package contract (reference CMakeLists.txt:175-184 and
examples/library/CMakeLists.txt:1-5): this repository's CMake build installs
libkunlunk200.so.0 (version 0.7.12), the headers and a package exporting
KunlunK200::kunlunk200, so that a consumer project of the reference library
configures, builds and links unchanged with find_package(KunlunK200 CONFIG).

CPU only: configure, build and install into a temporary prefix; build a
consumer project against it and run what needs no GPU (kunlun::version());
build the reference's own examples/library project unchanged when the
reference checkout is present.  The GPU half runs the consumer that
`make -C oracle cmake-consumer` produced (tests/test_gpu_consumers.py).
"""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = os.environ.get("KUNLUN_REFERENCE_DIR", "/root/reference")

_CONSUMER = """cmake_minimum_required(VERSION 3.22)
project(k200_package_probe LANGUAGES CXX)
find_package(KunlunK200 {version} CONFIG REQUIRED)
add_executable(probe probe.cpp)
target_link_libraries(probe PRIVATE KunlunK200::kunlunk200)
"""
_PROBE = """#include <kunlun/k200.h>
#include <k200_c.h>
#include <cstdio>
#include <cstring>
int main() {
    std::printf("%s %s\\n", kunlun::version(), k200_version());
    return std::strcmp(kunlun::version(), "0.7.12") != 0;
}
"""


def _run(cmd, **kw):
    r = subprocess.run(cmd, capture_output=True, text=True, **kw)
    assert r.returncode == 0, f"{' '.join(map(str, cmd))}\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    return r


@pytest.fixture(scope="module")
def prefix(tmp_path_factory):
    if shutil.which("cmake") is None:
        pytest.skip("cmake is not installed")
    base = tmp_path_factory.mktemp("cmake")
    build, pre = base / "build", base / "prefix"
    _run(["cmake", "-S", ROOT, "-B", str(build), "-DCMAKE_BUILD_TYPE=Release"])
    _run(["cmake", "--build", str(build), "-j", "8"], timeout=900)
    _run(["cmake", "--install", str(build), "--prefix", str(pre)])
    return pre


def test_install_layout(prefix):
    lib = prefix / "lib"
    assert (lib / "libkunlunk200.so.0.7.12").exists()
    assert os.readlink(lib / "libkunlunk200.so.0") == "libkunlunk200.so.0.7.12"
    assert (prefix / "include" / "kunlun" / "k200.h").exists() and (prefix / "include" / "k200_c.h").exists()
    pkg = lib / "cmake" / "KunlunK200"
    for f in ("KunlunK200Config.cmake", "KunlunK200ConfigVersion.cmake", "KunlunK200Targets.cmake"):
        assert (pkg / f).exists(), f
    soname = _run(["readelf", "-d", str(lib / "libkunlunk200.so.0.7.12")]).stdout
    assert "[libkunlunk200.so.0]" in soname
    # the same entry points as the in-tree build
    ours = _run(["nm", "-D", "--defined-only", str(lib / "libkunlunk200.so.0.7.12")]).stdout
    intree = _run(["nm", "-D", "--defined-only", os.path.join(ROOT, "kunlunk200_lib_b200", "lib",
                                                             "libkunlunk200.so.0.7.12")]).stdout
    names = lambda out: {l.split()[-1] for l in out.splitlines() if l.strip()}  # noqa: E731
    assert names(ours) == names(intree)


@pytest.mark.parametrize("version,ok", [("0.1", True), ("0.7.12", True), ("", True), ("1.0", False)])
def test_find_package_versions(prefix, tmp_path, version, ok):
    """SameMajorVersion: any 0.x request up to 0.7.12 is satisfied, 1.0 is not."""
    (tmp_path / "CMakeLists.txt").write_text(_CONSUMER.format(version=version))
    (tmp_path / "probe.cpp").write_text(_PROBE)
    r = subprocess.run(["cmake", "-S", str(tmp_path), "-B", str(tmp_path / "b"),
                        f"-DKunlunK200_DIR={prefix / 'lib' / 'cmake' / 'KunlunK200'}"],
                       capture_output=True, text=True)
    assert (r.returncode == 0) == ok, r.stdout + r.stderr
    if ok:
        _run(["cmake", "--build", str(tmp_path / "b")])
        out = _run([str(tmp_path / "b" / "probe")]).stdout
        assert out.split() == ["0.7.12", "0.7.12"]


def test_reference_example_builds_unchanged(prefix, tmp_path):
    src = os.path.join(REFERENCE, "examples", "library")
    if not os.path.exists(os.path.join(src, "CMakeLists.txt")):
        pytest.skip("reference checkout not present")
    _run(["cmake", "-S", src, "-B", str(tmp_path / "b"),
          f"-DKunlunK200_DIR={prefix / 'lib' / 'cmake' / 'KunlunK200'}"])
    _run(["cmake", "--build", str(tmp_path / "b")])
    exe = tmp_path / "b" / "kunlun-consumer"
    assert exe.exists()
    ldd = _run(["ldd", str(exe)]).stdout
    assert f"libkunlunk200.so.0 => {prefix / 'lib'}" in ldd, ldd
