"""The reference-named C++ host-code API (include/bsp/host_code.hpp) compiled
into a driver that mirrors the reference's own test drivers."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tenstorrent-wh-blockspmm_b200")
ORACLE = os.path.join(ROOT, "oracle")


def _build(tmp_path):
    exe = str(tmp_path / "test_host_code")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Werror", f"-I{ROOT}/include", f"-I{ORACLE}",
           os.path.join(ROOT, "tests", "cpp", "test_host_code.cpp"), f"-L{PKG}", "-lbsp",
           f"-L{ORACLE}", "-loracle", f"-Wl,-rpath,{PKG}", f"-Wl,-rpath,{ORACLE}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_host_code_header_compiles(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
def test_host_code_registries_on_gpu(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout
    assert r.stdout.count("PASS") >= 6 * 6 + 10 * 3 + 3 + 1
    assert "bsp::spgemm" in r.stdout and "bsp::attention_step" in r.stdout
    assert r.stdout.count("PASS bsr_sddmm_multicore_SnF") == 10


def _build_prog(tmp_path, src, libs):
    exe = str(tmp_path / os.path.splitext(os.path.basename(src))[0])
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Werror", f"-I{ROOT}/include", f"-I{ORACLE}",
           os.path.join(ROOT, "tests", "cpp", src), "-pthread"] + libs + ["-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_container_goldens_match_oracle(tmp_path):
    """The containers' own CPU products (spmm_bfloat16, omp_spmm_bf16, spmm,
    sddmm, spgemm) give the oracle's bits, on the CPU."""
    exe = _build_prog(tmp_path, "test_container_golden.cpp",
                      [f"-L{ORACLE}", "-loracle", f"-Wl,-rpath,{ORACLE}"])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and r.stdout.count("PASS") >= 18


def test_reference_driver_compiles(tmp_path):
    _build_prog(tmp_path, "test_reference_driver.cpp", [f"-L{PKG}", "-lbsp", f"-Wl,-rpath,{PKG}"])


@pytest.mark.gpu
def test_reference_shaped_driver_on_gpu(tmp_path):
    """A driver shaped like the reference's test_block_spmm.cpp / test_sddmm.cpp
    (host golden from the container, registry host functions, PCC) plus the
    buffer helpers and bsp_bsr_upload through the C ABI."""
    exe = _build_prog(tmp_path, "test_reference_driver.cpp", [f"-L{PKG}", "-lbsp", f"-Wl,-rpath,{PKG}"])
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:])
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr
    assert "FAIL" not in r.stdout
    assert r.stdout.count("PASS") == 6 * 4 + 2 + 2
