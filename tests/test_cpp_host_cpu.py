"""The C++ host side (astra-cuda_b200/cpp/: market.h's FillBatch, BBOBatch
and VecMarket, and the player-trading step, over the C ABI) builds, links,
and raises the reference's errors for bad constructor arguments; no GPU
needed."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def test_cpp_vec_market_builds_and_checks_arguments(tmp_path):
    from astra_cuda import _build
    lib = _build.build_cpp()
    inc, tlib = _build.torch_paths()
    exe = str(tmp_path / "vec_market_host_check")
    cmd = ["g++", "-std=c++17", "-O1", "-I", _build.INCLUDE_DIR, "-I", _build.CPP_DIR]
    for d in inc:
        cmd += ["-isystem", d]
    cmd += [os.path.join(HERE, "cpp", "vec_market_host_check.cpp"), "-o", exe,
            "-L", os.path.dirname(lib), "-lastra_vec_market", "-lastra_market",
            "-L", tlib, "-ltorch", "-ltorch_cpu", "-lc10",
            f"-Wl,-rpath,{os.path.dirname(lib)}", f"-Wl,-rpath,{tlib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-3000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
