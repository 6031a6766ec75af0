"""The exp used by both samplers (csrc/wcb_exp.h: Cody-Waite reduction and a
degree-7 Taylor polynomial in a fixed sequence of IEEE f32 operations), built for
the host with g++ and checked against float64 exp: within 1.5 ulp on [-87, 0],
exact at 0, monotone, and the documented edge values (x > 0 clamps to 1;
x < -87 and NaN give 0). The device build runs the same operation sequence
(__fmul_rn / __fadd_rn), and the device sampler draws the host sampler's tokens."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "wasm-chord_b200", "csrc")


@pytest.fixture(scope="module")
def wexp(tmp_path_factory):
    cxx = shutil.which(os.environ.get("CXX", "g++"))
    if cxx is None:
        pytest.skip("no C++ compiler")
    d = tmp_path_factory.mktemp("wexp")
    src = d / "wexp.cpp"
    src.write_text('#include "wcb_exp.h"\n'
                   'extern "C" void wexp(const float* x, float* y, long n) {\n'
                   '  for (long i = 0; i < n; ++i) y[i] = wcb::wcb_exp_nonpos(x[i]);\n}\n')
    lib = d / "libwexp.so"
    subprocess.run([cxx, "-O2", "-ffp-contract=off", "-std=c++17", "-shared", "-fPIC", "-I", CSRC, "-o", str(lib),
                    str(src)], check=True)
    L = ctypes.CDLL(str(lib))

    def run(x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        L.wexp(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), ctypes.c_long(x.size))
        return y
    return run


def test_within_one_and_a_half_ulp_on_the_sampling_range(wexp):
    x = -np.linspace(0.0, 87.0, 2_000_001).astype(np.float32)
    y = wexp(x)
    ref = np.exp(x.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    err = np.abs(y.astype(np.float64) - ref) / ulp
    assert err.max() <= 1.5, err.max()
    assert np.all(np.diff(y) <= 0)  # monotone: a larger logit never gets a smaller weight


def test_edge_values(wexp):
    x = np.array([0.0, -0.0, 1e-30, 0.5, 1e30, np.inf, -87.0001, -88.0, -1e30, -np.inf, np.nan], np.float32)
    y = wexp(x)
    assert list(y[:6]) == [1.0] * 6
    assert list(y[6:]) == [0.0] * 5
    assert wexp(np.array([-np.log(2.0)], np.float32))[0] == np.float32(0.5)
