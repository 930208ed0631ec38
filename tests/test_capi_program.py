"""The C ABI from a compiled C++ host: tests/capi/learn_runtime.cpp includes
include/heliox_b200.h and runs the LearnRuntime-shaped sequence (hx_create ->
hx_load_group -> hx_forward_capture -> hx_backward -> hx_reduce_grads_f32,
LearnRuntime.h:72-100's simulate_and_adjoint_into shape).  CPU: it compiles
and links against the library.  GPU: its trace and reduced gradient columns
match the oracle (voltages within 1e-9 of the trace scale; the float32
columns within 1e-6 of the largest)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "capi", "learn_runtime.cpp")
OUT_DIR = os.path.join(ROOT, "tests", "capi", "_build")
EXE = os.path.join(OUT_DIR, "learn_runtime")


def _compile():
    from heliox_b200 import build

    build.build()
    os.makedirs(OUT_DIR, exist_ok=True)
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    cmd = [cxx, "-std=c++20", "-O2", "-Wall", "-I" + os.path.join(ROOT, "include"), SRC, "-o", EXE,
           "-L" + os.path.join(ROOT, "heliox_b200"), "-lhx_b200", "-Wl,-rpath,$ORIGIN/../../../heliox_b200"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return EXE


def test_cpp_host_compiles_against_header():
    exe = _compile()
    assert os.access(exe, os.X_OK)
    # no GPU here: the program loads the library and fails loudly at hx_create
    # (or answers its usage line) instead of running anything on the host
    r = subprocess.run([exe], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr


def _write_case(path, g, T, probes, dLtdv, kind, index, dest, scale, N):
    i32 = lambda x: np.ascontiguousarray(x, dtype=np.int32).tobytes()  # noqa: E731
    f64 = lambda x: np.ascontiguousarray(x, dtype=np.float64).tobytes()  # noqa: E731
    hh, pas, ic = g.hh, g.pas, g.iclamp
    with open(path, "wb") as f:
        f.write(i32([g.ncell, g.nnode, hh.n, pas.n, ic.n, T, len(probes), len(kind)]))
        f.write(f64([g.celsius, g.dt, g.v_init]))
        f.write(i32(g.parent))
        for x in (g.a, g.b, g.area, g.cm):
            f.write(f64(x))
        f.write(i32(hh.nodes))
        for k in ("gnabar", "gkbar", "gl", "el", "ena", "ek"):
            f.write(f64(hh.fields[k]))
        f.write(i32(pas.nodes))
        for k in ("g", "e"):
            f.write(f64(pas.fields[k]))
        f.write(i32(ic.nodes))
        for k in ("del", "dur", "amp"):
            f.write(f64(ic.fields[k]))
        f.write(i32(probes))
        f.write(np.ascontiguousarray(dLtdv, dtype=np.float32).tobytes())
        f.write(i32(kind) + i32(index) + i32(dest))
        f.write(np.ascontiguousarray(scale, dtype=np.float32).tobytes())
        f.write(i32([N]))


@pytest.mark.gpu
def test_cpp_host_matches_oracle(tmp_path):
    from heliox_b200 import _lib, synth
    from oracle import oracle as O

    exe = _compile()
    g = synth.random_tree_batch(3, seed0=31, nmin=80, nmax=150)
    T = 2000
    probes = g.soma_nodes()
    dLtdv = (np.random.default_rng(2).standard_normal((T, probes.shape[0])) * 1e-3).astype(np.float32)
    # columns: every hh gnabar instance into column (instance % 5), pas.g into 5 + (instance % 3)
    kinds = [_lib.HX_P["hh.gnabar"]] * g.hh.n + [_lib.HX_P["pas.g"]] * g.pas.n
    index = list(range(g.hh.n)) + list(range(g.pas.n))
    dest = [i % 5 for i in range(g.hh.n)] + [5 + i % 3 for i in range(g.pas.n)]
    scale = np.linspace(0.5, 1.5, len(kinds)).astype(np.float32)
    N = 8
    case, out = str(tmp_path / "case.bin"), str(tmp_path / "out.bin")
    _write_case(case, g, T, probes, dLtdv, kinds, index, dest, scale, N)
    r = subprocess.run([exe, case, out], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    raw = open(out, "rb").read()
    nt = (T + 1) * probes.shape[0]
    trace = np.frombuffer(raw[: 8 * nt], dtype=np.float64).reshape(T + 1, -1)
    dw = np.frombuffer(raw[8 * nt:], dtype=np.float32)
    dl = np.zeros((T + 1, probes.shape[0]))
    dl[1:] = dLtdv.astype(np.float64)
    ref, gr = O.adjoint(g, T, dl)
    assert np.max(np.abs(trace - ref)) / np.max(np.abs(ref)) <= 1e-9
    want = np.zeros(N)
    np.add.at(want, np.array(dest), scale.astype(np.float64) * np.concatenate([gr["hh.gnabar"], gr["pas.g"]]))
    assert np.max(np.abs(dw - want)) <= 1e-6 * np.max(np.abs(want))
