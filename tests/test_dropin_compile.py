"""The reference's own OlmoBlock (OlmoBlock.h:19 holds OlmoAttention by value;
OlmoBlock.cpp:6-40 constructs it from (folder, index) and calls forward,
backward, step and zero_grad) compiles unchanged against the drop-in
OlmoAttention.h.  Runs where the reference sources are present (this checks
the drop-in's source compatibility, it executes nothing)."""
import os
import shutil
import subprocess

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "dirktensor_b200", "cpp")


def test_reference_olmoblock_compiles_against_dropin(tmp_path):
    ref = oracle.reference_dir()
    if not os.path.exists(os.path.join(ref, "OlmoBlock.cpp")):
        pytest.skip("reference sources not present")
    # OlmoBlock.h includes "OlmoAttention.h" with quotes, which the compiler
    # resolves in OlmoBlock.h's own directory before any -I path.  The two
    # OlmoBlock files are therefore compiled from a scratch directory (left
    # unmodified), so that the lookup reaches the drop-in's header through -I.
    for f in ("OlmoBlock.h", "OlmoBlock.cpp"):
        shutil.copy(os.path.join(ref, f), tmp_path / f)
    cmd = ["g++", "-std=c++23", "-c", "-o", str(tmp_path / "OlmoBlock.o"),
           "-I", DROPIN, "-I", os.path.join(DROPIN, "compat"), "-I", ref, str(tmp_path / "OlmoBlock.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    # The object refers to the drop-in's OlmoAttention: the constructor and
    # forward OlmoBlock.cpp:6,14 calls, and the out-of-line destructor that only
    # the drop-in declares (the reference's class has an implicit inline one),
    # all as undefined symbols that libdirktensor_dropin.so provides.
    nm = subprocess.run(["nm", "-C", str(tmp_path / "OlmoBlock.o")], capture_output=True, text=True).stdout
    undefined = [ln.split(None, 1)[1] for ln in nm.splitlines() if ln.strip().startswith("U ")]
    for sym in ("OlmoAttention::OlmoAttention(", "OlmoAttention::forward(", "OlmoAttention::~OlmoAttention()"):
        assert any(u.startswith(sym) for u in undefined), sym
