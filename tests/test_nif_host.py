"""The Erlang NIF (c_src/tq4_nif.c) against the C ABI it binds, on a host without Erlang: it
compiles with gcc against include/tq4.h and a stub of the erl_nif.h declarations it uses
(tests/nif_stub/erl_nif.h), and links against libtq4.so with every tq4 symbol it calls resolved.
A real ERTS build is c_src/Makefile's (not run here)."""

import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NIF = os.path.join(ROOT, "c_src", "tq4_nif.c")
LIBDIR = os.path.join(ROOT, "transmuter_b200")


def test_nif_compiles_against_the_header(tmp_path):
    out = tmp_path / "tq4_nif.so"
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-shared", "-fPIC",
           "-I", os.path.join(ROOT, "tests", "nif_stub"), "-I", os.path.join(ROOT, "include"), NIF,
           "-o", str(out), "-L", LIBDIR, "-ltq4", "-Wl,--no-as-needed"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    syms = subprocess.run(["nm", "-D", str(out)], capture_output=True, text=True, check=True).stdout
    assert re.search(r" T nif_init$", syms, re.M)
    called = set(re.findall(r"\b(tq4_[a-z_]+)\(", open(NIF).read()))
    exported = subprocess.run(["nm", "-D", "--defined-only", os.path.join(LIBDIR, "libtq4.so")],
                              capture_output=True, text=True, check=True).stdout
    missing = [f for f in called if not re.search(rf" T {f}$", exported, re.M)]
    assert not missing, missing


def test_nif_functions_match_the_adapter():
    """Every NIF the Elixir module declares exists in the C table with the same arity."""
    table = dict((n, int(a)) for n, a in re.findall(r'\{"(\w+)", (\d+), \w+, \w+\}', open(NIF).read()))
    ex = open(os.path.join(ROOT, "lib", "transmuter", "cuda_q4", "nif.ex")).read()
    declared = {}
    for name, args in re.findall(r"def (\w+)\(([^)]*)\), do: :erlang\.nif_error", ex):
        declared[name] = len([a for a in args.split(",") if a.strip()])
    assert declared == table
