"""The one-file submission (fastqr.stage): the staged file is valid Python,
carries every CUDA source and the C header, and -- built from its embedded
sources with nvcc for sm_100a into a fresh cache, exactly as on first import
in the reference's evaluator -- yields a library exporting every symbol
include/fastqr.h declares.  CPU only: no kernel runs."""
import ast
import os
import re
import subprocess
import sys
from pathlib import Path

from fastqr import stage
from fastqr.build import CSRC, INCLUDE

ROOT = Path(__file__).resolve().parents[1]


def test_staged_file_carries_every_source(tmp_path):
    out = stage.stage(tmp_path / "submission.py")
    text = out.read_text()
    tree = ast.parse(text)
    names = {n.name for n in tree.body if isinstance(n, ast.FunctionDef)}
    assert "custom_kernel" in names
    embedded = stage.sources()
    for p in CSRC.iterdir():
        if p.suffix in (".cu", ".cuh", ".h"):
            assert embedded[f"x/csrc/{p.name}"] == p.read_text()
    assert embedded["include/fastqr.h"] == (INCLUDE / "fastqr.h").read_text()
    # no fallback: the code calls no torch.geqrf (the embedded sources are text)
    calls = [n for n in ast.walk(tree) if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute)
             and n.func.attr == "geqrf"]
    assert not calls


def test_staged_file_builds_the_library_from_its_sources(tmp_path):
    out = stage.stage(tmp_path / "submission.py")
    cache = tmp_path / "cache"
    env = dict(os.environ, FASTQR_CACHE=str(cache))
    env.pop("FASTQR_LIB", None)
    # importing the file builds (nvcc) and loads the library; nothing touches a GPU
    code = ("import importlib.util, sys; "
            f"s = importlib.util.spec_from_file_location('submission', {str(out)!r}); "
            "m = importlib.util.module_from_spec(s); s.loader.exec_module(m); print(m._lib._name)")
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=1500)
    assert res.returncode == 0, res.stderr[-3000:]
    so = Path(res.stdout.strip().splitlines()[-1])
    assert so.exists() and cache in so.parents
    declared = re.findall(r"^\s*(?:int|size_t|const char \*)\s*(fqr_\w+)\(", (INCLUDE / "fastqr.h").read_text(), re.M)
    syms = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    for name in declared:
        assert re.search(rf"\bT {name}$", syms, re.M), name
