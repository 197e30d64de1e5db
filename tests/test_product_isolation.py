"""The product path never reaches the oracle: no file of the package imports, links or opens
anything under oracle/, and the library loader raises (no CPU fallback) when the CUDA library
is missing."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "math-plus_b200")


def test_package_never_names_the_oracle():
    pattern = re.compile(r"\boracle\b|liboracle|mp_oracle")
    hits = []
    for dirpath, _, files in os.walk(PKG):
        if "_build" in dirpath or "lib" == os.path.basename(dirpath):
            continue
        for fn in files:
            if fn.endswith((".py", ".cu", ".cuh", ".h", ".c", ".cpp")):
                path = os.path.join(dirpath, fn)
                with open(path, encoding="utf-8") as f:
                    for i, line in enumerate(f, 1):
                        if pattern.search(line):
                            hits.append(f"{os.path.relpath(path, ROOT)}:{i}: {line.strip()}")
    assert not hits, "\n".join(hits)
