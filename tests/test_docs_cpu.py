"""The documentation points at things that exist: every repository path in
the documents listed in ``DOCS`` (files, ``{a,b}`` groups, package-relative
module paths) and every ``tests/…py::test`` they cite."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DOCS = ["README.md", "DESIGN.md"]
PKG_DIRS = ("compression", "session", "transport", "engine", "connector", "store", "offline_search", "parallel",
            "ops", "utils", "models", "baselines")


def _expand(path: str) -> list:
    m = re.match(r"(.*)\{([^}]*)\}(.*)", path)
    if not m:
        return [path]
    return [m.group(1) + part + m.group(3) for part in m.group(2).split(",")]


def _basenames() -> set:
    names = set()
    for top in ("kvserve_b200", "csrc", "tests", "configs", "profiles"):
        for _, _, files in os.walk(os.path.join(ROOT, top)):
            names.update(files)
    return names


def _candidates(path: str) -> list:
    if "/" not in path:       # a bare file name, placed by the surrounding text
        return [path] if path in _basenames() else ["<none>"]
    if path.startswith(("kvserve_b200/", "csrc/", "tests/", "configs/", "profiles/")):
        return [path]
    if path.split("/")[0] in PKG_DIRS:
        return [os.path.join("kvserve_b200", path)]
    return []


@pytest.mark.parametrize("doc", DOCS)
def test_paths_in_docs_exist(doc):
    text = open(os.path.join(ROOT, doc), encoding="utf-8").read()
    missing = []
    for raw in re.findall(r"`([A-Za-z_][A-Za-z0-9_./{},*-]*\.(?:py|cu|cuh|h|md|json))`", text):
        if "*" in raw or raw.startswith("tests/test_pd_with_compression"):
            continue
        for p in _expand(raw):
            cands = _candidates(p)
            if "/" not in p:
                if cands == ["<none>"] and not os.path.exists(os.path.join(ROOT, p)):
                    missing.append(p)
                continue
            if cands and not any(os.path.exists(os.path.join(ROOT, c)) for c in cands):
                missing.append(p)
    for ref in re.findall(r"(tests/[a-z0-9_]+\.py)::([a-z0-9_]+)", text):
        path = os.path.join(ROOT, ref[0])
        if not os.path.exists(path) or f"def {ref[1]}" not in open(path, encoding="utf-8").read():
            missing.append("::".join(ref))
    assert not missing, missing
