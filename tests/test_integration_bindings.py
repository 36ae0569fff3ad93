"""The Rust declarations that INTEGRATION.md gives a maintainer match the C headers: every entry
point of include/*.h outside the graph layer has a `pub fn` with the same number of parameters,
and every `pub fn` is declared.  The graph layer (pcu_b200_graph_*, pcu_b200_prepared_*) is for
hosts without the reference's own graph, so the Rust side does not bind it.  No GPU needed."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _param_count(params):
    params = params.strip()
    if params in ("", "void"):
        return 0
    return params.count(",") + 1


def _c_declarations():
    decls = {}
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
        text = re.sub(r"//[^\n]*", " ", text)
        for name, params in re.findall(r"\b(pcu_b200_\w+)\s*\(([^;{}]*?)\)\s*;", text, flags=re.S):
            decls[name] = _param_count(params)
    return decls


def _rust_declarations():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return {name: _param_count(params)
            for name, params in re.findall(r"pub fn (pcu_b200_\w+)\s*\(([^)]*)\)", text, flags=re.S)}


def test_rust_bindings_match_the_headers():
    c, rust = _c_declarations(), _rust_declarations()
    assert len(c) > 40, sorted(c)  # the parse found the headers' declarations
    bound = {n: k for n, k in c.items() if not n.startswith(("pcu_b200_graph_", "pcu_b200_prepared_"))}
    missing = sorted(set(bound) - set(rust))
    assert not missing, missing
    undeclared = sorted(set(rust) - set(c))
    assert not undeclared, undeclared
    wrong = sorted((n, c[n], rust[n]) for n in rust if c[n] != rust[n])
    assert not wrong, wrong
