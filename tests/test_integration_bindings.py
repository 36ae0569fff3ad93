"""The Rust declarations that INTEGRATION.md gives a maintainer match the C headers: every entry
point of include/*.h outside the graph layer has a `pub fn` with the same parameters (count,
integer types, pointer depth and constness), and every `pub fn` is declared.  The graph layer
(pcu_b200_graph_*, pcu_b200_prepared_*) is for hosts without the reference's own graph, so the
Rust side does not bind it.  No GPU needed."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _params(params):
    params = params.strip()
    if params in ("", "void"):
        return []
    return [p.strip() for p in params.split(",")]


_INTEGERS = {"int": ("c_int",), "int32_t": ("i32", "c_int"), "uint32_t": ("u32",), "uint64_t": ("u64",),
             "size_t": ("usize",)}


def _agree(c_param, rust_param):
    """One C parameter and its Rust counterpart have the same type."""
    rust_type = rust_param.split(":", 1)[1].strip()
    depth = c_param.count("*")
    if depth != rust_type.count("*const") + rust_type.count("*mut"):
        return False
    if depth == 0:
        return rust_type in _INTEGERS.get(c_param.split()[0], ())
    if depth == 1:  # the pointee's constness
        return rust_type.startswith("*const") == c_param.startswith("const")
    return True


def _c_declarations():
    decls = {}
    for header in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not header.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
        text = re.sub(r"//[^\n]*", " ", text)
        for name, params in re.findall(r"\b(pcu_b200_\w+)\s*\(([^;{}]*?)\)\s*;", text, flags=re.S):
            decls[name] = _params(params)
    return decls


def _rust_declarations():
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    return {name: _params(params)
            for name, params in re.findall(r"pub fn (pcu_b200_\w+)\s*\(([^)]*)\)", text, flags=re.S)}


def test_rust_bindings_match_the_headers():
    c, rust = _c_declarations(), _rust_declarations()
    assert len(c) > 40, sorted(c)  # the parse found the headers' declarations
    bound = {n: k for n, k in c.items() if not n.startswith(("pcu_b200_graph_", "pcu_b200_prepared_"))}
    missing = sorted(set(bound) - set(rust))
    assert not missing, missing
    undeclared = sorted(set(rust) - set(c))
    assert not undeclared, undeclared
    wrong = sorted(n for n in rust if len(c[n]) != len(rust[n]))
    assert not wrong, wrong
    mismatched = [(n, cp, rp) for n in sorted(rust) for cp, rp in zip(c[n], rust[n]) if not _agree(cp, rp)]
    assert not mismatched, mismatched
