"""Static check (CPU): every Python call into the sm_100a extension passes as many
arguments as the bound C++ function takes.

Bindings are plain function pointers without Python-side defaults, so a call with the
wrong count raises only when it runs, which for these paths is on a machine with a GPU. The C++
parameter lists come from the sources in csrc/ (free functions bound with ``m.def``,
``EpComm`` / ``SymmBuffer`` methods bound with ``.def``). The Python receivers tracked
are: ``load()``, names and attributes assigned from ``load()``, and names and
attributes assigned from ``<module>.EpComm(...)`` / ``<module>.SymmBuffer(...)``.
"""
import ast
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
CSRC = sorted((ROOT / "csrc").glob("*.c*")) + sorted((ROOT / "csrc").glob("*.h"))
CLASSES = ("EpComm", "SymmBuffer")


def _params(text: str, start: int) -> int:
    """Number of parameters of the parenthesised list opening at text[start]."""
    depth, i, n, seen = 0, start, 0, False
    while True:
        c = text[i]
        if c in "(<[{":
            depth += 1
            if depth == 1 and c == "(":
                i += 1
                continue
        elif c in ")>]}":
            depth -= 1
            if depth == 0:
                break
        elif c == "," and depth == 1:
            n += 1
        elif not c.isspace() and depth >= 1:
            seen = True
        i += 1
    body = text[start + 1:i].strip()
    return 0 if body in ("", "void") else n + 1 if seen else 0


def _strip_comments(s: str) -> str:
    s = re.sub(r"/\*.*?\*/", "", s, flags=re.S)
    return re.sub(r"//[^\n]*", "", s)


def _class_body(src: str, name: str):
    m = re.search(rf"\bclass\s+{name}\s*{{", src)
    if not m:
        return None
    i, depth = m.end() - 1, 0
    for j in range(i, len(src)):
        depth += {"{": 1, "}": -1}.get(src[j], 0)
        if depth == 0:
            return src[i:j]
    return None


TYPE = r"(?:void|bool|int|int64_t|double|float|auto|size_t|uint64_t|py::\w+|at::Tensor|torch::Tensor|std::[\w:<>, ]+)"


def _definition_arity(src: str, fname: str):
    for m in re.finditer(rf"(?m)^[ \t]*(?:static\s+|inline\s+)*{TYPE}[\s&\*]+{re.escape(fname)}\s*\(", src):
        return _params(src, m.end() - 1)
    return None


def cpp_arities():
    srcs = {p: _strip_comments(p.read_text()) for p in CSRC}
    free, methods = {}, {c: {} for c in CLASSES}
    for path, src in srcs.items():
        for m in re.finditer(r'm\.def\(\s*"(\w+)"\s*,\s*&([\w:]+)', src):
            free[m.group(1)] = (m.group(2).split("::")[-1], path)
        for cls in CLASSES:
            for m in re.finditer(rf'\.def\(\s*"(\w+)"\s*,\s*&{cls}::(\w+)', src):
                methods[cls][m.group(1)] = m.group(2)
    out_free = {}
    for name, (fn, bound_in) in free.items():
        # the bound wrapper lives beside its m.def; kernel launchers of the same name in
        # other files (namespace sepx) take different arguments
        for path in [bound_in] + [p for p in srcs if p != bound_in]:
            n = _definition_arity(srcs[path], fn)
            if n is not None:
                out_free[name] = n
                break
    out_methods = {c: {} for c in CLASSES}
    for cls, table in methods.items():
        body = next((b for b in (_class_body(s, cls) for s in srcs.values()) if b), None)
        assert body is not None, cls
        for name, fn in table.items():
            n = _definition_arity(body, fn)
            if n is not None:
                out_methods[cls][name] = n
    return out_free, out_methods


def _kind(node, names, attrs):
    """'module', a bound class name, or None for a receiver expression."""
    if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id == "load":
        return "module"
    if isinstance(node, ast.Name):
        return names.get(node.id)
    if isinstance(node, ast.Attribute):
        return attrs.get(node.attr)
    return None


def _assigned_kind(value, names, attrs):
    if isinstance(value, ast.Call) and isinstance(value.func, ast.Attribute) and value.func.attr in CLASSES:
        if _kind(value.func.value, names, attrs) == "module":
            return value.func.attr
    if _kind(value, names, attrs) == "module":
        return "module"
    return None


def python_calls():
    files = [ROOT / "bench.py", ROOT / "__graft_entry__.py"]
    for d in ("spec_ep", "benchmarks", "examples", "tests"):
        files += sorted((ROOT / d).rglob("*.py"))
    trees = {f: ast.parse(f.read_text()) for f in files}
    # attributes (self.X, obj.X) that hold the module or a bound object, across files
    attrs = {}

    def local_names(fn):
        names = {}
        for node in ast.walk(fn):
            if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
                k = _assigned_kind(node.value, names, attrs)
                if k:
                    names[node.targets[0].id] = k
        return names

    scopes = [(f, fn) for f, tree in trees.items()
              for fn in ast.walk(tree) if isinstance(fn, (ast.FunctionDef, ast.Module))]
    for _ in range(2):
        for _, fn in scopes:
            names = local_names(fn)
            for node in ast.walk(fn):
                if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Attribute):
                    k = _assigned_kind(node.value, names, attrs)
                    if k:
                        attrs[node.targets[0].attr] = k
    calls = []
    for f, fn in scopes:
        names = local_names(fn)
        for node in ast.walk(fn):
            if isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute):
                k = _kind(node.func.value, names, attrs)
                if k is None:
                    continue
                if any(isinstance(a, ast.Starred) for a in node.args) or any(kw.arg is None for kw in node.keywords):
                    continue
                calls.append((f"{f.relative_to(ROOT)}:{node.lineno}", k, node.func.attr,
                              len(node.args) + len(node.keywords)))
    return calls


def test_every_extension_call_matches_its_cpp_signature():
    free, methods = cpp_arities()
    assert len(free) >= 20 and len(methods["EpComm"]) >= 10 and len(methods["SymmBuffer"]) >= 5
    bad, checked = [], 0
    for where, kind, name, n in python_calls():
        table = free if kind == "module" else methods[kind]
        if name in CLASSES and kind == "module":
            continue  # constructors: checked by the py::init signatures at runtime
        if name not in table:
            continue
        checked += 1
        if table[name] != n:
            bad.append(f"{where}: {kind}.{name} called with {n} arguments, C++ takes {table[name]}")
    assert checked >= 60, checked
    assert bad == []
