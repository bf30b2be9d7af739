"""bench.py on the CPU: every name its functions read resolves (a typo or a variable
from the other arm would only fail on a machine with a GPU, after the timed region), and the
reference arm's JSON line has the contract's keys."""
import builtins
import importlib.util
import json
import symtable
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _load_bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _unresolved(table, module_names):
    bad = []
    for child in table.get_children():
        if child.get_type() == "function":
            for sym in child.get_symbols():
                if sym.is_global() and sym.is_referenced():
                    name = sym.get_name()
                    if name not in module_names and not hasattr(builtins, name):
                        bad.append(f"{child.get_name()}: {name}")
        bad += _unresolved(child, module_names)
    return bad


def test_every_name_in_bench_resolves():
    src = (ROOT / "bench.py").read_text()
    mod = _load_bench()
    top = symtable.symtable(src, "bench.py", "exec")
    assert _unresolved(top, set(vars(mod))) == []


def test_reference_record_contract():
    mod = _load_bench()
    rec = mod.reference_record(8, 3609.0, "no training path")
    json.dumps(rec)
    assert rec["impl"] == "reference" and rec["metric"] == mod.METRIC and rec["n_gpus"] == 8
    assert rec["dispatch_combine_us_per_layer"] == 3609.0 and rec["unavailable"] == "no training path"
    assert not any("planned" in k for k in rec)  # the planned placement is this framework's, not the reference's


def _static_unresolved(path: Path):
    """Names read inside functions that no module-level binding, global statement or
    builtin provides (static: the file is not imported)."""
    import ast

    src = path.read_text()
    top = symtable.symtable(src, str(path), "exec")
    defined = {s.get_name() for s in top.get_symbols() if s.is_assigned() or s.is_imported() or s.is_namespace()}
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, ast.Global):
            defined |= set(node.names)
    defined |= {"__file__", "__name__", "__doc__"}
    return [f"{path.relative_to(ROOT)}: {bad}" for bad in _unresolved(top, defined)]


def test_no_unresolved_names_in_gpu_only_code():
    """Covers the GPU tests too: they only execute on a machine with a GPU."""
    files = [ROOT / "bench.py", ROOT / "__graft_entry__.py", ROOT / "setup.py"]
    for d in ("spec_ep", "benchmarks", "examples", "visualization", "tests"):
        files += sorted((ROOT / d).rglob("*.py"))
    bad = [b for f in files for b in _static_unresolved(f)]
    assert bad == []


def test_no_undefined_self_attributes():
    """Inside every class of the package, benchmarks, examples and tests, each
    ``self.X`` that is read is assigned, defined or inherited somewhere (bases from
    this repository or torch's Module / autograd Function)."""
    import ast

    import torch

    external = {"nn.Module": set(dir(torch.nn.Module)), "torch.nn.Module": set(dir(torch.nn.Module)),
                "torch.autograd.Function": set(dir(torch.autograd.Function)), "RuntimeError": set(dir(RuntimeError)),
                "Exception": set(dir(Exception)), "NamedTuple": set(dir(tuple)), "object": set()}
    classes = {}
    for d in ("spec_ep", "benchmarks", "examples", "tests"):
        for f in sorted((ROOT / d).rglob("*.py")):
            for c in [n for n in ast.walk(ast.parse(f.read_text())) if isinstance(n, ast.ClassDef)]:
                own = {n.name for n in c.body if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))}
                for n in c.body:
                    for t in (n.targets if isinstance(n, ast.Assign) else [n.target] if isinstance(n, ast.AnnAssign) else []):
                        if isinstance(t, ast.Name):
                            own.add(t.id)
                for n in ast.walk(c):
                    if (isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "self"
                            and isinstance(n.ctx, (ast.Store, ast.Del))):
                        own.add(n.attr)
                bases = [b.id if isinstance(b, ast.Name) else ast.unparse(b) for b in c.bases]
                classes[c.name] = (own, bases, c, f)

    def defined(name, seen=()):
        if name in external:
            return external[name]
        own, bases, _, _ = classes[name]
        out = set(own)
        for b in bases:
            if b not in seen:
                out |= defined(b, seen + (name,))
        return out

    bad = []
    for name, (_, _, c, f) in classes.items():
        full = defined(name)
        for n in ast.walk(c):
            if (isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "self"
                    and isinstance(n.ctx, ast.Load) and n.attr not in full and not n.attr.startswith("__")):
                bad.append(f"{f.relative_to(ROOT)}:{n.lineno}: {name}.{n.attr}")
    assert len(classes) >= 40 and bad == []


def test_entry_points_parse_their_command_lines():
    """``--help`` of the benchmark, the training launcher and the CPU analysis tools exits
    0 without a GPU (argument parsing comes before any CUDA work)."""
    import subprocess
    import sys

    for cmd in (["bench.py"], ["-m", "spec_ep.run"], ["benchmarks/replay_routing.py"], ["benchmarks/roofline.py"]):
        r = subprocess.run([sys.executable, *cmd, "--help"], cwd=ROOT, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and "usage" in r.stdout, (cmd, r.stderr[-500:])
