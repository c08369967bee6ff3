"""bench.py without a GPU: it imports, its argument parser accepts the driver's
flags, and every module-level name its functions read is defined (a missing
constant would only show up at the end of a GPU run)."""
import ast
import builtins
import importlib.util
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BENCH = os.path.join(ROOT, "bench.py")


def _load():
    spec = importlib.util.spec_from_file_location("bench_under_test", BENCH)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_bench_imports_and_parses_driver_flags(monkeypatch):
    mod = _load()
    monkeypatch.setattr(sys, "argv", ["bench.py", "--gpus", "1", "--steps", "3", "--warmup", "3"])
    args = mod.parse()
    assert args.steps == 3 and args.warmup == 3 and args.impl == "ours"
    monkeypatch.setattr(sys, "argv", ["bench.py", "--impl", "reference", "--only-mode", "unfused"])
    args = mod.parse()
    assert args.impl == "reference" and args.fused_only
    for name in ("WORKLOADS", "ALG_BYTES", "ALG_MUFU", "TRAFFIC_C2", "MUFU_PER_CELL", "MUFU_PER_SM_CLK"):
        assert hasattr(mod, name), name


def test_bench_has_no_undefined_globals():
    """Every bare name loaded inside bench.py is bound somewhere in the file
    (module level, a function's parameters or locals, a comprehension, an
    import) or is a builtin."""
    tree = ast.parse(open(BENCH).read())
    bound = set(dir(builtins)) | {"__file__", "__name__"}
    for node in ast.walk(tree):
        if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
            bound.add(node.name)
        if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda)):
            a = node.args
            for arg in a.args + a.kwonlyargs + a.posonlyargs + ([a.vararg] if a.vararg else []) + (
                    [a.kwarg] if a.kwarg else []):
                bound.add(arg.arg)
        elif isinstance(node, (ast.Import, ast.ImportFrom)):
            for alias in node.names:
                bound.add((alias.asname or alias.name).split(".")[0])
        elif isinstance(node, ast.Name) and isinstance(node.ctx, (ast.Store, ast.Del)):
            bound.add(node.id)
        elif isinstance(node, ast.ExceptHandler) and node.name:
            bound.add(node.name)
        elif isinstance(node, (ast.Global, ast.Nonlocal)):
            bound.update(node.names)
    loaded = {n.id for n in ast.walk(tree) if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Load)}
    assert loaded <= bound, sorted(loaded - bound)
