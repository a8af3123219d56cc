"""Every name a function of the GPU-only drivers reads is defined somewhere it
can see (a parameter, a local, an enclosing function, the module or the
builtins).  These modules run only on a GPU box, so a misspelt or stale name
(a variable renamed in one function, read in another) would otherwise surface
only there.
"""

import ast
import builtins
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FILES = ["bench.py", "qevict_b200/microbench.py", "qevict_b200/model.py", "qevict_b200/tp_model.py",
         "qevict_b200/peer_sum.py", "qevict_b200/layer_state.py", "qevict_b200/hf.py", "qevict_b200/attention.py"]


def _bound_in(node):
    """Names bound directly in a function or module body (not in nested functions)."""
    names = set()
    if isinstance(node, (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda)):
        a = node.args
        for arg in a.posonlyargs + a.args + a.kwonlyargs:
            names.add(arg.arg)
        if a.vararg:
            names.add(a.vararg.arg)
        if a.kwarg:
            names.add(a.kwarg.arg)
    stack = list(node.body) if not isinstance(node, ast.Lambda) else [node.body]
    while stack:
        n = stack.pop()
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef)):
            names.add(n.name)
            continue
        if isinstance(n, ast.Lambda):
            continue
        if isinstance(n, ast.Name) and isinstance(n.ctx, (ast.Store, ast.Del)):
            names.add(n.id)
        elif isinstance(n, (ast.Import, ast.ImportFrom)):
            for al in n.names:
                names.add((al.asname or al.name).split(".")[0])
        elif isinstance(n, ast.ExceptHandler) and n.name:
            names.add(n.name)
        elif isinstance(n, (ast.Global, ast.Nonlocal)):
            names.update(n.names)
        stack.extend(ast.iter_child_nodes(n))
    return names


def _loads_in(node):
    """Names read directly in a function body (not in nested functions or classes)."""
    out = []
    stack = list(node.body) if not isinstance(node, ast.Lambda) else [node.body]
    while stack:
        n = stack.pop()
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.ClassDef, ast.Lambda)):
            # decorators and defaults are evaluated in this scope
            if not isinstance(n, ast.Lambda):
                stack.extend(n.decorator_list)
            if not isinstance(n, ast.ClassDef):
                stack.extend(n.args.defaults + [d for d in n.args.kw_defaults if d is not None])
            continue
        if isinstance(n, ast.Name) and isinstance(n.ctx, ast.Load):
            out.append((n.id, n.lineno))
        stack.extend(ast.iter_child_nodes(n))
    return out


def _comprehension_targets(node):
    names = set()
    for n in ast.walk(node):
        if isinstance(n, ast.comprehension):
            for t in ast.walk(n.target):
                if isinstance(t, ast.Name):
                    names.add(t.id)
    return names


def _check(tree):
    problems = []
    module_names = _bound_in(tree) | set(dir(builtins)) | {"__file__", "__name__"}

    def visit(fn, visible):
        scope = visible | _bound_in(fn) | _comprehension_targets(fn)
        for name, line in _loads_in(fn):
            if name not in scope:
                problems.append((name, line))
        for child in _direct_functions(fn):       # nested functions see this scope
            visit(child, scope)

    for f in _direct_functions(tree):
        visit(f, module_names)
    return problems


def _direct_functions(node):
    found = []
    stack = list(ast.iter_child_nodes(node))
    while stack:
        n = stack.pop()
        if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef, ast.Lambda)):
            found.append(n)
            continue
        stack.extend(ast.iter_child_nodes(n))
    return found


@pytest.mark.parametrize("path", FILES)
def test_every_read_name_is_defined(path):
    tree = ast.parse(open(os.path.join(ROOT, path)).read())
    problems = _check(tree)
    assert not problems, f"{path}: names read but never defined: {problems}"


def _self_attributes(cls):
    """Attributes a class defines or assigns to self anywhere in its methods."""
    import inspect
    import textwrap
    names = set(dir(cls))
    tree = ast.parse(textwrap.dedent(inspect.getsource(cls)))
    for n in ast.walk(tree):
        if (isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "self"
                and isinstance(n.ctx, ast.Store)):
            names.add(n.attr)
    return names


@pytest.mark.parametrize("func,cls", [("run_ours", "qevict_b200.model:StickyLlamaDecoder"),
                                      ("run_tp", "qevict_b200.tp_model:TpStickyLlamaDecoder")])
def test_bench_uses_only_attributes_the_decoder_has(func, cls):
    """Every `model.<name>` bench.py's driver reads exists on the decoder class it builds."""
    import importlib
    mod, name = cls.split(":")
    attrs = _self_attributes(getattr(importlib.import_module(mod), name))
    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == func)
    used = {(n.attr, n.lineno) for n in ast.walk(fn)
            if isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name) and n.value.id == "model"}
    missing = sorted((a, line) for a, line in used if a not in attrs)
    assert not missing, f"bench.py {func}: {name} has no {missing}"
