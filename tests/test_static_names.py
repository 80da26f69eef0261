"""A lint lane without a linter: every name a function reads must be bound somewhere (its own scope,
an enclosing one, the module or builtins). The GPU-only Python paths never run in the CPU suite, so a
misspelt name there would otherwise wait for a GPU box to be found.
Reference: Makefile:8-11 (ruff E9, F63, F7, F82 as the lint lane)."""
import builtins
import pathlib
import symtable

ROOT = pathlib.Path(__file__).resolve().parent.parent
IMPLICIT = {"__class__", "__file__", "__name__", "__doc__", "__builtins__", "__spec__", "__package__"}


def undefined_names(path: pathlib.Path):
    top = symtable.symtable(path.read_text(), str(path), "exec")
    module_names = set(top.get_identifiers())
    found = []

    def ok(name: str) -> bool:
        return name in module_names or hasattr(builtins, name) or name in IMPLICIT

    def walk(table):
        for sym in table.get_symbols():
            if table.get_type() != "module" and sym.is_referenced() and sym.is_global() and not sym.is_declared_global():
                if not ok(sym.get_name()):
                    found.append((table.get_name(), table.get_lineno(), sym.get_name()))
        for child in table.get_children():
            walk(child)

    for sym in top.get_symbols():
        if sym.is_referenced() and not (sym.is_assigned() or sym.is_imported() or sym.is_namespace()):
            if not (hasattr(builtins, sym.get_name()) or sym.get_name() in IMPLICIT):
                found.append(("<module>", 0, sym.get_name()))
    walk(top)
    return found


def test_no_function_reads_an_unbound_name():
    files = sorted((ROOT / "fastafd_b200").rglob("*.py")) + [ROOT / "bench.py", ROOT / "__graft_entry__.py",
                                                             ROOT / "baseline" / "reference_arm.py"]
    assert len(files) > 40
    bad = {str(f.relative_to(ROOT)): undefined_names(f) for f in files}
    bad = {k: v for k, v in bad.items() if v}
    assert not bad, bad


def test_the_check_sees_an_unbound_name(tmp_path):
    p = tmp_path / "m.py"
    p.write_text("import os\n\ndef f(x):\n    return os.path.join(x, missing_name)\n")
    assert undefined_names(p) == [("f", 3, "missing_name")]
