"""Static contracts on the CUDA / C++ sources (no GPU): every entry point that Python binds
exists in the sources, device code cannot trap or spin without a bound, and nothing that is
closed on the target machines is named."""
import re
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parent.parent / "fastafd_b200" / "csrc"
CUDA_FILES = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h"))
ALL_FILES = CUDA_FILES + sorted(CSRC.glob("*/*.cpp"))


def _code(path: Path) -> str:
    """Source without comments (contracts are about code, not prose)."""
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def test_every_bound_symbol_is_defined_in_the_sources():
    from fastafd_b200.ops import _lib

    defined = set()
    for f in ALL_FILES:
        defined |= set(re.findall(r"\b(afd_[a-z0-9_]+)\s*\(", _code(f)))
    missing = [name for name in _lib._SIGNATURES if name not in defined]
    assert not missing, f"bound in ops/_lib.py but not defined under csrc/: {missing}"


def test_device_code_never_traps_or_asserts():
    for f in CUDA_FILES:
        code = _code(f)
        assert "__trap" not in code and "asm(\"trap" not in code and "asm volatile(\"trap" not in code, f.name
        assert not re.search(r"\bassert\s*\(", code), f"device assert in {f.name}"
        assert "__brkpt" not in code, f.name


def test_every_spin_loop_has_a_bound():
    """`while (true)` / `for (;;)` loops and loops on a flag must sit next to a time or iteration
    limit: the waits in common.cuh compare the global timer with a timeout and break."""
    for f in CUDA_FILES:
        code = _code(f)
        for m in re.finditer(r"while\s*\(\s*(true|1)\s*\)|for\s*\(\s*;\s*;\s*\)", code):
            body = code[m.end():m.end() + 900]
            assert re.search(r"timeout|globaltimer|max_iter|limit", body) and "break" in body or "return" in body, \
                f"unbounded loop in {f.name} near offset {m.start()}"
    common = _code(CSRC / "common.cuh")
    assert "globaltimer_ns() - t0 > timeout_ns" in common           # flag waits
    assert "globaltimer_ns() - t0 > kMbarTimeoutNs" in common        # mbarrier waits


def test_nothing_closed_is_named():
    for f in ALL_FILES:
        text = f.read_text()                                          # comments count here
        needle = "::".join(["multicast", "cluster"])               # spelled in two parts on purpose
        assert needle not in text, f"cluster-multicast qualifier in {f.name}"
        for call in ("Memcpy" + "BatchAsync", "Memcpy3D" + "BatchAsync"):
            assert call not in text, f"{call} named in {f.name}"
        assert "wgmma" not in _code(f), f"Hopper-only instruction in {f.name}"


def test_tensor_core_kernels_are_blackwell_native():
    gemm = _code(CSRC / "grouped_gemm.cu") + _code(CSRC / "common.cuh")
    for needle in ("tcgen05.mma", "tcgen05.alloc", "tcgen05.ld", "tcgen05.commit", "cp.async.bulk.tensor"):
        assert needle in gemm, f"{needle} missing from the GEMM path"
    # peer pointers in the same kernel as the tensor-core tiles (fused GEMM + M2N store)
    assert "peer_combine" in _code(CSRC / "grouped_gemm.cu") and "st_relaxed_sys" in _code(CSRC / "grouped_gemm.cu")


@pytest.mark.parametrize("name", ["grouped_gemm.cu", "moe_comm.cu", "tp_comm.cu"])
def test_flag_protocol_uses_one_system_fence_per_launch(name):
    """The release chain is data -> fence.gpu -> counter -> fence.sys -> flag, with the
    system-scope fence issued only by the CTA that arrives last."""
    code = _code(CSRC / name)
    for m in re.finditer(r"__threadfence_system\(\)", code):
        before = code[max(0, m.start() - 400):m.start()]
        if "set_flag_kernel" in before:          # the one-thread helper kernel
            continue
        assert "gridDim.x - 1" in before, f"system fence outside the last-CTA branch in {name}"


def _c_struct_fields(src: str, name: str):
    """(name, kind) of the fields of `struct name { ... };` in declaration order (a nested struct's body is
    skipped, its instance counts as one field of kind struct)."""
    import re

    start = src.index("struct " + name + " {")
    i = src.index("{", start) + 1
    depth, body, nested = 1, [], 0
    while depth:
        ch = src[i]
        if ch == "{":
            depth += 1
            nested += 1
        elif ch == "}":
            depth -= 1
            if depth == 1:
                body.append("NESTED_END ")
        if depth == 1 and ch not in "{}":
            body.append(ch)
        i += 1
    text = re.sub(r"//[^\n]*", "", "".join(body))
    fields = []          # (name, kind): kind in ptr, int, float, long, u64, struct, with "[]" appended for arrays
    for decl in text.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        if decl.startswith("struct") and "NESTED_END" in decl:        # `struct X { ... } inst`
            fields.append((decl.split("NESTED_END")[-1].strip(), "struct"))
            continue
        decl = decl.replace("NESTED_END", "").strip()
        m = re.match(r"(?:const\s+)?(unsigned long long|void|int|float|long|[A-Za-z_][A-Za-z_0-9:]*)\s*(\*?)\s*(.*)$", decl, re.S)
        base, star, rest = m.group(1), m.group(2), m.group(3)
        kind = "ptr" if star else {"int": "int", "float": "float", "long": "long", "unsigned long long": "u64"}.get(base, "struct")
        for part in rest.split(","):
            dm = re.match(r"\s*\*?\s*([A-Za-z_][A-Za-z_0-9]*)\s*(\[[^\]]*\])?\s*$", part)
            fields.append((dm.group(1), kind + ("[]" if dm.group(2) else "")))
    return fields


def _ctypes_kind(t) -> str:
    import ctypes as C

    if hasattr(t, "_length_"):
        return _ctypes_kind(t._type_) + "[]"
    if issubclass(t, C.Structure):
        return "struct"
    return {C.c_void_p: "ptr", C.c_int: "int", C.c_float: "float", C.c_long: "long", C.c_ulonglong: "u64",
            C.c_uint: "int"}[t]


@pytest.mark.parametrize("py_cls,c_file,c_name", [
    ("GroupedGemmDesc", "grouped_gemm.cu", "AfdGroupedGemmDesc"),
    ("DispatchDesc", "moe_comm.cu", "AfdDispatchDesc"),
    ("RouteDispatchDesc", "moe_comm.cu", "AfdRouteDispatchDesc"),
    ("GroupDesc", "moe_comm.cu", "AfdGroupDesc"),
    ("CombineDesc", "moe_comm.cu", "AfdCombineDesc"),
    ("DirectDesc", "moe_direct.cu", "AfdDirectDesc"),
    ("RouteDirectDesc", "moe_direct.cu", "AfdRouteDirectDesc"),
])
def test_ctypes_descriptors_list_the_fields_of_their_c_structs_in_order(py_cls, c_file, c_name):
    """A descriptor crosses the language boundary by layout: the ctypes class must name the same fields in
    the same order and with the same kind of type (pointer, int, float, long, 64-bit, struct, array) as the C
    struct it is passed as; a mismatch would only show on a GPU."""
    import os

    from fastafd_b200.ops import _lib

    src = open(os.path.join(os.path.dirname(_lib.__file__), "..", "csrc", c_file)).read()
    c_fields = _c_struct_fields(src, c_name)
    py_fields = [(f[0], _ctypes_kind(f[1])) for f in getattr(_lib, py_cls)._fields_]
    assert py_fields == c_fields, [(a, b) for a, b in zip(py_fields, c_fields) if a != b] or (py_fields, c_fields)


def _c_api_arity():
    """name -> number of parameters of every `extern "C" ... afd_name(...)` in the sources."""
    arity = {}
    for path in sorted(CSRC.rglob("*.c*")):
        code = re.sub(r"//[^\n]*", "", path.read_text())
        for m in re.finditer(r'extern\s+"C"\s+[A-Za-z_ \*]+?\b(afd_[a-z0-9_]+)\s*\(([^)]*)\)', code, re.S):
            params = m.group(2).strip()
            arity[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return arity


def test_python_call_sites_pass_as_many_arguments_as_the_c_functions_take():
    """ctypes checks nothing: a call with one argument too few reads garbage on the GPU side. Every
    direct call `lib().afd_x(a, b, ...)` (no star-arguments) must match the C parameter count."""
    import ast

    arity = _c_api_arity()
    assert len(arity) > 30
    pkg = CSRC.parent
    checked, bad = 0, []
    for path in sorted(pkg.rglob("*.py")):
        tree = ast.parse(path.read_text())
        for node in ast.walk(tree):
            if not (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute) and node.func.attr.startswith("afd_")):
                continue
            if any(isinstance(a, ast.Starred) for a in node.args) or node.keywords:
                continue
            name = node.func.attr
            if name not in arity:
                continue                     # e.g. a symbol of the NCCL wrapper declared inside extern "C" { }
            checked += 1
            if len(node.args) != arity[name]:
                bad.append((str(path.relative_to(pkg)), node.lineno, name, len(node.args), arity[name]))
    assert checked > 30, checked
    assert not bad, bad


def test_host_process_groups_are_not_bound_to_a_device():
    """A default process group bound to a device (`device_id=`) makes torch split an NCCL communicator inside
    every later `new_group` on the non-member ranks only; with a gloo sub-group the members never join the
    split and the job deadlocks during start-up. The harness and the workers therefore create a plain gloo
    default group, and the CUDA tensor-parallel set-up makes no sub-group at all."""
    import ast

    root = CSRC.parent.parent
    for rel in ("bench.py", "fastafd_b200/worker/main.py"):
        tree = ast.parse((root / rel).read_text())
        calls = [n for n in ast.walk(tree) if isinstance(n, ast.Call) and isinstance(n.func, ast.Attribute)
                 and n.func.attr == "init_process_group"]
        assert calls, rel
        for c in calls:
            assert not any(k.arg == "device_id" for k in c.keywords), f"{rel}: device-bound default group"
            args = [a.value for a in c.args if isinstance(a, ast.Constant)]
            args += [k.value.value for k in c.keywords if k.arg == "backend" and isinstance(k.value, ast.Constant)]
            assert args == ["gloo"], (rel, args)
    src = (root / "fastafd_b200" / "engine.py").read_text()
    body = src[src.index("def make_tp_comms("):src.index("class AfdEngine:")]
    cuda_part = body[body.index('if device.type == "cuda":'):body.index("mine = None")]
    assert "new_group" not in cuda_part


def test_every_registered_hot_path_knob_is_read_somewhere():
    from fastafd_b200.env import HOT_PATH_KNOBS

    pkg = CSRC.parent
    text = "".join(p.read_text() for p in list(pkg.rglob("*.py")) + list(CSRC.rglob("*.cu*")) if p.name != "env.py")
    assert [k for k in HOT_PATH_KNOBS if k not in text] == []


def test_every_region_of_every_peer_heap_layout_is_aligned_and_disjoint():
    """Peer heaps are carved by layouts that both sides compute on their own: regions must start on a 256-byte
    boundary (bulk copies and tensor maps want 16, vector stores 16, the flag words their own cache line), must
    not overlap, and the per-source / per-lane blocks inside a row region must start on 16 bytes too. Checked for
    the model shapes that are served and for odd token counts."""
    import itertools

    from fastafd_b200.cad.gpu import attention_window_layout, model_window_layout
    from fastafd_b200.config import get_model_config
    from fastafd_b200.moe.afd_moe import MoeCommConfig, ag_layout, eg_layout
    from fastafd_b200.parallel.tp_fused import tp_layout

    def check(lay, what):
        spans = sorted(lay.entries.values())
        for (off, n), nxt in zip(spans, spans[1:] + [(lay.size, 0)]):
            assert off % 256 == 0, (what, off)
            assert off + n <= nxt[0], (what, "overlap", off, n, nxt)
        assert lay.size % 256 == 0

    for name, num_ag, num_eg, lanes, tokens, fp8 in itertools.product(
            ("qwen3-30b-a3b", "qwen3-235b-a22b-fp8", "minimax-m2.5-fp8", "qwen3.5-397b-a17b-fp8", "glm-4.5-air"),
            (1, 4, 6), (1, 2, 4), (1, 2, 3), (1, 44, 129, 2048), (False, True)):
        c = get_model_config(name)
        m = MoeCommConfig(num_ag=num_ag, num_eg=num_eg, num_lanes=lanes, max_tokens=tokens, hidden=c.hidden_size,
                          topk=c.num_experts_per_tok, num_experts=c.num_experts, intermediate=c.moe_intermediate_size,
                          fp8=fp8, block_tok=32, direct_tokens=min(tokens, 64))
        check(ag_layout(m), (name, "ag"))
        check(eg_layout(m), (name, "eg"))
        assert (tokens * m.row_bytes) % 16 == 0 and (tokens * (c.hidden_size // 128) * 4) % 4 == 0      # per-source blocks
        assert (m.direct_cap * m.row_bytes) % 16 == 0                                                   # per-expert stripes
    for name, tp, lanes, tokens in itertools.product(("qwen3-30b-a3b", "qwen3-235b-a22b-fp8"), (2, 4, 8), (1, 2), (1, 11, 64)):
        c = get_model_config(name)
        check(tp_layout(tp, lanes, tokens, c.hidden_size), (name, "tp"))
        assert (tokens * c.hidden_size * 2) % 16 == 0
    for name, attn, lanes, tokens in itertools.product(("minimax-m2.5-fp8", "qwen3-30b-a3b"), (1, 2, 7), (1, 2), (1, 77, 256)):
        c = get_model_config(name)
        check(attention_window_layout(c, lanes, tokens), (name, "cad-attn"))
        check(model_window_layout(c, attn, lanes, tokens), (name, "cad-model"))
