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
