"""CPU checks of the C ABI: the library loads and exports every symbol include/*.h declares
(sdb.h, the op-level entry points; sdasm.h, the reference's hook surface).

No compute call is made here (there is no GPU on the CPU runner).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "stable-diffusion.assembly_b200" / "libsdb.so"


def declared_functions(header: Path, prefix: str = "sdb_") -> list[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(" + prefix + r"[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        pytest.skip("libsdb.so not built")
    return ctypes.CDLL(str(LIB))


def test_header_declarations_are_exported(lib):
    names = declared_functions(ROOT / "include" / "sdb.h")
    assert names, "no declarations found"
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_hook_surface_is_exported(lib):
    """The reference's sdasm.h functions (sources/sdasm.h:38-78), all nine."""
    names = declared_functions(ROOT / "include" / "sdasm.h", "sdasm_")
    assert len(names) == 9, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_hook_surface_answers_without_a_device(lib):
    """Calls that need no GPU: a node of an operation not taken, the work size, ToDo's factor."""
    import ggml_graph as gg

    g = gg.Graph("host")
    a = g.new_f32((8, 4), fill=1.0)
    node = g.scale(a, 2.0)
    size = ctypes.c_size_t(7)
    assert not lib.sdasm_work_size(ctypes.byref(node.s), 1, ctypes.byref(size))
    assert size.value == 7
    assert gg.compute_nodes(lib, [node], 0) == 0
    assert lib.sdasm_token_downsampling(ctypes.c_int64(64), ctypes.c_int64(64)) == 1


def test_binding_lists_every_export():
    import sdb

    names = declared_functions(ROOT / "include" / "sdb.h")
    assert sorted(sdb.EXPORTS) == names


def test_tuning_parser(lib):
    import sdb

    sdb._lib = None
    sdb.load()
    assert sdb.get_tuning("winograd") in (0, 1, 2)
    sdb.set_tuning("winograd=1,block_n=256")
    assert sdb.get_tuning("winograd") == 1 and sdb.get_tuning("block_n") == 256
    sdb.set_tuning("winograd=2,block_n=0")
    with pytest.raises(sdb.SdbError):
        sdb.set_tuning("nonsense=1")
    with pytest.raises(sdb.SdbError):
        sdb.set_tuning("winograd=7")
    assert "unknown" in sdb.load().sdb_last_error().decode() or "bad value" in sdb.load().sdb_last_error().decode()


def test_tuning_gemm_knobs(lib):
    """The linear layers' GEMM knobs: gemm_fused 0..2 and the fused kernel's tile widths 160 and 192."""
    import sdb

    sdb.load()
    assert sdb.get_tuning("gemm_fused") == 1
    try:
        for v in (0, 2, 1):
            sdb.set_tuning(f"gemm_fused={v}")
            assert sdb.get_tuning("gemm_fused") == v
        for v in (128, 160, 192, 256, 0):
            sdb.set_tuning(f"block_n={v}")
            assert sdb.get_tuning("block_n") == v
        for bad in ("gemm_fused=3", "block_n=144"):
            with pytest.raises(sdb.SdbError):
                sdb.set_tuning(bad)
    finally:
        sdb.set_tuning("gemm_fused=1,block_n=0")


def test_token_downsampling(lib):
    """hooks.cc:166-172: 1 unless todo >= 2 and the grid has todo_tokens tokens."""
    import sdb

    sdb.load()
    assert sdb.token_downsampling(64, 64) == 1
    sdb.set_tuning("todo=2,todo_tokens=4096")
    try:
        assert sdb.token_downsampling(64, 64) == 2
        assert sdb.token_downsampling(32, 32) == 1
        assert sdb.token_downsampling(0, 64) == 1
    finally:
        sdb.set_tuning("todo=1")


def test_unsupported_shapes_are_not_taken(lib):
    """A mul_mat whose inner dimensions disagree is 'not taken' (0), without touching memory."""
    import sdb

    sdb.load()
    w, x, y = sdb.Tensor(), sdb.Tensor(), sdb.Tensor()
    for t, ne in ((w, [64, 32, 1, 1]), (x, [48, 10, 1, 1]), (y, [32, 10, 1, 1])):
        t.type = sdb.TYPE_F32
        for k in range(4):
            t.ne[k] = ne[k]
        t.nb[0] = 4
        t.nb[1] = 4 * ne[0]
        t.nb[2] = t.nb[1] * ne[1]
        t.nb[3] = t.nb[2]
        t.data = 16  # never dereferenced
    assert sdb.load().sdb_mul_mat_supported(w, x, y) == 0
