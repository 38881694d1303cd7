"""CPU checks of the C ABI: libfrag.so loads without a GPU, exports every
entry point include/frag.h declares, and rejects bad arguments on the host
(these calls return before touching CUDA)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from kernelproblems_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "frag.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FRAG_API\s+[\w\s\*]+?\b(frag_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "frag_rmsnorm_fwd" in names and "frag_embedding_bwd" in names and "frag_rope" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"libfrag.so does not export {name}"


def test_bindings_cover_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES), \
        "ctypes signatures and include/frag.h disagree"


def test_version_and_status_strings():
    assert "sm_100a" in _lib.version()
    lib = _lib.load()
    for code in range(7):
        assert lib.frag_status_string(code)
    assert b"unknown" in lib.frag_status_string(99)


def test_invalid_arguments_rejected_on_host():
    lib = _lib.load()
    null = None
    assert lib.frag_rmsnorm_fwd(null, null, null, null, 4, 8, 1e-5, null) == 1
    assert lib.frag_rmsnorm_fwd(null, null, null, null, -1, 8, 1e-5, null) == 1
    assert lib.frag_rmsnorm_fwd(null, null, null, null, 0, 8, 1e-5, null) == 0  # empty: no work
    assert lib.frag_add_rmsnorm_fwd(null, null, null, null, null, null, 4, 8, 1e-5, null) == 1
    assert lib.frag_rmsnorm_bwd(null, null, null, null, null, null, null, null, null, 4, 8, 1e-5,
                                null, 0, null) == 1
    assert lib.frag_rmsnorm_bwd(null, null, null, null, null, null, null, null, null, 0, 0, 1e-5,
                                null, 0, null) == 0
    assert lib.frag_embedding_fwd(null, null, null, -1, 4, 4, 0, 4, null, null) == 1
    assert lib.frag_embedding_fwd(null, null, null, 0, 4, 4, 0, 4, null, null) == 0
    assert lib.frag_embedding_bwd(null, null, null, -1, 4, 4, 0, 4, -1, null, 0, null, null) == 1
    assert lib.frag_dw_reduce(null, 1, 4, null, null, null) == 1
    assert lib.frag_rope(None, 1, 1, 1, 128, null, 0, 0, 0, null, 0, 0, 1e4, 0, 0, null) == 1
    t = (_lib.RopeTensor * 1)(_lib.RopeTensor(0, 0, 1, 0, 0, 0, 0, 0, 0))
    assert lib.frag_rope(t, 1, 1, 1, 128, null, 0, 0, 0, null, 0, 0, 1e4, 7, 0, null) == 1  # bad layout
    assert lib.frag_rope(t, 3, 1, 1, 128, null, 0, 0, 0, null, 0, 0, 1e4, 0, 0, null) == 1  # > 2 tensors
    assert lib.frag_rope(t, 1, 1, 1, 127, null, 0, 0, 0, null, 0, 0, 1e4, 0, 0, null) == 2  # odd D
    T = _lib.RopeTensor
    for descs, layout in (([T(16, 32, 1, 0, 0, 0, 0, 0, 0, 0, 1)], 1),    # fp32 in, bf16 out
                          ([T(16, 32, 1, 0, 0, 0, 0, 0, 0, 1, 1)], 0),    # fp32 in, neox
                          ([T(16, 32, 1, 0, 0, 0, 0, 0, 0, 1, 1),
                            T(16, 32, 1, 0, 0, 0, 0, 0, 0, 0, 0)], 1),    # mixed input types
                          ([T(16, 32, 1, 0, 0, 0, 0, 0, 0, 0, 5)], 1)):   # unknown in_dtype
        arr = (T * len(descs))(*descs)
        assert lib.frag_rope(arr, len(descs), 1, 1, 128, null, 0, 0, 0, null, 0, 0, 1e4, layout, 0,
                             null) == 1
    fb = lib.frag_rmsnorm_fwd_bwd
    assert fb(null, null, 8, null, null, null, null, null, null, null, null, null, null, 4, 8, 1e-5,
              null, 0, null) == 1                                                  # x3 without x2
    assert fb(null, null, null, null, null, null, null, null, null, null, null, null, null, -1, 8,
              1e-5, null, 0, null) == 1
    assert fb(null, null, null, null, null, null, null, null, null, null, null, null, null, 4, 8,
              1e-5, null, 0, null) == 1                                            # null x, dy
    assert fb(null, null, null, null, null, null, null, null, null, null, null, null, null, 0, 8,
              1e-5, null, 0, null) == 0                                            # empty, no dw
    cv = lib.frag_convert_rows
    assert cv(null, 0, 8, null, null, 1, 8, 4, 8, null) == 1     # null src / dst
    assert cv(16, 2, 8, 32, null, 1, 8, 4, 8, null) == 1         # unknown dtype
    assert cv(16, 0, 4, 32, null, 1, 8, 4, 8, null) == 2         # source rows overlap
    assert cv(null, 0, 8, null, null, 1, 8, 0, 8, null) == 0     # empty
    assert cv(16, 0, 8, 32, null, 1, 8, -1, 8, null) == 1
    seg = _lib.CopySegment
    segs = (seg * 17)()
    assert lib.frag_copy_rows_grouped(segs, 0, null) == 0                       # nothing to copy
    assert lib.frag_copy_rows_grouped(segs, 17, null) == 1                      # > 16 segments
    assert lib.frag_copy_rows_grouped(segs, -1, null) == 1
    assert lib.frag_copy_rows_grouped(None, 1, null) == 1
    assert lib.frag_copy_rows_grouped(segs, 16, null) == 0                      # all empty
    bad = (seg * 2)(seg(None, None, 0, 0, 0, 64), seg(None, None, 64, 64, -1, 64))
    assert lib.frag_copy_rows_grouped(bad, 2, null) == 1                        # negative rows
    bad = (seg * 1)(seg(None, None, 64, 64, 2, 64))
    assert lib.frag_copy_rows_grouped(bad, 1, null) == 1                        # null pointers
    bad = (seg * 1)(seg(4096, 8192, 16, 64, 2, 64))
    assert lib.frag_copy_rows_grouped(bad, 1, null) == 2                        # rows overlap
    vp = lib.frag_embedding_fwd_vp_peer
    arr = (C.c_void_p * 8)(*([16] * 8))
    st = C.c_void_p(16)
    assert vp(null, null, 0, 0, 64, 0, 0, arr, arr, st, 0, 0, null, null) == 1      # world 0
    assert vp(null, null, 0, 0, 64, 0, 0, arr, arr, st, 0, 9, null, null) == 1      # > 8 ranks
    assert vp(null, null, 0, 0, 64, 0, 0, arr, arr, st, 2, 2, null, null) == 1      # rank >= world
    assert vp(null, null, 0, 0, 64, 0, 0, arr, arr, None, 0, 2, null, null) == 1    # no state
    assert vp(null, null, 4, 0, 64, 0, 0, arr, arr, st, 0, 2, null, null) == 1      # ids missing
    assert vp(null, null, 0, 0, 60, 0, 0, arr, arr, st, 0, 2, null, null) == 2      # D % 8
    dx = lib.frag_dw_exchange_peer
    assert dx(null, 64, arr, arr, st, 0, 0, null, null) == 1      # world 0
    assert dx(null, 64, arr, arr, None, 0, 2, null, null) == 1    # no state
    assert dx(null, 64, arr, arr, st, 0, 2, null, null) == 1      # no vectors
    assert dx(16, 62, arr, arr, st, 0, 2, 16, null) == 2          # N % 4
    assert lib.frag_peer_alloc(0, None, None) == 1
    assert lib.frag_peer_open(None, None) == 1
    assert lib.frag_peer_close(None) == 1 and lib.frag_peer_free(None) == 1


def test_fraggerror_message():
    e = _lib.FragError("frag_x", 4)
    assert "FRAG_ERR_WORKSPACE" in str(e) and e.status == 4


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setenv("FRAG_LIBRARY", str(tmp_path / "nope.so"))
    with pytest.raises(FileNotFoundError):
        _lib.load()
    monkeypatch.undo()
    _lib._lib = None
    _lib.load()


@pytest.mark.parametrize("key,n_inputs", [("v8/f6251e84e3fa", 8), ("v8/43f0c930291e", 7),
                                          ("v8/7e38211c7f1c", 2)])
def test_broken_reference_input_fails_like_the_reference(key, n_inputs):
    """These problems' own get_inputs pass a 0-d tensor where the graph
    indexes [1] of a tuple; the reference Model raises IndexError there, and
    so does the drop-in (before touching the GPU)."""
    import torch
    from kernelproblems_b200.problems import PROBLEMS
    with pytest.raises(IndexError):
        PROBLEMS[key](torch.randn([]), *[None] * (n_inputs - 1))
