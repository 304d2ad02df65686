"""The C-ABI library: it builds for sm_100a, loads without a GPU, and exports every symbol the header declares."""
import ctypes
import os
import re

import pytest

from gravityocr_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gravity_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gr_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert _declared() == sorted(L.EXPORTS)


def test_library_loads_and_exports_every_symbol():
    if not os.path.exists(L.LIB_PATH):
        from gravityocr_b200.build import build
        build()
    lib = ctypes.CDLL(L.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name
    lib = L.load()
    assert lib.gr_version() >= 100
    assert lib.gr_status_string(4).decode() == "device wait timed out"


def test_product_library_is_not_the_timeline_build():
    """The per-CTA timeline stamps exist only in the separately built libgravity_b200_timeline.so (-DGR_TIMELINE);
    the library the product loads has none of their code or symbols."""
    if not os.path.exists(L.LIB_PATH):
        from gravityocr_b200.build import build
        build()
    lib = ctypes.CDLL(L.LIB_PATH)
    for unit in ("linear", "attention", "attention_tc", "rowwise", "sampling"):
        assert not hasattr(lib, "gr_timeline_read_" + unit)


def test_workspace_queries_without_gpu():
    lib = L.load()
    # fixed ticket region + partials; argmax scratch grows with rows
    a = L.linear_workspace_bytes(59392, 17, 1)
    b = L.linear_workspace_bytes(59392, 64, 1)
    assert 0 < a < b
    assert L.attention_workspace_bytes(1, 17, 16, 8, 4) >= 65536


def test_argument_errors_are_returned_not_raised():
    lib = L.load()
    e = L.Epilogue()
    e.mode = 99
    rc = lib.gr_linear(None, 128, 64, None, 1, ctypes.byref(e), 0, None, 0, None, 0, None, None)
    assert rc == 1  # GR_ERR_ARG, no CUDA call made
    rc = lib.gr_bd_attention(None, None, None, 0, None, 0, None, 1, 17, 1, 0, 16, 8, 16, 64, 1, None, None, 0, None,
                             None)
    assert rc == 1


def test_sampling_rejects_a_vocabulary_above_its_bound():
    """sample_rows' per-warp 32-bit bucket words hold at most 4,095 entries a warp: a larger vocabulary is refused
    before any CUDA call (the pointers below are never dereferenced)."""
    lib = L.load()
    s = L.Sampling()
    s.vocab, s.filter = 65025, L.FILTER_JOINT
    s.temperature = s.top_k = s.top_p = s.min_p = s.req_pool_idx = s.rng = 16
    assert lib.gr_sample_rows(16, 1, 1, None, ctypes.byref(s), L.COIN_FIRST, None, 16, None, None, 0, None,
                              None) == 1
    assert lib.gr_logits_process(16, 1, 1, None, ctypes.byref(s), None) == 1


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(L, "_lib", None)
    with pytest.raises(RuntimeError, match="not found"):
        L.load(str(tmp_path / "nope.so"))


def test_product_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "gravityocr_b200")
    for dp, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                src = open(os.path.join(dp, f)).read()
                assert not re.search(r"^\s*(from|import)\s+oracle", src, flags=re.M), f
