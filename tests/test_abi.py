"""The C-ABI library loads and exports every symbol the public header declares
(no GPU needed: argument validation runs before any CUDA call)."""

import os
import re

import pytest

from sparsepr_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "sparsepr_b200.h")


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spr_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.PROTOTYPES)


def test_version_and_error_message(lib):
    assert lib.spr_version() >= 100
    with pytest.raises(RuntimeError, match="SPR_ERR_SHAPE.*ck <= 2048"):
        _lib.call("spr_select_budget", None, None, None, 1, 1, 4096, None, None, None, None)
    with pytest.raises(RuntimeError, match="SPR_ERR_SHAPE.*d=128"):
        _lib.call("spr_block_sparse_attn", None, None, None, None, None, None, None, 1, 8, 8, 64, 1, 1, None, None,
                  None, None, 0, None)
    with pytest.raises(RuntimeError, match="SPR_ERR_SHAPE.*m=0"):
        _lib.call("spr_probe_rows_attn", None, None, None, None, None, None, None, 1, 8, 8, 128, 1, 1, 0, None, None,
                  None, 0, None)
    with pytest.raises(RuntimeError, match="SPR_ERR_WORKSPACE"):
        _lib.call("spr_label_sort", None, 1, 100, 4, None, None, None, None, 0, None)
    with pytest.raises(RuntimeError, match="SPR_ERR_SHAPE.*d=42"):
        _lib.call("spr_kmeans_assign", None, 0, 1, 10, 42, 4, None, 0, None, None, 0, None)


def test_workspace_queries(lib):
    small = _lib.query("spr_kmeans_workspace_bytes", 1, 1000, 48, 64)
    big = _lib.query("spr_kmeans_workspace_bytes", 40, 75600, 48, 1000)
    assert 0 < small < big
    assert _lib.query("spr_block_sparse_attn_workspace_bytes", 40, 75600, 200) >= 40 * 201 * 4
