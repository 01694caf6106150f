"""The C-ABI library builds, loads without a GPU and exports every declared symbol."""
import ctypes
import re
from pathlib import Path

import pytest

from gsa_gdn_benchmarkstudy_b200 import _lib
from gsa_gdn_benchmarkstudy_b200.build import build

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"GSA_API\s+[\w\s\*]+?\b(gsa_\w+)\s*\(", h.read_text())
    return names


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    # and the ctypes signature table covers exactly the declared set
    assert set(names) == set(_lib.SIGNATURES)


def test_host_only_entry_points(lib):
    assert lib.gsa_version() >= 10000
    assert lib.gsa_status_string(0) == b"ok"
    assert lib.gsa_status_string(3) == b"unsupported shape or dtype"
    assert lib.gsa_bitmask_words(1) == 4
    assert lib.gsa_bitmask_words(128) == 4
    assert lib.gsa_bitmask_words(129) == 8
    assert lib.gsa_bitmask_words(16384) == 512


def test_argument_checks_run_before_any_device_work(lib):
    # Invalid sizes are rejected on the host with GSA_ERR_INVALID_ARG (1) /
    # GSA_ERR_UNSUPPORTED (3) before the library touches CUDA.
    rc = lib.gsa_topk_select(None, 0, 1, 1, 8, 0, 0, None, None, None, 0, None)
    assert rc == 1
    rc = lib.gsa_masked_attention(None, 0, None, 0, None, 0, None, 0, None, 0, None, 0,
                                  1.0, 1, 1, 1, 0, 1, 64, None)
    assert rc == 3
    assert b"d == 128" in lib.gsa_last_error_string()
    rc = lib.gsa_rope_gates(None, None, None, None, 0, 7, 1, 1, 1, 16, None, None, None, None,
                            None, None)
    assert rc == 3
    # empty work is a no-op success
    assert lib.gsa_indexer_scores(None, 0, None, 0, None, 0, None, 1.0, 0, 0, 4, 4, 0, 4, 64,
                                  None, 4, 0, None) == 0


def test_adaptive_k_entry_points_on_the_host(lib):
    assert lib.gsa_adaptive_k_width(4096, 160) == 160
    assert lib.gsa_adaptive_k_width(64, 160) == 64
    # scores 1*4 rows * 8 floats = 128 B, row_var 16 B, var_sum on a 16 B boundary
    assert lib.gsa_indexer_topk_adaptive_workspace_size(1, 4, 5) == 160
    assert lib.gsa_indexer_topk_adaptive_workspace_size(0, 4, 5) == 0
    # k_min > k_max and k_max < 1 are rejected before any device work
    rc = lib.gsa_topk_select_adaptive(None, 8, 1, 1, 8, 0, 4, 9, 8, None, None, 1, None, None,
                                      None, None, 0, None)
    assert rc == 1 and b"k_min <= k_max" in lib.gsa_last_error_string()
    rc = lib.gsa_indexer_topk_adaptive(None, 0, None, 0, None, 0, None, 1.0, 0, 1, 1, 8, 0, 4,
                                       64, 4, 0, 0, None, 0, None, None, None, None, 0, None)
    assert rc == 1
    rc = lib.gsa_row_variance(None, 8, 1, 1, 8, 0, None, None, None)
    assert rc == 1



def test_fused_projection_layout_queries(lib):
    # hidden 2048, 4 indexer heads of 64: q 8 + k 8 + v/vg 16 + rest 10 column tiles
    # of 256 rows; rest columns og 2048 | iq 256 | ik 64 | iw 4 = 2372 -> 2432
    assert lib.gsa_fused_projection_rows(2048, 4, 64) == 42 * 256
    assert lib.gsa_fused_projection_rest_width(2048, 4, 64) == 2432
    assert lib.gsa_fused_projection_rows(512, 4, 64) == (2 + 2 + 4 + 4) * 256
    # hidden sizes that are not a multiple of 256 are not served
    assert lib.gsa_fused_projection_rows(640, 4, 64) == 0
    assert lib.gsa_fused_projection_rest_width(640, 4, 64) == 0
    # host-side checks before any device work: d != 128 is unsupported (3),
    # negative sizes are invalid (1), no rows is a no-op
    rc = lib.gsa_fused_projection(None, 0, None, None, 4, 512, 8, 64, 4, 64, 4, 0, None, None,
                                  0, None, None, None, None, 0, None)
    assert rc == 3 and b"d == 128" in lib.gsa_last_error_string()
    rc = lib.gsa_fused_projection(None, 0, None, None, -1, 512, 4, 128, 4, 64, 4, 0, None, None,
                                  0, None, None, None, None, 0, None)
    assert rc == 1
    assert lib.gsa_fused_projection(None, 0, None, None, 0, 512, 4, 128, 4, 64, 4, 0, None, None,
                                    0, None, None, None, None, 0, None) == 0
