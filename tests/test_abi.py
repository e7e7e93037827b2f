"""C-ABI library: loads without a GPU, exports every declared symbol, validates input."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(kvq_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from kvquant.kernels.cuda_ops import load_library
    return load_library()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 20
    for required in ("kvq_rope_apply", "kvq_lut_matvec", "kvq_sparse_matvec_csr",
                     "kvq_lut_lookup", "kvq_key_scores", "kvq_value_output",
                     "kvq_decode_attention", "kvq_quantize_keys_plan", "kvq_quantize_values_emit"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(Path(lib._name)))
    missing = [n for n in declared_symbols() if not hasattr(raw, n)]
    assert not missing, missing


def test_python_binding_covers_header(lib):
    from kvquant.kernels.cuda_ops import _SIGNATURES
    assert set(declared_symbols()) == set(_SIGNATURES)


def test_version(lib):
    assert lib.kvq_version() >= 100


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    # odd head_dim
    rc = lib.kvq_rope_apply(None, None, None, None, 1, 1, 1, 3, 0, 1, None)
    assert rc == 1 and b"even D" in lib.kvq_last_error()
    # positions beyond the table
    rc = lib.kvq_rope_apply(None, None, None, None, 1, 1, 8, 128, 4, 10, None)
    assert rc == 1
    rc = lib.kvq_lut_matvec(None, None, 300, None, None, None, None, 4, 4, 1, None)
    assert rc == 1 and b"lut_size too large" in lib.kvq_last_error()
    # unsupported bit width / group size
    rc = lib.kvq_key_scores(None, None, None, None, None, None, None, 5, None, None,
                            1, 1, 1, 64, 2, None, None)
    assert rc == 3
    rc = lib.kvq_key_scores(None, None, None, None, None, None, None, 4, None, None,
                            1, 1, 3, 64, 2, None, None)
    assert rc == 3
    # capacity too small for T
    rc = lib.kvq_key_scores(None, None, None, None, None, None, None, 4, None, None,
                            1, 1, 1, 65, 2, None, None)
    assert rc == 1
    # code tiles are staged with 16-byte copies: a null or unaligned codes pointer
    # is refused (the pointer is never dereferenced on this path)
    for codes in (None, ctypes.c_void_p(8)):
        rc = lib.kvq_key_scores(codes, None, None, None, None, None, None, 4, None, None,
                                1, 1, 1, 64, 2, None, None)
        assert rc == 1 and b"16-byte aligned" in lib.kvq_last_error()
    # workspace too small
    rc = lib.kvq_quantize_keys_plan(None, 1, 64, 128, 0, 1, None, None, 0.01, 1, None, 2, None,
                                    None, 0, None)
    assert rc == 1 and b"workspace" in lib.kvq_last_error()
    # error message is per call: a later valid query clears nothing but a new error replaces it
    rc = lib.kvq_softmax(None, 1, 0, 1.0, None, None, 0, None)
    assert rc == 1 and b"softmax" in lib.kvq_last_error()


def test_workspace_queries(lib):
    assert lib.kvq_quantize_keys_workspace(1, 4096, 32) >= 32 * 128 * 256 * 4
    assert lib.kvq_decode_attention_workspace(1, 32, 1, 4096) >= 2 * 32 * 4096 * 4
    assert lib.kvq_softmax_workspace(32, 4096) >= 32 * 8


def test_shard_entry_points_reject_bad_arguments(lib):
    import ctypes as ct
    # a sink belongs to position 0 only
    rc = lib.kvq_key_scores_stats_at(None, None, None, None, None, ct.c_void_p(16), None, 4, None,
                                     None, 1, 1, 1, 64, 2, 32, None, 0.1, ct.c_void_p(16), None)
    assert rc == 1 and b"pos0" in lib.kvq_last_error()
    rc = lib.kvq_merge_shards(None, None, 0, 4, None, None)
    assert rc == 1
    rc = lib.kvq_value_output_scores_ml(None, None, None, None, None, 64, None, None, 4, None,
                                        None, 0.1, 1, 1, 1, 64, 2, None, None, None, 0, None)
    assert rc == 1 and b"ml_out" in lib.kvq_last_error()

