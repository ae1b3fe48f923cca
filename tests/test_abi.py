"""The C-ABI library loads on a machine without a GPU and exports every entry
point declared in include/orthocache_b200.h; the ctypes table covers them all.
No compute calls (those need a GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "orthocache_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(oc_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    for n in ("oc_fwht512", "oc_score_blocks", "oc_stream_compact", "oc_indirect_attention", "oc_decode_step"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from orthocache_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from orthocache_b200 import build
        build.build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from orthocache_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()
    lib = _lib.load()
    assert lib.oc_version() >= 100
    assert lib.oc_status_string(-2) == b"bad shape"


def test_host_side_validation_without_gpu():
    """Argument checks run on the host before any launch: bad shapes fail with
    a status code and a message, without touching the device."""
    from orthocache_b200 import _lib
    lib = _lib.load()
    rc = lib.oc_score_blocks(ctypes.c_void_p(16), None, 1, 1, 1000, 8, 128, 0, 0, 1, 64, 64, 256, 256, 512,
                             0.0, 5.0, None, None, None, None, None, None, None, None, 0, None)
    assert rc == -2 and b"multiple of 512" in lib.oc_last_error()
    rc = lib.oc_stream_compact(None, 1, 4, 1, None, None, None)
    assert rc == -1
    assert lib.oc_stratified_bucket(16, 5) == 8
    assert lib.oc_stratified_bucket(16, 0) == 4
    assert lib.oc_stratified_bucket(1, 1) == 1
    assert lib.oc_indirect_attention_workspace_bytes(1, 1, 32, 8, 128, 512, 128) > 0
    # an unsupported head_dim is an error code, never a host-side crash
    assert lib.oc_indirect_attention_workspace_bytes(1, 1, 32, 8, 0, 512, 4) == 0
    assert lib.oc_indirect_attention_workspace_bytes(1, 1, 32, 8, 16384, 512, 4) == 0
    assert lib.oc_decode_step_workspace_bytes(1, 1, 32, 8, 0, 65536) == 0
    rc = lib.oc_indirect_attention_noalloc(None, None, None, 1, None, 4, 0, None, 1, 0, 1, 1, 32, 8, 0,
                                           2048, 512, 4, ctypes.c_void_p(16), 1, None)
    assert rc == -2 and b"head_dim" in lib.oc_last_error()


@pytest.mark.parametrize("seq_len,head_dim,q_heads,kv_heads,needle", [
    (-512, 128, 32, 8, b"seq_len"),
    (512, 0, 32, 8, b"head_dim"),
    (512, 7, 32, 8, b"head_dim"),
    (512, 128, 30, 8, b"q_heads"),
    (512, 128, 32, 0, b"kv_heads"),
])
def test_decode_step_shape_errors_without_gpu(seq_len, head_dim, q_heads, kv_heads, needle):
    """Both one-launch decode entry points reject a bad shape on the host with
    OC_ERR_SHAPE before any launch (the pointers are never dereferenced)."""
    from orthocache_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    rc = lib.oc_decode_step_from_metadata(p, p, p, 1, p, p, p, 1, 1, q_heads, kv_heads, head_dim, seq_len, 0.0, 5.0,
                                          p, p, p, p, 1, p, 1 << 30, None)
    assert rc == -2 and needle in lib.oc_last_error()
    rc = lib.oc_decode_step(p, p, p, 1, 1, 1, q_heads, kv_heads, head_dim, seq_len, 0.0, 5.0, p, p, p, p, 1,
                            p, 1 << 30, None)
    assert rc == -2 and needle in lib.oc_last_error()
