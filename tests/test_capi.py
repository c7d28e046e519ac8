"""The C-ABI library loads and exports every entry point include/*.h declares (CPU only).

No test here launches a kernel: argument validation runs before any CUDA call, so the
error paths can be exercised without a GPU.
"""
import ctypes
import glob
import os
import re

import pytest

from tritonllmcompiler_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names += re.findall(r"TLLM_API\s+[\w\s\*]+?\b(tllm_\w+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_the_four_ops():
    names = _declared_functions()
    for n in ["tllm_flash_attn_fwd", "tllm_paged_attn_decode", "tllm_paged_attn_workspace_size",
              "tllm_rmsnorm_rope", "tllm_swiglu", "tllm_last_error", "tllm_debug_status"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert set(_declared_functions()) <= set(_lib.SIGNATURES), "ctypes signatures incomplete"


def test_library_is_built_for_sm100a_only():
    # The build passes exactly one -gencode (compute_100a -> sm_100a).
    from tritonllmcompiler_b200 import build

    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version_matches_reference_package():
    import tritonllmcompiler_b200 as pkg

    assert _lib.load().tllm_version() == b"0.2.0" == pkg.__version__.encode()


def _arr(*v):
    return (ctypes.c_int64 * len(v))(*v)


def test_invalid_arguments_return_status_and_message():
    lib = _lib.load()
    rc = lib.tllm_swiglu(1, 1, 1, 1, -1, 4, 4, 4, 4, 4, 4, 0, None)
    assert rc == 1 and b"negative" in lib.tllm_last_error()
    rc = lib.tllm_rmsnorm_rope(1, 1, 1, 1, 1, 1, 1, 1, 48, _arr(1, 1, 1, 1), 1, _arr(1, 1),
                               _arr(1, 1), _arr(1, 1, 1, 1), 1e-6, 0, None)
    assert rc == 1 and b"head dim 48" in lib.tllm_last_error()
    rc = lib.tllm_flash_attn_fwd(1, 1, 1, 1, 1, 1, 8, 8, 64, _arr(512, 512, 64, 2), _arr(512, 512, 64, 1),
                                 _arr(512, 512, 64, 1), _arr(512, 512, 64, 1), 0.1, 0, 0, None)
    assert rc == 1 and b"unit innermost stride" in lib.tllm_last_error()
    rc = lib.tllm_paged_attn_decode(16, 16, 16, 16, 16, 16, None, 0, 1, 1, 64, 24, 4, 4,
                                    _arr(64, 64, 64, 1), _arr(4096, 256, 64, 1),
                                    _arr(4096, 256, 64, 1), _arr(4, 1), _arr(64, 64, 64, 1),
                                    0.1, 0, 0, None)
    assert rc == 1 and b"block_size 24" in lib.tllm_last_error()
    with pytest.raises(RuntimeError, match="block_size 24"):
        _lib.check(rc)


def test_extension_entries_validate_arguments():
    lib = _lib.load()
    rc = lib.tllm_swiglu_variant(16, 16, 16, 16, 256, 128, 64, 64, 128, 128, 128, 0, 7, None)
    assert rc == 1 and b"unknown kernel variant 7" in lib.tllm_last_error()
    rc = lib.tllm_swiglu_fp8_variant(16, 16, 16, 16, 256, 128, 64, 64, 64, 64, 128, 1.0, 1.0, 1.0,
                                     0, 3, None)
    assert rc == 1 and b"unknown kernel variant 3" in lib.tllm_last_error()
    rc = lib.tllm_flash_attn_fp8_fwd(16, 16, 16, 16, 1, 1, 64, 64, 96, _arr(96, 96, 96, 1),
                                     _arr(96, 96, 96, 1), _arr(96, 96, 96, 1), _arr(96, 96, 96, 1),
                                     0.1, 1.0, 1.0, 1.0, 0, 0, None)
    assert rc == 1 and b"head dim 96" in lib.tllm_last_error()
    rc = lib.tllm_flash_attn_fp8_fwd(16, 16, 16, 16, 1, 1, 64, 64, 128, _arr(8192, 8192, 128, 1),
                                     _arr(8192, 8192, 128, 1), _arr(8192, 8192, 64, 1),
                                     _arr(8192, 8192, 128, 1), 0.1, 1.0, -1.0, 1.0, 0, 0, None)
    assert rc == 1 and b"scales" in lib.tllm_last_error()
    rc = lib.tllm_copy2d_async(16, 64, 16, 32, 64, 4, None)
    assert rc == 1 and b"pitch" in lib.tllm_last_error()
    assert lib.tllm_copy2d_async(None, 0, None, 0, 0, 0, None) == 0  # nothing to copy


def test_column_sharded_entry_validates_before_any_launch():
    """Argument errors of the in-kernel-handshake entry are reported without touching a GPU:
    a rank outside the group, epoch 0 (the flags' initial value), more than 8 destinations,
    a row stride that cannot hold every rank's slice, a variant that does not exist."""
    import ctypes

    lib = _lib.load()
    vp = ctypes.c_void_p
    d2 = (vp * 2)(16, 32)
    done = vp(48)

    def call(dsts, flags, ndst, rank, epoch, ldo, variant=0, m=256, n=128, k=64):
        return lib.tllm_swiglu_colshard_peers(16, 16, 16, dsts, flags, ndst, rank, done, epoch, m,
                                              n, k, k, n, n, ldo, 0, variant, None)

    assert call(d2, d2, 2, 2, 1, 256) == 1 and b"rank 2" in lib.tllm_last_error()
    assert call(d2, d2, 2, 0, 0, 256) == 1 and b"epoch 0" in lib.tllm_last_error()
    d9 = (vp * 9)(*([16] * 9))
    assert call(d9, d9, 9, 0, 1, 2048) == 1 and b"destinations" in lib.tllm_last_error()
    assert call(d2, d2, 2, 1, 1, 200) == 1 and b"row stride" in lib.tllm_last_error()
    assert call(d2, d2, 2, 0, 1, 256, variant=4) == 1 and b"variant 4" in lib.tllm_last_error()
    assert call(d2, d2, 2, 0, 1, 256, m=0) == 1 and b"positive" in lib.tllm_last_error()


def test_errors_are_thread_local():
    import threading

    lib = _lib.load()
    lib.tllm_swiglu(1, 1, 1, 1, -1, 4, 4, 4, 4, 4, 4, 0, None)
    seen = {}

    def other():
        seen["msg"] = lib.tllm_last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == b""
    assert b"negative" in lib.tllm_last_error()


def test_workspace_size_is_zero_for_a_single_split():
    lib = _lib.load()
    # 2 blocks of 16 tokens: one split, no partials to merge.
    assert lib.tllm_paged_attn_workspace_size(2, 2, 64, 16, 2) == 0
    big = lib.tllm_paged_attn_workspace_size(64, 32, 128, 16, 512)
    assert big > 0 and big % 4 == 0
