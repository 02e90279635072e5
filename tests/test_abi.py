"""The C ABI library loads and exports every symbol include/*.h declares (CPU only)."""
import ctypes
import glob
import os
import re

import pytest

from santapp_b200 import _build, _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(santa_[a-z0-9_]+)\s*\(",
                             src, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for want in ("santa_build_summary", "santa_decode", "santa_decode_select",
                 "santa_decode_workspace_bytes", "santa_status_string"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.santa_status_string(0) == b"ok"
    assert b"workspace" in lib.santa_status_string(-4)
    assert b"sm_100a" in lib.santa_version()


def test_struct_layout_matches_c():
    # SantaDecodeParams: 4 x int32, float, int32, 2 x uint64, int32 (+pad), pointer
    assert ctypes.sizeof(_lib.SantaDecodeParams) == 56
    assert _lib.SantaDecodeParams.seed.offset == 24
    assert _lib.SantaDecodeParams.step_dev.offset == 48
    # SantaGeometry: 8 x int32, pointer, 4 x int32
    assert ctypes.sizeof(_lib.SantaGeometry) == 56
    assert _lib.SantaGeometry.block_table.offset == 32
    assert _lib.SantaGeometry.reserved.offset == 52
    assert _lib.SantaSummary.max_groups.offset == 72


def test_workspace_queries_validate_arguments():
    lib = _lib.load()
    geo = _lib.SantaGeometry(8, 4, 7, 128, 32768, 32768, 32704, _lib.DTYPE_BF16)
    n = ctypes.c_size_t()
    assert lib.santa_build_summary_workspace_bytes(ctypes.byref(geo), 256, ctypes.byref(n)) == 0
    assert n.value > 0
    p = _lib.SantaDecodeParams(_lib.MODE_HYBRID, 16, 0, 256, 0.088, 0, 0, 0, 0)
    assert lib.santa_decode_workspace_bytes(ctypes.byref(geo), ctypes.byref(p), 256,
                                            ctypes.byref(n)) == 0
    bad = _lib.SantaGeometry(8, 4, 7, 96, 32768, 32768, 32704, _lib.DTYPE_BF16)
    assert lib.santa_decode_workspace_bytes(ctypes.byref(bad), ctypes.byref(p), 256,
                                            ctypes.byref(n)) == _lib.SANTA_ERR_UNSUPPORTED
    bad = _lib.SantaGeometry(8, 4, 7, 128, 32768, 32768, 40000, _lib.DTYPE_BF16)
    assert lib.santa_decode_workspace_bytes(ctypes.byref(bad), ctypes.byref(p), 256,
                                            ctypes.byref(n)) == _lib.SANTA_ERR_INVALID_ARGUMENT
    # 512 segments of 2M rows: the attention kernel's 32-bit row-cost scale would overflow
    big = _lib.SantaGeometry(64, 8, 4, 128, 1 << 21, 1 << 21, (1 << 21) - 64, _lib.DTYPE_BF16)
    assert lib.santa_decode_workspace_bytes(ctypes.byref(big), ctypes.byref(p), 256,
                                            ctypes.byref(n)) == _lib.SANTA_ERR_UNSUPPORTED
    p_bad = _lib.SantaDecodeParams(_lib.MODE_HYBRID, 16, 0, 5000, 0.088, 0, 0, 0, 0)
    assert lib.santa_decode_workspace_bytes(ctypes.byref(geo), ctypes.byref(p_bad), 256,
                                            ctypes.byref(n)) == _lib.SANTA_ERR_INVALID_ARGUMENT
    # a compute call without a workspace is refused before touching the device
    s = _lib.SantaSummary(*([256] * 9), 256)  # aligned dummy addresses, never dereferenced
    assert lib.santa_decode(ctypes.byref(geo), ctypes.byref(p), 1, 1, 1, ctypes.byref(s), None,
                            None, 1, 1, None, None, None, 0, None) == _lib.SANTA_ERR_WORKSPACE


def test_python_entry_points_refuse_cpu_tensors():
    import torch
    from santapp_b200.attention import santapp as S
    k = torch.zeros(1, 1, 16, 64)
    with pytest.raises(ValueError, match="CUDA"):
        S.build_summary(k, k, torch.zeros(1, 1, 8, dtype=torch.int64), 2, sample_end=8)


def test_build_is_sm100a():
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.ARCH_FLAGS)


def test_paged_geometry_is_validated():
    """Paged caches: page_size a power of two, capacity = max_pages x
    page_size, pool rows below 2^31 - 2 (the gather kernel's row codes).
    Workspace queries only validate: the table pointer is never read."""
    lib = _lib.load()
    n = ctypes.c_size_t()
    table = ctypes.c_void_p(4096)

    def geo(page_size, max_pages, num_pages, capacity=32768):
        return _lib.SantaGeometry(8, 4, 7, 128, capacity, 32768, 32704, _lib.DTYPE_BF16,
                                  table, page_size, max_pages, num_pages, 0)

    ok = geo(256, 128, 1024)
    assert lib.santa_build_summary_workspace_bytes(ctypes.byref(ok), 256, ctypes.byref(n)) == 0
    for bad in (geo(96, 342, 1024, capacity=96 * 342), geo(256, 64, 1024), geo(0, 128, 1024),
                geo(256, 128, 0)):
        assert lib.santa_build_summary_workspace_bytes(
            ctypes.byref(bad), 256, ctypes.byref(n)) == _lib.SANTA_ERR_INVALID_ARGUMENT
    huge = geo(1 << 16, 1, 1 << 13, capacity=1 << 16)   # 2^13 x 4 x 2^16 = 2^31 rows
    huge.n_total, huge.sample_end = 1 << 15, (1 << 15) - 64
    assert lib.santa_build_summary_workspace_bytes(
        ctypes.byref(huge), 256, ctypes.byref(n)) == _lib.SANTA_ERR_UNSUPPORTED


def test_paged_append_validates_arguments():
    lib = _lib.load()
    fake = ctypes.c_void_p(4096)
    args = [1, 1, 28, 4, 128] + [fake] * 7
    # page size not a power of two, then a missing table
    assert lib.santa_rope_append_paged(*args, fake, 96, 4, 4, 0, None, None,
                                       None) == _lib.SANTA_ERR_INVALID_ARGUMENT
    assert lib.santa_rope_append_paged(*args, None, 64, 4, 4, 0, None, None,
                                       None) == _lib.SANTA_ERR_INVALID_ARGUMENT
    # past the last page of the table
    assert lib.santa_rope_append_paged(*args, fake, 64, 4, 4, 256, None, None,
                                       None) == _lib.SANTA_ERR_INVALID_ARGUMENT


def test_peer_exchange_layout_matches_the_library():
    """The Python layout of a peer-memory exchange buffer (the one the
    emulated-shard GPU test writes words into) and the library's size query
    agree for every shard count the scaling runs use; shard counts past the
    limit are refused."""
    from santapp_b200.attention.sharded import exchange_layout
    lib = _lib.load()
    n = ctypes.c_size_t()
    for shards in (1, 2, 4, 8, _lib.MAX_SHARDS):
        for rows, topk, d in ((512, 32, 128), (224, 16, 128), (14, 8, 64)):
            assert lib.santa_p2p_buffer_bytes(shards, rows, topk, d, ctypes.byref(n)) == 0
            lay = exchange_layout(shards, rows, topk, d)
            assert n.value == lay["bytes"], (shards, rows, topk, d)
            # regions in order, keys after the set-up block, lines 16-byte aligned
            assert lay["keys"] < lay["parts"] < lay["stage"] < lay["bytes"]
            assert lay["parts"] % 16 == 0 and lay["stage"] % 16 == 0
            assert lay["parts"] - lay["keys"] >= 2 * shards * rows * topk * 8
    assert lib.santa_p2p_buffer_bytes(_lib.MAX_SHARDS + 1, 512, 32, 128, ctypes.byref(n)) != 0
    assert lib.santa_p2p_buffer_bytes(2, 0, 32, 128, ctypes.byref(n)) != 0


def test_exchange_words_carry_the_epoch():
    """Key words carry the tag epoch % 255 + 1 in bits 24-31 (the byte a
    global cluster id below 2^24 - 1 leaves all ones) and partial words the
    32-bit epoch in the high half, so a consumer tells this step's words from
    the previous step's in the same parity slot (epochs two apart)."""
    import torch
    from santapp_b200.attention.sharded import key_words, partial_words
    order = torch.tensor([0x3F800000 | 0x80000000, 0x40000000 | 0x80000000], dtype=torch.int64)
    cid = torch.tensor([5, (1 << 24) - 2], dtype=torch.int64)
    keys = (order << 32) | (0xFFFFFFFF - cid)
    for epoch in (1, 2, 254, 255, 256, 1000):
        w = key_words(keys, epoch)
        tag = (w >> 24) & 0xFF
        assert bool((tag == epoch % 255 + 1).all())
        assert int(((key_words(keys, epoch + 2) >> 24) & 0xFF)[0]) != int(tag[0])
        # everything but the tag byte is the key's
        assert bool(((w & -0xFF000001) == (keys & -0xFF000001)).all())
        p = torch.tensor([1.5, -2.25, 0.0], dtype=torch.float32)
        pw = partial_words(p, epoch)
        assert bool((((pw >> 32) & 0xFFFFFFFF) == epoch).all())
        assert torch.equal((pw & 0xFFFFFFFF).to(torch.int32).view(torch.float32), p)
