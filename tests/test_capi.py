"""The C-ABI library builds for sm_100a, loads without a GPU and exports every entry point the header
declares (host-only entry points are callable here)."""

import os
import re

from viktor_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "viktor_b200.h")).read()
    return sorted(set(re.findall(r"^(?:int|size_t)\s+(vk_\w+)\(", src, re.M)))


def test_header_and_binding_agree():
    assert declared() == sorted(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared():
        assert hasattr(lib, name), name


def test_host_only_entry_points():
    lib = _lib.load()
    assert lib.vk_version() >= 100
    # split-K workspace: tickets + (m, l) + partial outputs, grows with the number of 256-position splits
    a = lib.vk_decode_attention_workspace_bytes(256, 3200)
    b = lib.vk_decode_attention_workspace_bytes(256, 3200 + 256)
    assert a > 256 * 13 * 8 * 64 * 4 and b > a
    assert lib.vk_decode_attention_workspace_bytes(0, 100) == 0


def test_argument_errors_are_status_codes():
    """Bad arguments come back as VK_ERR_ARG without touching a device."""
    lib = _lib.load()
    assert lib.vk_add_rmsnorm(None, None, None, None, 4, 512, 1e-6, None) == _lib.VK_ERR_ARG
    assert lib.vk_add_rmsnorm(None, None, None, None, 0, 512, 1e-6, None) == _lib.VK_OK
    assert lib.vk_linear(None, None, None, 4, 64, 512, 0, 0, None) == _lib.VK_ERR_ARG
    # the failure-path probe: its wait limit must lie in (0, 1 s]
    assert lib.vk_test_bounded_wait(0, None, None) == _lib.VK_ERR_ARG
    assert lib.vk_test_bounded_wait(2_000_000_000, None, None) == _lib.VK_ERR_ARG
    assert lib.vk_decode_attention(None, None, None, None, None, 4, 0, 4, 100, 12800, 128, None, 0,
                                   None) == _lib.VK_ERR_ARG
    # sampling needs the noise buffer and a positive, finite temperature
    fake = 16  # any non-null address: validation fails before anything is dereferenced
    ptrs = [fake] * 6  # tok, run, pos, plen, rope_off, out
    assert lib.vk_sample_update(fake, 7, fake, fake, fake, 0, *ptrs, 4, 4, fake, fake, fake, 2, 7, 2, 0, None,
                                None, None, None, 7, 0.7, None) == _lib.VK_ERR_ARG
    for t in (0.0, -1.0, float("inf"), float("nan")):
        assert lib.vk_sample_update(fake, 7, fake, fake, fake, 0, *ptrs, 4, 4, fake, fake, fake, 2, 7, 2, 0, None,
                                    None, None, fake, 7, t, None) == _lib.VK_ERR_ARG
    assert lib.vk_sample_update(fake, 7, fake, fake, fake, 0, *ptrs, 4, 4, fake, fake, fake, 2, 7, 2, 0, None,
                                None, None, fake, 6, 0.7, None) == _lib.VK_ERR_ARG  # ld_noise < V


def test_int8_prefix_entry_points_validate_arguments():
    """The int8 prefix entry points: workspace sizing (host only) and argument checks that fail before any
    device access (S8 a multiple of 128, 0 < max_tail <= S, the workspace large enough, no null pointers)."""
    lib = _lib.load()
    w = lib.vk_decode_attention_i8_workspace_bytes(128, 2176, 1101)
    assert w > 0 and lib.vk_decode_attention_i8_workspace_bytes(128, 2176, 2202) > w
    assert lib.vk_decode_attention_i8_workspace_bytes(0, 2176, 1101) == 0
    fake = 16  # any 16-byte-aligned non-null address: validation fails before anything is dereferenced
    S, rows = 3200, 128

    def attn(S8=2176, max_tail=1101, ws_bytes=w, q=fake):
        return lib.vk_decode_attention_i8(q, fake, fake, fake, fake, fake, fake, fake, fake, fake, rows, 0, rows, S,
                                          S * 128, 128, S8, max_tail, fake, ws_bytes, None)

    assert attn(S8=2100) == _lib.VK_ERR_ARG          # not a multiple of 128
    assert attn(max_tail=0) == _lib.VK_ERR_ARG
    assert attn(max_tail=S + 1) == _lib.VK_ERR_ARG
    assert attn(ws_bytes=w - 1) == _lib.VK_ERR_ARG   # workspace too small
    assert attn(q=None) == _lib.VK_ERR_ARG
    assert lib.vk_kv_quantize(fake, fake, rows, S, S * 128, 128, fake, 0, rows, fake, fake, fake, fake, 2100,
                              None) == _lib.VK_ERR_ARG
    assert lib.vk_kv_quantize(fake, fake, rows, S, S * 128, 128, None, 0, rows, fake, fake, fake, fake, 2176,
                              None) == _lib.VK_ERR_ARG
    assert lib.vk_kv_quantize(fake, fake, rows, S, S * 128, 128, fake, 1, rows, fake, fake, fake, fake, 2176,
                              None) == _lib.VK_ERR_ARG  # rows past the cache
    assert lib.vk_kv_quantize(None, None, 0, 0, 0, 0, None, 0, 0, None, None, None, None, 0, None) == _lib.VK_OK


def test_stitch_entry_points_validate_arguments():
    lib = _lib.load()
    out = (_lib.C.c_int * 3)()
    assert lib.vk_align(None, 3, b"ACG", 3, 0, -1, out, None, 0) == _lib.VK_ERR_ARG
    assert lib.vk_align(b"ACG", 3, b"ACG", 3, 3, -1, out, None, 0) == _lib.VK_ERR_ARG  # unknown mode
    buf = _lib.C.create_string_buffer(4)
    assert lib.vk_align(b"ACG", 3, b"ACG", 3, 0, -1, out, buf, 4) == _lib.VK_ERR_ARG  # CIGAR buffer too small
    cut = (_lib.C.c_int * 2)()
    assert lib.vk_overlap_cut(None, 5, b"ACGTA", 5, 10, 1.0, cut) == _lib.VK_ERR_ARG
    n = _lib.C.c_int64(0)
    assert lib.vk_stitch(None, None, None, 2, 6, None, 0, _lib.C.byref(n)) == _lib.VK_ERR_ARG
    assert lib.vk_stitch(None, None, None, 0, 6, None, 0, _lib.C.byref(n)) == _lib.VK_OK and n.value == 0
