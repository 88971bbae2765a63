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
