"""The C-ABI library loads and exports every entry point include/pir2b.h
declares (no compute calls: this runs without a GPU)."""

import ctypes
import os
import re

import pytest

from pir2_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pir2b.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pir2b_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert {"pir2b_quant_rows", "pir2b_gemm", "pir2b_norm_quant_rows", "pir2b_pack_nvfp4"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name
    assert set(declared()) <= set(_lib.SIGNATURES)


def test_version_and_error_string_without_gpu():
    lib = _lib.lib()
    assert lib.pir2b_version() >= 100
    assert isinstance(lib.pir2b_last_error(), bytes)


def test_argument_errors_are_reported_without_touching_the_device():
    lib = _lib.lib()
    status = lib.pir2b_quant_rows(None, 0, None, 0, None, None, 0, 3, 1, 8, None, None, None)
    assert status == _lib.EINVAL
    assert b"bits" in lib.pir2b_last_error()
    status = lib.pir2b_gemm(None, None, None, None, None, 0, None, None, 0, 8, 1, 12, 128, None, 12, 12, -1, None)
    assert status == _lib.EINVAL
    with pytest.raises(ValueError, match="npad"):
        _lib.check(status, "pir2b_gemm")
    # head_dim % 8 != 0, then a key sequence beyond the shared-memory kernel.
    status = lib.pir2b_attention_rows(None, 48, None, 48, None, 48, None, 48, 1, 1, 1, 4, 12, 1.0, None)
    assert status == _lib.EINVAL and b"head_dim" in lib.pir2b_last_error()
    status = lib.pir2b_attention_rows(None, 192, None, 192, None, 192, None, 192, 1, 1, 1 << 21, 4, 48, 1.0, None)
    assert status == _lib.EINVAL
    # Causal attention: head_dim 64 is not instantiated; hq not a multiple of hk.
    status = lib.pir2b_attention_causal(None, None, None, 1, 16, 16, 8, 64, 1.0, None, 2048, None)
    assert status == _lib.EINVAL and b"head_dim 128" in lib.pir2b_last_error()
    status = lib.pir2b_attention_causal(None, None, None, 1, 16, 12, 8, 128, 1.0, None, 2048, None)
    assert status == _lib.EINVAL


def _plan(lib, bits, m, npad, kpad):
    out = [ctypes.c_int() for _ in range(4)] + [ctypes.c_int64(), ctypes.c_int(), ctypes.c_int()]
    status = lib.pir2b_gemm_plan(bits, m, npad, kpad, 148, *[ctypes.byref(v) for v in out])
    return status, [v.value for v in out]


def test_gemm_planner_always_returns_a_launchable_plan():
    """Host-side sweep of the tile planner (no GPU): every plan covers all
    rows, fits the 227 KB opt-in shared memory, keeps split-K partials and
    staging inside the stage buffers and uses a power-of-two cluster."""
    lib = _lib.lib()
    lib.pir2b_gemm_plan.restype = ctypes.c_int
    for bits in (8, 4):
        for m in (1, 2, 15, 16, 17, 33, 64, 65, 128, 200, 256, 257, 300, 544, 1024, 1088, 4096):
            for k in (128, 256, 1536, 2048, 6144):
                for n in (8, 64, 520, 1536, 2048, 4096, 6144, 12288, 52224):
                    status, (bn, mt, splits, stages, smem, wt, pair) = _plan(lib, bits, m, n, k)
                    assert status == 0, (bits, m, k, n)
                    assert bn % 16 == 0 and 16 <= bn <= 256
                    assert bn * mt >= m and bn * (mt - 1) < m
                    assert splits in (1, 2, 4, 8) and splits <= k // 128
                    assert 2 <= stages <= 12 and 0 < smem <= 232448
                    if pair:
                        # 2-SM tiles: int8, more than 64 tokens, no split-K,
                        # each CTA stages half of the token tile, and the
                        # output tiles fit the idle stage ring.
                        assert bits == 8 and m > 64 and splits == 1 and bn >= 32 and wt in (1, 2)
                        assert stages * (16384 * wt + bn * 64) >= wt * bn * 256
                        continue
                    assert wt in (1, 2) and (wt == 1 or (bits == 8 and splits == 1 and stages >= 3))
                    if splits > 1:
                        assert stages * (16384 + bn * 128) >= bn * (512 + 128)


def test_vlm_prefill_plans_fill_the_machine_in_one_wave():
    """Many-token int8 GEMMs take 2-SM tiles (each CTA of a pair stages half
    of the token tile; persistent over tiles): every M = 544 projection of
    the VLM prefill, and the batched M = 34816 ones.  A long K that the
    one-SM plan splits over a cluster keeps the one-SM plan when the pair
    grid would have at most 64 CTAs (M = 128 / 256, K = 6144, N = 2048)."""
    lib = _lib.lib()
    lib.pir2b_gemm_plan.restype = ctypes.c_int
    for m in (544, 34816):
        for k, n in ((2048, 4096), (2048, 2048), (2048, 12288), (6144, 2048), (1536, 6144)):
            status, (bn, mt, splits, stages, smem, wt, pair) = _plan(lib, 8, m, n, k)
            assert status == 0 and pair == 1 and splits == 1 and bn % 64 == 0, (m, k, n)
    for m in (128, 256):
        status, (bn, mt, splits, stages, smem, wt, pair) = _plan(lib, 8, m, 2048, 6144)
        assert status == 0 and pair == 0 and splits > 1, m
