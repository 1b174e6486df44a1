"""The allocation-free GEMM entry point (ov_gemm_f16_noalloc).

Some callers cannot call cudaMalloc (a host that gave all device memory to
its own pool, or a latency-critical path where an allocation would block
on the device).  ov_gemm_f16_noalloc serves them from a static device
array.  Its output must match the allocating entry point ov_gemm_f16 (given
a workspace of its own) within the GEMM tolerance of the other tests, on
two calls in a row, since every call reuses the same static scratch.

This file is collected last so a failure here stops a `-x` run only after
every other test has run; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest

torch = pytest.importorskip("torch")

from omnivoice_b200 import _native as N  # noqa: E402

pytestmark = pytest.mark.gpu


def _ok(status):
    if status != 0:
        raise AssertionError(N.last_error())


@pytest.mark.parametrize("M,N_,K,epi,tile", [(240, 1024, 3072, N.OV_EPI_ACCUM_F32, None),
                                             (620, 1024, 2048, N.OV_EPI_ACCUM_F32, None),
                                             (500, 8200, 1024, N.OV_EPI_STORE_F32, None),
                                             (620, 1024, 3072, N.OV_EPI_ACCUM_F32, "128x4"),
                                             (240, 1024, 2048, N.OV_EPI_ACCUM_F32, "64x2")])
def test_noalloc_gemm_matches_allocating_entry_point(cuda_device, native, monkeypatch, M, N_, K,
                                                     epi, tile):
    if tile is not None:
        # Serialised split-K (the tile chooser reads OV_GEMM_TILE on every
        # call): the splits of a tile add into y in order behind a per-tile
        # counter, and those counters are what the static array holds.
        monkeypatch.setenv("OV_GEMM_TILE", tile)
        bn, splits = map(int, tile.split("x"))
        tiles = -(-M // 128) * -(-N_ // bn)
        assert native.ov_gemm_workspace_bytes(M, K, N_, epi) == 4 * tiles
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g).half().cuda()
    w = (torch.randn(N_, K, generator=g) * 0.02).half().cuda()
    base = torch.randn(M, N_, generator=g).cuda()
    need = native.ov_gemm_workspace_bytes(M, K, N_, epi)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    want = base.clone()
    _ok(native.ov_gemm_f16(x.data_ptr(), K, w.data_ptr(), want.data_ptr(), N_, M, K, N_, epi,
                           None, ws.data_ptr(), ws.numel(), stream))
    ref = x.double() @ w.double().T
    if epi == N.OV_EPI_ACCUM_F32:
        ref = ref + base.double()
    bound = K * 2.0 ** -23 * (x.double().abs() @ w.double().abs().T) + 1e-5 * base.double().abs() + 1e-6
    for _ in range(3):  # calls in a row share the static scratch
        got = base.clone()
        _ok(native.ov_gemm_f16_noalloc(x.data_ptr(), K, w.data_ptr(), got.data_ptr(), N_, M, K,
                                       N_, epi, None, stream))
        torch.cuda.synchronize()
        assert ((got.double() - ref).abs() <= bound).all()
        assert ((got.double() - want.double()).abs() <= bound).all()
    # Reads (and clears) the library's error word and this entry point's
    # own status word: no bounded wait of any call above ran out.
    flags = ctypes.c_uint32()
    _ok(native.ov_take_device_errors(ctypes.byref(flags), stream))
    assert flags.value == 0
