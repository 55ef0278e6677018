"""The C-ABI library loads, exports every declared entry point, and validates arguments (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from cutex_b200 import _lib
from cutex_b200.kernels import dense_gemm_contract as C

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = h.read_text()
        names += re.findall(r"CUTEX_API\s+[\w\s\*]+?\b(cutex_\w+)\s*\(", text)
    return names


def test_header_declares_the_abi():
    names = declared_functions()
    assert "cutex_mxfp8_gemm" in names and "cutex_mxfp8_query" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_checked_build_exports_the_same_abi():
    """libcutex_mxfp8_checked.so (-DCUTEX_CHECKED) is built beside the product library
    with the same entry points; only it reports itself as checked."""

    from cutex_b200.build import CHECKED_LIB_PATH

    checked = ctypes.CDLL(str(CHECKED_LIB_PATH))
    for name in declared_functions():
        assert hasattr(checked, name), name
    checked.cutex_version.restype = ctypes.c_char_p
    assert checked.cutex_build_checked() == 1 and checked.cutex_version().decode().endswith(" checked")
    lib = _lib.load()
    assert lib.cutex_build_checked() == 0 and not _lib.version().endswith("checked")
    # The product build's self-test launches nothing; argument checks come before any CUDA call.
    assert lib.cutex_selftest_device_check(None) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert lib.cutex_device_check_record(None, None, None) == _lib.CUTEX_ERR_INVALID_ARGUMENT


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_lib.GemmConfigC) == 16 * 4
    assert ctypes.sizeof(_lib.GemmInfoC) == 14 * 4 + 8
    assert _lib.GemmInfoC.scheduler.offset == 13 * 4
    assert ctypes.sizeof(_lib.EpilogueC) == 80
    assert _lib.EpilogueC.out_dtype.offset == 32 and _lib.EpilogueC.d_scales.offset == 40


def test_status_strings():
    for code in range(9):
        assert _lib.status_string(code).startswith("CUTEX_")
    assert "UNKNOWN" in _lib.status_string(99)
    assert _lib.version().startswith("cutex-b200")


FAKE = 1 << 20  # a 16-byte aligned non-null address; never dereferenced by argument validation


def gemm(a=FAKE, b=FAKE, sfa=FAKE, sfb=FAKE, d=FAKE, M=256, N=256, K=256, ldd=256, cfg=None, ws=None, wsb=0):
    c = cfg if cfg is not None else _lib.GemmConfigC()
    return _lib.load().cutex_mxfp8_gemm(a, b, sfa, sfb, d, M, N, K, ldd, ctypes.byref(c), ws, wsb, None)


def test_default_raster_group_follows_k():
    """CTA pairs, library choice: 16-tile groups at K <= 8192, 8 above; explicit groups are kept."""

    lib = _lib.load()

    def group(m, n, k, **cfg):
        info = _lib.GemmInfoC()
        c = _lib.make_config(**cfg)
        assert lib.cutex_mxfp8_query(ctypes.byref(c), m, n, k, ctypes.byref(info)) == 0
        return info.raster_group

    assert group(16384, 2048, 16384) == 8
    assert group(8192, 28672, 8192) == 16
    assert group(8192, 28672, 8192, raster_group=4) == 4
    assert group(4096, 4096, 4096, kernel=1, tile_n=128) == 8


@pytest.mark.parametrize(
    "kwargs,status",
    [
        ({"a": None}, _lib.CUTEX_ERR_INVALID_ARGUMENT),
        ({"d": None}, _lib.CUTEX_ERR_INVALID_ARGUMENT),
        ({"M": 0}, _lib.CUTEX_ERR_SHAPE),
        ({"K": -128}, _lib.CUTEX_ERR_SHAPE),
        ({"K": 200}, _lib.CUTEX_ERR_ALIGN),
        ({"N": 24, "ldd": 24}, _lib.CUTEX_ERR_ALIGN),
        ({"ldd": 255}, _lib.CUTEX_ERR_ALIGN),
        ({"ldd": 128}, _lib.CUTEX_ERR_ALIGN),
        ({"a": FAKE + 8}, _lib.CUTEX_ERR_ALIGN),
        ({"sfb": FAKE + 4}, _lib.CUTEX_ERR_ALIGN),
        ({"wsb": -1}, _lib.CUTEX_ERR_INVALID_ARGUMENT),
    ],
)
def test_gemm_argument_validation(kwargs, status):
    assert gemm(**kwargs) == status


def test_query_resolves_plans_without_launching():
    info = _lib.GemmInfoC()
    cfg = _lib.GemmConfigC()
    lib = _lib.load()
    assert lib.cutex_mxfp8_query(ctypes.byref(cfg), C.M, C.N, C.K, ctypes.byref(info)) == 0
    assert info.kernel == _lib.KERNEL_2CTA and info.tile_m == 256 and info.tile_n == 256
    assert info.cluster_size == 2 and info.num_tiles == 64 * 64
    assert info.smem_bytes <= 232448 and info.grid_ctas == 2 * 64 * 64 and info.scheduler == 0
    static = _lib.make_config(scheduler=1)
    assert lib.cutex_mxfp8_query(ctypes.byref(static), C.M, C.N, C.K, ctypes.byref(info)) == 0
    assert info.scheduler == 1 and info.grid_ctas <= 148
    bad = _lib.make_config(scheduler=2)
    assert lib.cutex_mxfp8_query(ctypes.byref(bad), 256, 256, 256, ctypes.byref(info)) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    cfg = _lib.make_config(kernel=1, tile_n=128, stages=5, scheduler=1)
    assert lib.cutex_mxfp8_query(ctypes.byref(cfg), 300, 272, 384, ctypes.byref(info)) == 0
    assert (info.tile_m, info.tile_n, info.stages, info.num_tiles) == (128, 128, 5, 3 * 3)
    bad = _lib.make_config(tile_n=96)
    assert lib.cutex_mxfp8_query(ctypes.byref(bad), 256, 256, 256, ctypes.byref(info)) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    bad = _lib.GemmConfigC()
    bad.reserved[3] = 1
    assert lib.cutex_mxfp8_query(ctypes.byref(bad), 256, 256, 256, ctypes.byref(info)) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    bad = _lib.make_config(stages=9)
    assert lib.cutex_mxfp8_query(ctypes.byref(bad), 256, 256, 256, ctypes.byref(info)) == _lib.CUTEX_ERR_INVALID_ARGUMENT


def test_quantize_argument_validation():
    lib = _lib.load()
    assert lib.cutex_mxfp8_quantize(None, 0, 4, 128, 128, FAKE, FAKE, None) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert lib.cutex_mxfp8_quantize(FAKE, 2, 4, 128, 128, FAKE, FAKE, None) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert lib.cutex_mxfp8_quantize(FAKE, 0, 4, 96, 96, FAKE, FAKE, None) == _lib.CUTEX_ERR_ALIGN
    assert lib.cutex_mxfp8_quantize(FAKE, 0, 0, 128, 128, FAKE, FAKE, None) == _lib.CUTEX_ERR_SHAPE


def test_python_wrapper_rejects_with_value_errors():
    from cutex_b200.kernels.dense_gemm import GemmConfig, query

    with pytest.raises(ValueError):
        query(256, 256, 200)
    with pytest.raises(ValueError):
        query(256, 256, 256, GemmConfig(tile_n=64))
    q = query(16, 28672, 8192)
    assert q["kernel"] == _lib.KERNEL_SKINNY and q["tile_m"] == 16 and q["split_k"] == 0
    assert q["workspace_bytes"] == 2 * 148 * 128 * 128 * 4 + 1024  # CPU-side default of 148 SMs
    q128 = query(128, 28672, 8192)
    assert q128["tile_m"] == 128 and q128["split_k"] == 0 and q128["workspace_bytes"] == q["workspace_bytes"]
    assert query(128, 28672, 8192, GemmConfig(kernel=_lib.KERNEL_SKINNY))["split_k"] == 0
    assert query(100, 256, 256, GemmConfig(split_k=1))["workspace_bytes"] == 0
    assert query(129, 256, 256)["kernel"] != _lib.KERNEL_SKINNY
    with pytest.raises(ValueError):
        query(200, 256, 256, GemmConfig(kernel=_lib.KERNEL_SKINNY))
    with pytest.raises(ValueError):
        query(16, 256, 256, GemmConfig(kernel=_lib.KERNEL_SKINNY, split_k=4))


def test_host_gemm_argument_checks_without_a_device():
    from cutex_b200.kernels import HostGemm

    with pytest.raises(_lib.CutexArgumentError):
        HostGemm(256, 256, 128, blocks=0)
    with pytest.raises(_lib.CutexArgumentError):
        HostGemm(256, 256, 128, blocks=17)
    with pytest.raises(ValueError):
        HostGemm(256, 250, 128)  # N not a multiple of 16


def test_columnwise_quantiser_rejects_bad_shapes_without_launching():
    lib = _lib.load()
    dummy = 256  # 16-byte aligned placeholder: every case is rejected before any launch
    assert lib.cutex_mxfp8_quantize_columnwise(dummy, 1, 100, 64, 64, dummy, dummy, None) == _lib.CUTEX_ERR_ALIGN
    assert lib.cutex_mxfp8_quantize_columnwise(dummy, 1, 128, 64, 60, dummy, dummy, None) == _lib.CUTEX_ERR_ALIGN
    assert lib.cutex_mxfp8_quantize_columnwise(dummy, 2, 128, 64, 64, dummy, dummy, None) == (
        _lib.CUTEX_ERR_INVALID_ARGUMENT)
    assert lib.cutex_mxfp8_quantize_columnwise(None, 1, 128, 64, 64, dummy, dummy, None) == (
        _lib.CUTEX_ERR_INVALID_ARGUMENT)
    assert lib.cutex_mxfp8_quantize_columnwise(dummy, 1, 0, 64, 64, dummy, dummy, None) == _lib.CUTEX_ERR_SHAPE


def test_fused_epilogue_argument_checks_without_launching():
    lib = _lib.load()
    p = 256  # 16-byte aligned placeholder: every case below is rejected before any launch
    cfg = _lib.make_config()

    def call(epi, M=256, N=256, K=128, ldd=256):
        return lib.cutex_mxfp8_gemm_ex(p, p, p, p, p, M, N, K, ldd, ctypes.byref(cfg), ctypes.byref(epi), None, 0,
                                       None)

    e = _lib.EpilogueC(alpha=1.0, out_dtype=2)
    assert call(e) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    e = _lib.EpilogueC(alpha=1.0, out_dtype=1)  # e4m3 out without a scale buffer
    assert call(e) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    e = _lib.EpilogueC(alpha=1.0, out_dtype=1, d_scales=p)
    assert call(e, N=272, ldd=272) == _lib.CUTEX_ERR_ALIGN  # N % 128 for the scale atoms
    e = _lib.EpilogueC(alpha=1.0, bias=p + 8)
    assert call(e) == _lib.CUTEX_ERR_ALIGN
    e = _lib.EpilogueC(alpha=1.0, beta=1.0, c=p, ldc=100)
    assert call(e) == _lib.CUTEX_ERR_ALIGN
    e = _lib.EpilogueC(alpha=1.0)
    e.reserved[2] = 1
    assert call(e) == _lib.CUTEX_ERR_INVALID_ARGUMENT


def test_allgather_argument_checks_without_launching():
    lib = _lib.load()
    p = 256  # 16-byte aligned placeholder: every case below is rejected before any CUDA call
    peers = (ctypes.c_void_p * 2)(p, p)

    def maps(n_peers=2, M=256, N=256, ldd=512, buf=p, nbytes=256):
        return lib.cutex_mxfp8_allgather_maps(peers, n_peers, M, N, ldd, buf, nbytes, None)

    assert maps(n_peers=0) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert maps(n_peers=8) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert maps(nbytes=128) == _lib.CUTEX_ERR_WORKSPACE  # 128 bytes per descriptor
    assert maps(buf=p + 16) == _lib.CUTEX_ERR_ALIGN
    assert maps(ldd=128) == _lib.CUTEX_ERR_ALIGN
    assert maps(M=0) == _lib.CUTEX_ERR_SHAPE
    assert lib.cutex_mxfp8_allgather_maps((ctypes.c_void_p * 2)(p, p + 2), 2, 256, 256, 512, p, 256, None) == (
        _lib.CUTEX_ERR_ALIGN)

    cfg = _lib.make_config()

    def gemm(n_peers=2, M=256, N=256, K=128, ldd=512, buf=p):
        return lib.cutex_mxfp8_gemm_allgather(p, p, p, p, p, M, N, K, ldd, buf, n_peers, ctypes.byref(cfg), None)

    assert gemm(n_peers=0) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert gemm(buf=None) == _lib.CUTEX_ERR_INVALID_ARGUMENT
    assert gemm(buf=p + 32) == _lib.CUTEX_ERR_ALIGN
    assert gemm(ldd=200) == _lib.CUTEX_ERR_ALIGN
