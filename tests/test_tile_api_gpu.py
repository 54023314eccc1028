"""The device-level tile API (include/tk_sm7x/tile_b200.cuh) from a user kernel,
and ports of the reference's examples/gemm_row_stats.cu and
examples/gemm_row_softmax.cu (a GEMM tile followed by row statistics / softmax)."""

import ctypes as C
import os
import subprocess

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from oracle import fixtures as fx
from cuda_util import dev, host

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.fixture(scope="module")
def tile_api(tmp_path_factory):
    so = tmp_path_factory.mktemp("tile_api") / "libtile_api.so"
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
                    "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "device_api", "tile_api_kernels.cu"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.tile_api_run.restype = C.c_int
    lib.tile_api_run.argtypes = [C.c_void_p, C.c_int, C.c_int] + [C.c_void_p] * 7
    lib.tile_scale_run.restype = C.c_int
    lib.tile_scale_run.argtypes = [C.c_void_p, C.c_void_p, C.c_float]
    return lib


def run_api(lib, tiles, ld=16):
    """tiles: (n, 16, 16) FP32; stored with leading dimension ld."""
    n = tiles.shape[0]
    buf = np.full((n, 16, ld), np.nan, dtype=np.float32)
    buf[:, :, :16] = tiles
    d_in = dev(buf)
    outs = [torch.full((n * 16,), float("nan"), device="cuda") for _ in range(5)]
    outs += [torch.full((n * 256,), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    assert lib.tile_api_run(d_in.data_ptr(), ld, n, *[o.data_ptr() for o in outs]) == 0
    return [host(o) for o in outs]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("ld", [16, 20, 17])
def test_tile_api_matches_reference_tree_and_batched_kernels(tile_api, ld):
    g = np.load(os.path.join(HERE, "golden", "row_reduce.npz"))
    tiles = np.concatenate([g["tiles"], oracle.gen_normal_f32(3, 2.0, 64 * 256).reshape(64, 16, 16)])
    sums, maxs, rsums, rmaxs, tsums, sm, cs = run_api(tile_api, tiles, ld)
    want_sum = oracle.tile_row_reduce(tiles, "sum").reshape(-1)
    want_max = oracle.tile_row_reduce(tiles, "max").reshape(-1)
    for got in (sums, rsums, tsums):
        assert np.array_equal(bits(got), bits(want_sum))
    for got in (maxs, rmaxs):
        assert np.array_equal(bits(got), bits(want_max))
    assert oracle.tile_row_softmax_check(tiles, sm, False)[0] == 0
    assert oracle.tile_row_softmax_check(tiles, cs, True)[0] == 0
    # The batched entry points are built on the same functions: identical bits.
    batched = tk_b200.tile_row_ops(dev(tiles.astype(np.float32)))
    assert np.array_equal(bits(host(batched["softmax"]).reshape(-1)), bits(sm))
    assert np.array_equal(bits(host(batched["causal"]).reshape(-1)), bits(cs))


@pytest.fixture(scope="module")
def refnames(tmp_path_factory):
    so = tmp_path_factory.mktemp("refnames") / "librefnames.so"
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
                    "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"),
                    os.path.join(HERE, "device_api", "refnames_kernels.cu"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.refnames_run.restype = C.c_int
    lib.refnames_run.argtypes = [C.c_void_p, C.c_int] + [C.c_void_p] * 4
    return lib


def test_reference_named_device_api(refnames):
    """tk_sm7x::row_sum / row_max / row_softmax / row_softmax_causal called with the
    reference's device signatures from <tk_sm7x/reduce.cuh> and <tk_sm7x/softmax.cuh>:
    sums and maxima bit-identical to the reference tree (golden tiles included),
    probabilities within 512 * 2^-23, causal zeros exact."""
    g = np.load(os.path.join(HERE, "golden", "row_reduce.npz"))
    tiles = np.concatenate([g["tiles"], oracle.gen_normal_f32(5, 2.0, 61 * 256).reshape(61, 16, 16)])
    n = tiles.shape[0]
    d_in = dev(np.ascontiguousarray(tiles, dtype=np.float32))
    outs = [torch.full((n * 16,), float("nan"), device="cuda") for _ in range(2)]
    outs += [torch.full((n * 256,), float("nan"), device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    assert refnames.refnames_run(d_in.data_ptr(), n, *[o.data_ptr() for o in outs]) == 0
    sums, maxs, sm, cs = [host(o) for o in outs]
    assert np.array_equal(bits(sums), bits(oracle.tile_row_reduce(tiles, "sum").reshape(-1)))
    assert np.array_equal(bits(maxs), bits(oracle.tile_row_reduce(tiles, "max").reshape(-1)))
    assert oracle.tile_row_softmax_check(tiles, sm, False)[0] == 0
    assert oracle.tile_row_softmax_check(tiles, cs, True)[0] == 0


def example_tile():
    """A and B of examples/gemm_row_stats.cu:74-80 (numerators / 8, exact in FP16)."""
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    a = ((r * 3 + c * 5) % 13 - 6) / 8.0
    b = ((r * 7 + c * 2) % 11 - 5) / 8.0
    return oracle.f32_to_f16_bits(a), oracle.f32_to_f16_bits(b), a @ b


def test_example_gemm_row_stats(tile_api):
    """examples/gemm_row_stats.cu:82-116: C, row sums and row maxima all exact."""
    a, b, exact = example_tile()
    c = host(tk_b200.gemm(dev(a), dev(b)))
    assert np.array_equal(c.astype(np.float64), exact)
    sums, maxs, *_ = run_api(tile_api, c[None])
    assert np.array_equal(sums.astype(np.float64), exact.sum(axis=1))
    assert np.array_equal(maxs.astype(np.float64), exact.max(axis=1))
    # The fused full-row statistics GEMM gives the same on this one-tile problem.
    _, mx, sm = tk_b200.gemm_rowstats(dev(a), dev(b))
    assert np.array_equal(host(mx).astype(np.float64), exact.max(axis=1))
    assert np.array_equal(host(sm).astype(np.float64), exact.sum(axis=1))


def test_example_gemm_row_softmax(tile_api):
    """examples/gemm_row_softmax.cu:90-140: exact logits, probabilities within
    512 * 2^-23 of FP64, each row summing to 1 within the same bound."""
    a, b, exact = example_tile()
    logits = host(tk_b200.gemm(dev(a), dev(b)))
    assert np.array_equal(logits.astype(np.float64), exact)
    *_, sm, _ = run_api(tile_api, logits[None])
    want = np.exp(exact - exact.max(axis=1, keepdims=True))
    want /= want.sum(axis=1, keepdims=True)
    got = sm.reshape(16, 16).astype(np.float64)
    assert np.all((got >= 0) & (got <= 1))
    assert np.max(np.abs(got - want)) <= oracle.SOFTMAX_BOUND
    assert np.all(np.abs(got.sum(axis=1) - 1.0) <= oracle.SOFTMAX_BOUND)


@pytest.mark.parametrize("factor", [0.25, -0.5])
def test_tile_scale_exact(tile_api, factor):
    """tests/tile_scale.cu:47-63: C = A B with A = diag((i + 1) / 16) and
    B[i][j] = (16 i + j - 128) / 8 (the library GEMM, exact for these values), then
    the tile scaled by a power of two in registers: every element exactly
    factor * (i + 1) / 16 * (16 i + j - 128) / 8."""
    i = np.arange(16)[:, None].astype(np.float32)
    j = np.arange(16)[None, :].astype(np.float32)
    a = np.where(i == j, (i + 1) / 16, 0).astype(np.float32)
    b = ((16 * i + j - 128) / 8).astype(np.float32)
    da = torch.from_numpy(a).half().cuda()
    db = torch.from_numpy(b).half().cuda()
    c = tk_b200.gemm(da, db)
    out = torch.full((256,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    assert tile_api.tile_scale_run(c.data_ptr(), out.data_ptr(), factor) == 0
    want = (np.float32(factor) * ((i + 1) / 16) * ((16 * i + j - 128) / 8)).astype(np.float32)
    assert np.array_equal(bits(host(out).reshape(16, 16)), bits(want))
