"""Batched 16x16 tile row ops on the GPU against the CPU oracle.

Reductions must be bit-exact (the reference's canonical tree,
tests/row_reduce_reference.cuh:16-24, signed-zero ties included); softmax must
stay within 512 * 2^-23 of the FP64 reference with exact causal zeros
(tests/tile_softmax.cu:20, tests/tile_causal_softmax.cu:86-110)."""

import os

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from oracle import fixtures as fx
from cuda_util import cudart, dev, host, seed_stale_error

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def run_all(tiles_np):
    t = dev(tiles_np.astype(np.float32))
    out = tk_b200.tile_row_ops(t)
    return {k: host(v) for k, v in out.items()}, t


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_golden_tiles_bit_exact():
    g = np.load(os.path.join(GOLDEN, "row_reduce.npz"))
    out, _ = run_all(g["tiles"])
    assert np.array_equal(bits(out["sum"]), bits(g["row_sum"]))
    assert np.array_equal(bits(out["max"]), bits(g["row_max"]))


def test_random_tiles_bit_exact_and_softmax_bound():
    tiles = oracle.gen_normal_f32(1, 2.0, 65536 * 256).reshape(-1, 16, 16)
    out, t = run_all(tiles)
    assert np.array_equal(bits(out["sum"]), bits(oracle.tile_row_reduce(tiles, "sum")))
    assert np.array_equal(bits(out["max"]), bits(oracle.tile_row_reduce(tiles, "max")))
    for causal, key in ((False, "softmax"), (True, "causal")):
        fails, err = oracle.tile_row_softmax_check(tiles, out[key], causal)
        assert fails == 0, (key, err)
        assert err <= oracle.SOFTMAX_BOUND
    # The source is unchanged by the call (tests/tile_reduce.cu:80-86).
    assert np.array_equal(bits(host(t).reshape(-1, 16, 16)), bits(tiles))


@pytest.mark.parametrize("kind", range(4))
def test_softmax_reference_fixtures(kind):
    logits = fx.softmax_logits(8, kind)
    out, _ = run_all(logits)
    fails, err = oracle.tile_row_softmax_check(logits, out["softmax"], False)
    assert fails == 0 and err <= oracle.SOFTMAX_BOUND
    # Repeating the call gives identical bits (tests/tile_softmax.cu:165).
    again, _ = run_all(logits)
    assert np.array_equal(bits(again["softmax"]), bits(out["softmax"]))


@pytest.mark.parametrize("extreme", [False, True])
def test_causal_softmax_reference_fixtures(extreme):
    logits = fx.causal_logits(extreme)[None]
    out, _ = run_all(logits)
    fails, err = oracle.tile_row_softmax_check(logits, out["causal"], True)
    assert fails == 0, err
    r, c = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
    assert np.all(bits(out["causal"][0][c > r]) == 0)  # exactly +0.0


def test_single_op_entry_points_match_fused():
    tiles = oracle.gen_normal_f32(7, 2.0, 512 * 256)
    t = dev(tiles)
    fused, _ = run_all(tiles)
    lib = tk_b200.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for fn, key, shape in ((lib.tk_tile_row_sum_f32, "sum", (512, 16)), (lib.tk_tile_row_max_f32, "max", (512, 16)),
                           (lib.tk_tile_row_softmax_f32, "softmax", (512, 16, 16)),
                           (lib.tk_tile_row_softmax_causal_f32, "causal", (512, 16, 16))):
        o = torch.full(shape, float("nan"), device="cuda")
        assert fn(t.data_ptr(), 512, o.data_ptr(), stream) == 0
        assert np.array_equal(bits(host(o)), bits(fused[key])), key


def test_in_place_softmax_and_unaligned_path():
    tiles = oracle.gen_normal_f32(8, 2.0, 300 * 256)
    want, _ = run_all(tiles)
    lib = tk_b200.lib()
    stream = torch.cuda.current_stream().cuda_stream
    t = dev(tiles)
    assert lib.tk_tile_row_softmax_f32(t.data_ptr(), 300, t.data_ptr(), stream) == 0
    assert np.array_equal(bits(host(t)), bits(want["softmax"].reshape(-1)))
    # 4-byte but not 16-byte aligned input and outputs take the scalar path.
    buf = torch.zeros(300 * 256 + 1, device="cuda")
    buf[1:] = torch.from_numpy(tiles).cuda()
    outs = torch.full((300 * 16 + 1,), float("nan"), device="cuda")
    outm = torch.full((300 * 256 + 1,), float("nan"), device="cuda")
    assert lib.tk_tile_row_ops_f32(buf.data_ptr() + 4, 300, outs.data_ptr() + 4, None, outm.data_ptr() + 4,
                                   None, stream) == 0
    assert np.array_equal(bits(host(outs)[1:]), bits(want["sum"].reshape(-1)))
    assert np.array_equal(bits(host(outm)[1:]), bits(want["softmax"].reshape(-1)))


def test_empty_and_ragged_counts():
    lib = tk_b200.lib()
    stream = torch.cuda.current_stream().cuda_stream
    t = torch.zeros(256, device="cuda")
    o = torch.full((16,), 7.0, device="cuda")
    assert lib.tk_tile_row_sum_f32(t.data_ptr(), 0, o.data_ptr(), stream) == 0
    assert torch.all(o == 7.0)
    for n in (1, 3, 17, 33, 4097):  # tile counts that leave warps and blocks partly idle
        tiles = oracle.gen_normal_f32(n, 2.0, n * 256)
        guard = torch.full((n * 16 + 64,), float("nan"), device="cuda")
        assert lib.tk_tile_row_max_f32(dev(tiles).data_ptr(), n, guard.data_ptr() + 32 * 4, stream) == 0
        g = host(guard)
        assert np.array_equal(bits(g[32:32 + n * 16]), bits(oracle.tile_row_reduce(tiles, "max").reshape(-1)))
        assert np.all(np.isnan(g[:32])) and np.all(np.isnan(g[32 + n * 16:]))  # guard words untouched


def test_error_state_contract():
    rt = cudart()
    lib = tk_b200.lib()
    t = torch.zeros(256, device="cuda")
    o = torch.full((16,), 5.0, device="cuda")
    torch.cuda.synchronize()
    code = seed_stale_error()
    # Invalid call: cudaErrorInvalidValue, stale error preserved, consumed exactly once.
    assert lib.tk_tile_row_sum_f32(None, 1, o.data_ptr(), None) == tk_b200.CUDA_ERROR_INVALID_VALUE
    assert rt.cudaPeekAtLastError() == code
    assert rt.cudaGetLastError() == code
    assert rt.cudaPeekAtLastError() == 0
    assert torch.all(o == 5.0)
    # Valid call clears a stale error.
    seed_stale_error()
    assert lib.tk_tile_row_sum_f32(t.data_ptr(), 1, o.data_ptr(), None) == 0
    assert rt.cudaPeekAtLastError() == 0
    torch.cuda.synchronize()
    assert torch.all(o == 0.0)


def test_full_size_sweep_properties():
    """1,048,576 tiles (1 GiB) from std::mt19937(1), N(0, 4): reductions bit-exact on
    every tile; softmax within bound on a sample that includes the first and last tiles."""
    n = 1 << 20
    tiles = oracle.gen_normal_f32(1, 2.0, n * 256)
    t = dev(tiles)
    out = tk_b200.tile_row_ops(t)
    s, m = host(out["sum"]), host(out["max"])
    assert np.array_equal(bits(s), bits(oracle.tile_row_reduce(tiles, "sum")))
    assert np.array_equal(bits(m), bits(oracle.tile_row_reduce(tiles, "max")))
    rng = np.random.default_rng(0)
    idx = np.unique(np.concatenate([[0, n - 1], rng.integers(0, n, 8192)]))
    tiles3 = tiles.reshape(n, 16, 16)
    for key, causal in (("softmax", False), ("causal", True)):
        got = out[key][torch.from_numpy(idx).cuda()]
        fails, err = oracle.tile_row_softmax_check(tiles3[idx], host(got), causal)
        assert fails == 0, (key, err)
