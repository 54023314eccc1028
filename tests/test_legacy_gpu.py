"""Legacy-path comparison on the same GPU: ThunderKittens-SM7x's own GEMM and
attention kernels (src/gemm.cu, src/attention.cu), built as compute_75 PTX by
``make -C oracle legacy`` and JIT-compiled by the driver, next to the sm_100a
library. The reference's results are checked against the oracle with the same
bounds as ours, and the timing datapoint is printed (run with ``-s`` to see it):

    python -m pytest tests/test_legacy_gpu.py -m gpu -s

This is a sanity datapoint for the legacy WMMA path on B200, not a Blackwell
reference."""

import math

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from oracle import fixtures as fx
from cuda_util import dev, host

pytestmark = pytest.mark.gpu


def legacy():
    lib = oracle.legacy_lib()
    if lib is None:
        pytest.skip("oracle/_ref/libtk_legacy.so not built (make -C oracle legacy needs the reference sources)")
    return lib


def test_legacy_gemm_256_matches_oracle_and_native():
    """Config 1 (256^3, seed 0, uniform [-1, 1]): both paths within error_bound(k, S)."""
    lib = legacy()
    m = n = k = 256
    a, b = oracle.gen_gemm_uniform(0, m, n, k, k, n)
    da, db = dev(a), dev(b)
    c_legacy = torch.full((m, n), float("nan"), device="cuda")
    assert lib.tkl_gemm_f16_f16_f32_nn(m, n, k, da.data_ptr(), k, db.data_ptr(), n, c_legacy.data_ptr(), n,
                                       None) == 0
    c_native = tk_b200.gemm(da, db)
    torch.cuda.synchronize()
    r, s = oracle.gemm_ref(m, n, k, a, k, b, n)
    legacy_c, native_c = host(c_legacy), host(c_native)
    assert oracle.gemm_check(k, legacy_c, r, s, n, n)[0] == 0
    assert oracle.gemm_check(k, native_c, r, s, n, n)[0] == 0
    same = np.mean(legacy_c.view(np.uint32) == native_c.view(np.uint32))
    print(f"\nlegacy vs sm_100a GEMM 256^3: {100 * same:.1f} % of cells bit-identical, "
          f"max |diff| {np.max(np.abs(legacy_c - native_c)):.3g}")


@pytest.mark.parametrize("case", fx.ATTENTION_CASES, ids=lambda c: c[0])
def test_legacy_attention_tile_cases(case):
    """The reference's own kernel on this GPU meets its own bound, and the sm_100a
    entry point agrees with it on every exact-equality cell."""
    lib = legacy()
    name, which, causal, exact_uniform, midpoint, exact_large, identity_v = case
    q, k, v = fx.attention_inputs(which)
    qkv = dev(np.concatenate([q.reshape(-1), k.reshape(-1), v.reshape(-1)]))
    qp = qkv.data_ptr()
    kp, vp = (qp, qp) if which == fx.ATT_ALIAS else (qp + 512, qp + 1024)
    out_legacy = torch.full((256,), float("nan"), device="cuda")
    out_native = torch.full((256,), float("nan"), device="cuda")
    assert lib.tkl_attention_forward_16x16(qp, kp, vp, out_legacy.data_ptr(), 1 if causal else 0, None) == 0
    assert tk_b200.attention_16x16_raw(qp, kp, vp, out_native, causal) == 0
    torch.cuda.synchronize()
    want = oracle.attention_ref(q, k, v, 16, 16, 0.25, causal)
    bound = oracle.attention_bound(v, 16, 16)[None, :]
    got_legacy = host(out_legacy).reshape(16, 16)
    got_native = host(out_native).reshape(16, 16)
    assert np.all(np.abs(got_legacy - want) <= bound)
    exact = fx.attention_exact_mask(exact_uniform, midpoint, exact_large, causal, identity_v)
    assert np.array_equal(got_legacy[exact], got_native[exact])


def _time(fn, iters):
    fn()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iters):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / iters


def _best_of(fn, reps=5, warm=2):
    """The reference's bench method (bench/gemm_throughput.cu:94-120): best of
    `reps` event-timed calls after `warm` warm-up calls, in ms."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    best = math.inf
    for _ in range(reps):
        best = min(best, _time(fn, 1))
    return best


def test_legacy_path_datapoint():
    """GEMM at the reference bench's square sizes (bench/gemm_throughput.cu:22-30, plus
    256 and 8192) and the one-tile attention per public call
    (bench/attention_throughput.cu:128-165), through both paths on this GPU."""
    lib = legacy()
    gen = torch.Generator(device="cuda").manual_seed(2)
    lines = [f"legacy-path datapoint on {torch.cuda.get_device_name()}"]
    native_8192 = legacy_8192 = None
    for size in (256, 512, 1024, 2048, 4096, 8192):
        m = n = k = size
        a = (torch.rand(m, k, device="cuda", generator=gen) * 2 - 1).half()
        b = (torch.rand(k, n, device="cuda", generator=gen) * 2 - 1).half()
        c = torch.empty(m, n, device="cuda")
        flops = 2.0 * m * n * k
        ms_legacy = _best_of(lambda: lib.tkl_gemm_f16_f16_f32_nn(m, n, k, a.data_ptr(), k, b.data_ptr(), n,
                                                                  c.data_ptr(), n, None),
                             reps=3 if size == 8192 else 5)
        ms_native = _best_of(lambda: tk_b200.gemm_raw(m, n, k, a, k, b, n, c, n))
        lines.append(f"  GEMM {size}^3: legacy {1e3 * ms_legacy:9.1f} us {flops / ms_legacy / 1e9:8.1f} TFLOP/s | "
                     f"sm_100a {1e3 * ms_native:8.1f} us {flops / ms_native / 1e9:8.1f} TFLOP/s | "
                     f"x{ms_legacy / ms_native:.1f}")
        if size == 8192:
            native_8192, legacy_8192 = ms_native, ms_legacy
    q = torch.zeros(256, dtype=torch.float16, device="cuda")
    out = torch.empty(256, device="cuda")
    for causal in (0, 1):
        us_legacy = 1e3 * _time(lambda: lib.tkl_attention_forward_16x16(q.data_ptr(), q.data_ptr(), q.data_ptr(),
                                                                          out.data_ptr(), causal, None), 2000)
        us_native = 1e3 * _time(lambda: tk_b200.attention_16x16_raw(q, q, q, out, bool(causal)), 2000)
        lines.append(f"  attention 16x16{' causal' if causal else ''} per call: legacy {us_legacy:.2f} us | "
                     f"sm_100a {us_native:.2f} us")
    print("\n" + "\n".join(lines))
    assert math.isfinite(legacy_8192) and native_8192 < legacy_8192
