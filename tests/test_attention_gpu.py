"""Attention forward on the GPU through the C ABI, against the CPU oracle.

The ten one-tile cases of the reference (tests/attention_correctness.cu:263-324)
with its bound (512 * 2^-23 + 2^-11 + gamma(32)) * sum_t |V[t, c]| and its
exact-equality cells; then general [B, H, S, D] shapes with the bound
generalised to gamma(2S)."""

import math

import numpy as np
import pytest
import torch

import oracle
import tk_b200
from oracle import fixtures as fx
from cuda_util import cudart, dev, host, seed_stale_error

pytestmark = pytest.mark.gpu

GUARD_BEFORE, GUARD_AFTER = -12345.0, 12345.0  # tests/attention_correctness.cu:22-23


@pytest.fixture(params=[1, 2], ids=["cta1", "cta_pair"])
def attn_kernel(request):
    """head_dim 128 multi-block problems have two kernels: the single-CTA one (1, the
    default) and the CTA-pair one (2, tcgen05 cta_group::2). Both run every case."""
    lib = tk_b200.lib()
    old = lib.tk_attention_set_cta_group(request.param)
    try:
        yield request.param
    finally:
        lib.tk_attention_set_cta_group(old)


def run_tile(q, k, v, causal, stream=None, alias=False):
    qkv = dev(np.concatenate([q.reshape(-1), k.reshape(-1), v.reshape(-1)]))
    buf = torch.full((258,), float("nan"), device="cuda")
    buf[0], buf[257] = GUARD_BEFORE, GUARD_AFTER
    qp = qkv.data_ptr()
    kp, vp = (qp, qp) if alias else (qp + 512, qp + 1024)
    s = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    assert tk_b200.attention_16x16_raw(qp, kp, vp, buf.data_ptr() + 4, causal, s) == 0
    if stream is not None:
        stream.synchronize()
    out = host(buf)
    assert out[0] == GUARD_BEFORE and out[257] == GUARD_AFTER
    return out[1:257].reshape(16, 16)


@pytest.mark.parametrize("case", fx.ATTENTION_CASES, ids=lambda c: c[0])
def test_reference_tile_cases(case):
    name, which, causal, exact_uniform, midpoint, exact_large, identity_v = case
    q, k, v = fx.attention_inputs(which)
    want, prob = oracle.attention_ref(q, k, v, 16, 16, 0.25, causal, want_prob=True)
    stream = torch.cuda.Stream()  # a non-blocking stream, as the reference test uses
    got = run_tile(q, k, v, causal, stream=stream, alias=which == fx.ATT_ALIAS)
    bound = oracle.attention_bound(v, 16, 16)[None, :]
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - want) <= bound), np.max(np.abs(got - want) - bound)
    exact = fx.attention_exact_mask(exact_uniform, midpoint, exact_large, causal, identity_v)
    assert np.array_equal(got[exact].astype(np.float64), want[exact])


def test_causal_last_row_matches_unmasked():
    """tests/attention_correctness.cu:293-309: row 15 sees every key either way."""
    q, k, v = fx.attention_inputs(fx.ATT_SHIFTED_IDENTITY)
    full = run_tile(q, k, v, False)
    causal = run_tile(q, k, v, True)
    bound = 512 * 2.0 ** -23 + 2.0 ** -11 + (32 * 2.0 ** -23) / (1 - 32 * 2.0 ** -23)
    assert np.all(np.abs(full[15] - causal[15]) <= bound)


def test_error_state_contract():
    rt = cudart()
    q = torch.zeros(256, dtype=torch.float16, device="cuda")
    out = torch.full((256,), 9.0, device="cuda")
    torch.cuda.synchronize()
    code = seed_stale_error()
    assert tk_b200.attention_16x16_raw(q, None, q, out) == tk_b200.CUDA_ERROR_INVALID_VALUE
    assert rt.cudaPeekAtLastError() == code
    assert rt.cudaGetLastError() == code and rt.cudaPeekAtLastError() == 0
    seed_stale_error()
    assert tk_b200.attention_16x16_raw(q, q, q, out) == 0
    assert rt.cudaPeekAtLastError() == 0
    torch.cuda.synchronize()
    assert torch.all(out == 0.0)


def general_case(b, h, s, d, causal, seed, rows=None, pairs=None, misaligned=False, alias=False):
    count = b * h * s * d
    q, k, v = oracle.gen_qkv_normal(seed, 1.0, count)
    if alias:
        k, v = q, q
    scale = 1.0 / math.sqrt(d)
    keep = []
    if misaligned:
        buf = dev(np.concatenate([[0], q, k, v]).astype(np.uint16))
        keep.append(buf)
        qp = buf.data_ptr() + 2
        kp, vp = qp + 2 * count, qp + 4 * count
    else:
        tq, tk_, tv = dev(q), dev(k), dev(v)
        keep += [tq, tk_, tv]
        qp, kp, vp = tq.data_ptr(), tk_.data_ptr(), tv.data_ptr()
        if alias:
            kp = vp = qp
    out = torch.full((count,), float("nan"), device="cuda")
    assert tk_b200.attention_raw(qp, kp, vp, out, b, h, s, d, scale, causal) == 0
    got = host(out).reshape(b * h, s, d)
    qs, ks, vs = (x.reshape(b * h, s, d) for x in (q, k, v))
    for bh in (range(b * h) if pairs is None else pairs):
        bound = oracle.attention_bound(vs[bh], s, d)
        spans = [(0, s)] if rows is None else [(int(r), int(r) + 1) for r in rows]
        for lo, hi in spans:
            want = oracle.attention_ref(qs[bh], ks[bh], vs[bh], s, d, scale, causal, lo, hi)
            err = np.abs(got[bh, lo:hi] - want)
            assert np.all(err <= bound[None, :]), (bh, lo, float(np.max(err - bound[None, :])))


@pytest.mark.parametrize("shape", [
    (1, 2, 16, 16), (2, 3, 7, 16), (1, 1, 1, 16), (1, 1, 17, 16), (1, 1, 100, 64), (2, 3, 128, 128),
    (1, 2, 300, 64), (1, 2, 257, 32), (1, 1, 1000, 128), (1, 1, 129, 128), (2, 1, 640, 16)],
    ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("causal", [False, True])
def test_general_shapes(shape, causal):
    b, h, s, d = shape
    general_case(b, h, s, d, causal, seed=sum(shape))


def test_general_aliased_and_misaligned(attn_kernel):
    general_case(1, 2, 200, 64, True, seed=5, alias=True)
    general_case(1, 1, 200, 128, False, seed=6, misaligned=True)


@pytest.mark.parametrize("causal", [False, True])
def test_large_8x32x4096x128_sampled(causal, attn_kernel):
    """The large configuration (seed 4, N(0, 1), scale 1/sqrt(128)); 4 (b, h) pairs x
    sampled query rows including the first and last."""
    rng = np.random.default_rng(1)
    rows = np.unique(np.concatenate([[0, 4095], rng.integers(0, 4096, 30)]))
    general_case(8, 32, 4096, 128, causal, seed=4, rows=rows, pairs=[0, 77, 180, 255])


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("heads_q,heads_kv,s,d", [(8, 2, 300, 64), (4, 1, 300, 64), (6, 3, 300, 64),
                                                  (4, 2, 16, 16), (6, 2, 9, 16)])
def test_grouped_query_attention(heads_q, heads_kv, s, d, causal):
    """Query head h attends with key/value head h / (heads_q / heads_kv)."""
    b = 2
    group = heads_q // heads_kv
    q, _, _ = oracle.gen_qkv_normal(40 + heads_q, 1.0, b * heads_q * s * d)
    _, k, v = oracle.gen_qkv_normal(50 + heads_kv, 1.0, b * heads_kv * s * d)
    out = torch.full((b * heads_q * s * d,), float("nan"), device="cuda")
    tq, tk_, tv = dev(q), dev(k), dev(v)
    scale = 1.0 / math.sqrt(d)
    assert tk_b200.attention_gqa_raw(tq, tk_, tv, out, b, heads_q, heads_kv, s, d, scale, causal) == 0
    got = host(out).reshape(b * heads_q, s, d)
    qs = q.reshape(b * heads_q, s, d)
    ks, vs = k.reshape(b * heads_kv, s, d), v.reshape(b * heads_kv, s, d)
    for bh in range(b * heads_q):
        kv = (bh // heads_q) * heads_kv + (bh % heads_q) // group
        want = oracle.attention_ref(qs[bh], ks[kv], vs[kv], s, d, scale, causal)
        bound = oracle.attention_bound(vs[kv], s, d)
        assert np.all(np.abs(got[bh] - want) <= bound[None, :]), bh


@pytest.mark.parametrize("causal", [False, True])
def test_more_items_than_sms_every_head(causal):
    """300 (batch, head) items of one query-tile pair each: more work items than SMs,
    so the persistent CTAs take items from the shared counter and run several items
    each; every output row of every head is checked."""
    general_case(1, 300, 256, 64, causal, seed=7)



@pytest.mark.parametrize("shape", [(1, 1, 1, 128), (2, 3, 128, 128), (1, 2, 129, 128), (1, 1, 300, 128),
                                   (2, 1, 1000, 128), (1, 2, 517, 128)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("causal", [False, True])
def test_head128_shapes(shape, causal, attn_kernel):
    """head_dim 128 on single-block, tail and multi-block shapes."""
    b, h, s, d = shape
    general_case(b, h, s, d, causal, seed=11 + sum(shape))


@pytest.mark.parametrize("causal", [False, True])
def test_head128_many_items_gqa_and_misaligned(causal, attn_kernel):
    """More items than SMs (dynamic scheduling), grouped-query heads and misaligned
    operands at head_dim 128."""
    general_case(1, 160, 512, 128, causal, seed=21)
    general_case(1, 1, 200, 128, causal, seed=22, misaligned=True)
    b, heads_q, heads_kv, s, d = 2, 6, 2, 257, 128
    group = heads_q // heads_kv
    q, _, _ = oracle.gen_qkv_normal(61, 1.0, b * heads_q * s * d)
    _, k, v = oracle.gen_qkv_normal(62, 1.0, b * heads_kv * s * d)
    out = torch.full((b * heads_q * s * d,), float("nan"), device="cuda")
    tq, tk_, tv = dev(q), dev(k), dev(v)
    assert tk_b200.attention_gqa_raw(tq, tk_, tv, out, b, heads_q, heads_kv, s, d, 1 / math.sqrt(d), causal) == 0
    got = host(out).reshape(b * heads_q, s, d)
    qs = q.reshape(b * heads_q, s, d)
    ks, vs = k.reshape(b * heads_kv, s, d), v.reshape(b * heads_kv, s, d)
    for bh in range(b * heads_q):
        kv = (bh // heads_q) * heads_kv + (bh % heads_q) // group
        want = oracle.attention_ref(qs[bh], ks[kv], vs[kv], s, d, 1 / math.sqrt(d), causal)
        bound = oracle.attention_bound(vs[kv], s, d)
        assert np.all(np.abs(got[bh] - want) <= bound[None, :]), bh


@pytest.mark.parametrize("scale", [-0.3, 0.0])
def test_non_positive_scale(scale, attn_kernel):
    """A negative or zero scale (scores are scaled before the max; masked keys stay -inf)."""
    b, h, s, d = 1, 2, 300, 128
    q, k, v = oracle.gen_qkv_normal(31, 1.0, b * h * s * d)
    out = torch.full((b * h * s * d,), float("nan"), device="cuda")
    tq, tk_, tv = dev(q), dev(k), dev(v)
    for causal in (False, True):
        assert tk_b200.attention_raw(tq, tk_, tv, out, b, h, s, d, scale, causal) == 0
        got = host(out).reshape(b * h, s, d)
        for bh in range(b * h):
            sl = slice(bh * s * d, (bh + 1) * s * d)
            want = oracle.attention_ref(q[sl], k[sl], v[sl], s, d, scale, causal)
            bound = oracle.attention_bound(v[sl], s, d)
            assert np.all(np.abs(got[bh] - want) <= bound[None, :]), (causal, bh)


@pytest.mark.parametrize("causal", [False, True])
def test_cta_pair_kernel_matches_single_cta(causal):
    """The two head_dim 128 kernels on the same inputs: both inside the bound (checked
    above); here they also agree with each other to within the same bound, over every
    row of a multi-item problem with a ragged tail (S = 1300)."""
    b, h, s, d = 1, 6, 1300, 128
    q, k, v = oracle.gen_qkv_normal(77, 1.0, b * h * s * d)
    tq, tk_, tv = dev(q), dev(k), dev(v)
    lib = tk_b200.lib()
    outs = []
    old = lib.tk_attention_set_cta_group(1)
    try:
        for kernel in (1, 2):
            lib.tk_attention_set_cta_group(kernel)
            out = torch.full((b * h * s * d,), float("nan"), device="cuda")
            assert tk_b200.attention_raw(tq, tk_, tv, out, b, h, s, d, 1 / math.sqrt(d), causal) == 0
            outs.append(host(out).reshape(b * h, s, d))
    finally:
        lib.tk_attention_set_cta_group(old)
    for bh in range(b * h):
        bound = oracle.attention_bound(v.reshape(b * h, s, d)[bh], s, d)
        assert np.all(np.abs(outs[0][bh] - outs[1][bh]) <= 2 * bound[None, :]), bh
    assert tk_b200.device_status() == 0
