"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/*.h declares, and rejects invalid arguments before touching CUDA
(the validation matrix of the reference's tests/gemm_correctness.cu:316-418 and
tests/attention_correctness.cu:226-244)."""

import ctypes as C
import os
import re
import subprocess

import pytest

import tk_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INVALID = tk_b200.CUDA_ERROR_INVALID_VALUE


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fname in os.listdir(inc):
        if fname.endswith(".h"):
            text = open(os.path.join(inc, fname)).read()
            names |= set(re.findall(r"^TK_API\s+[a-zA-Z_0-9]+\s+(tk_[a-z0-9_]+)\s*\(", text, re.M))
    return sorted(names)


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(tk_b200.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(tk_b200.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert tk_b200.lib().tk_abi_version() == 101


def test_library_exports_nothing_undeclared():
    out = subprocess.run(["nm", "-D", "--defined-only", tk_b200.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted(set(re.findall(r"\b(tk_[a-z0-9_]+)\b", out)))
    assert exported == declared_symbols()


FAKE = 0x10000  # never dereferenced: validation rejects before any CUDA call


def gemm_args(**over):
    args = dict(m=16, n=16, k=16, a=FAKE, lda=16, b=FAKE * 2, ldb=16, c=FAKE * 3, ldc=16)
    args.update(over)
    return args


@pytest.mark.parametrize("over", [
    dict(a=None), dict(b=None), dict(c=None),
    dict(m=0), dict(n=0), dict(k=0), dict(m=-16), dict(n=-16), dict(k=-16),
    dict(m=17), dict(n=17), dict(k=17), dict(lda=15), dict(ldb=15), dict(ldc=15),
], ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
def test_gemm_invalid_arguments(over):
    a = gemm_args(**over)
    code = tk_b200.lib().tk_gemm_f16_f16_f32_nn(a["m"], a["n"], a["k"], a["a"], a["lda"], a["b"], a["ldb"],
                                                 a["c"], a["ldc"], None)
    assert code == INVALID
    code = tk_b200.lib().tk_gemm_f16_f16_f32_nn_rowstats(a["m"], a["n"], a["k"], a["a"], a["lda"], a["b"],
                                                          a["ldb"], a["c"], a["ldc"], FAKE * 4, FAKE * 5, None)
    assert code == INVALID


@pytest.mark.parametrize("over", [
    dict(a=None), dict(b=None), dict(c=None), dict(m=0), dict(n=17), dict(k=-16), dict(lda=15),
    dict(ldb=15), dict(ldc=15),
], ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
def test_gemm_rowsoftmax_invalid_arguments(over):
    a = gemm_args(**over)
    code = tk_b200.lib().tk_gemm_f16_f16_f32_nn_rowsoftmax(a["m"], a["n"], a["k"], a["a"], a["lda"], a["b"],
                                                            a["ldb"], a["c"], a["ldc"], FAKE * 8, 16, None)
    assert code == INVALID


def test_gemm_rowsoftmax_output_rules():
    lib = tk_b200.lib()
    a = gemm_args(m=32)
    call = lambda probs, ldp, ldc=16: lib.tk_gemm_f16_f16_f32_nn_rowsoftmax(  # noqa: E731
        32, 16, 16, a["a"], 16, a["b"], 16, a["c"], ldc, probs, ldp, None)
    assert call(None, 16) == INVALID            # no output
    assert call(FAKE * 8, 15) == INVALID        # ldp < n
    assert call(a["c"] + 64, 16) == INVALID     # partial overlap of P and C
    assert call(a["c"], 32) == INVALID          # same base, different pitch
    assert call(a["c"] - 4 * 16 * 32 + 4, 16) == INVALID  # P's last row reaches C


def test_gemm_rowstats_needs_both_outputs():
    a = gemm_args()
    lib = tk_b200.lib()
    assert lib.tk_gemm_f16_f16_f32_nn_rowstats(16, 16, 16, a["a"], 16, a["b"], 16, a["c"], 16, None,
                                               FAKE * 5, None) == INVALID
    assert lib.tk_gemm_f16_f16_f32_nn_rowstats(16, 16, 16, a["a"], 16, a["b"], 16, a["c"], 16, FAKE * 4,
                                               FAKE * 4, None) == INVALID


@pytest.mark.parametrize("missing", range(4))
@pytest.mark.parametrize("causal", [False, True])
def test_attention_16x16_null_arguments(missing, causal):
    ptrs = [FAKE, FAKE * 2, FAKE * 3, FAKE * 4]
    ptrs[missing] = None
    lib = tk_b200.lib()
    fn = lib.tk_attention_forward_16x16_causal if causal else lib.tk_attention_forward_16x16
    assert fn(*ptrs, None) == INVALID


@pytest.mark.parametrize("over", [
    dict(batch=0), dict(heads=0), dict(seq=0), dict(head_dim=48), dict(head_dim=256),
    dict(causal=2), dict(scale=float("nan")), dict(scale=float("inf")), dict(q=None), dict(out=None),
], ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
def test_attention_invalid_arguments(over):
    a = dict(q=FAKE, k=FAKE, v=FAKE, out=1 << 40, batch=1, heads=1, seq=64, head_dim=64, scale=0.125,
             causal=0)
    a.update(over)
    assert tk_b200.lib().tk_attention_forward_f16(a["q"], a["k"], a["v"], a["out"], a["batch"], a["heads"],
                                                  a["seq"], a["head_dim"], a["scale"], a["causal"],
                                                  None) == INVALID


def test_attention_output_must_not_overlap_inputs():
    # out overlapping q (1 x 1 x 64 x 64 binary16 = 8 KiB) is rejected.
    assert tk_b200.lib().tk_attention_forward_f16(FAKE, FAKE * 4, FAKE * 4, FAKE + 4096, 1, 1, 64, 64,
                                                  0.125, 0, None) == INVALID


def test_rowops_invalid_arguments():
    lib = tk_b200.lib()
    assert lib.tk_tile_row_sum_f32(None, 4, FAKE, None) == INVALID
    assert lib.tk_tile_row_max_f32(FAKE, 4, None, None) == INVALID
    assert lib.tk_tile_row_ops_f32(FAKE, 4, None, None, None, None, None) == INVALID
    # misaligned (not 4-byte) pointers
    assert lib.tk_tile_row_sum_f32(FAKE + 2, 4, FAKE * 8, None) == INVALID
    assert lib.tk_tile_row_softmax_f32(FAKE, 4, FAKE * 8 + 1, None) == INVALID
    # partial overlap of output and input (in place is allowed only for softmax, exactly)
    assert lib.tk_tile_row_softmax_f32(FAKE, 4, FAKE + 256, None) == INVALID
    assert lib.tk_tile_row_sum_f32(FAKE, 4, FAKE, None) == INVALID
    # outputs overlapping each other in the fused call
    assert lib.tk_tile_row_ops_f32(FAKE, 4, FAKE * 8, FAKE * 8 + 32, None, None, None) == INVALID
    # size overflow
    assert lib.tk_tile_row_sum_f32(FAKE, (1 << 64) // 1024 + 1, FAKE * 8, None) == INVALID


def test_valid_call_without_gpu_reports_an_error_not_a_crash():
    """On a machine without a usable device a valid call returns a CUDA error."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    code = tk_b200.lib().tk_tile_row_sum_f32(FAKE, 4, FAKE * 8, None)
    assert code not in (0, INVALID)


def test_gqa_invalid_arguments():
    lib = tk_b200.lib()
    # heads_q not a multiple of heads_kv, and zero key/value heads
    assert lib.tk_attention_forward_gqa_f16(FAKE, FAKE, FAKE, 1 << 40, 1, 6, 4, 64, 64, 0.125, 0, None) == INVALID
    assert lib.tk_attention_forward_gqa_f16(FAKE, FAKE, FAKE, 1 << 40, 1, 6, 0, 64, 64, 0.125, 0, None) == INVALID
