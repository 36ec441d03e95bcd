"""GEMM parity on the GPU through the C ABI, against the CPU oracle.

Follows the reference's tests/gemm_test.cu case for case at its tolerances for FP32
(term-scaled 1e-6: the FP32-faithful 3xTF32 tensor-core path and the FFMA path must both
hold it), then the TF32 and BF16 modes at their own bounds, tile and pipeline edges, and
the single-GEMM benchmark case against the golden vectors from the reference's code.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from cuvit import kernels
from cuvit.kernels import GemmProblem, gemm_problem
from helpers import (assert_close, assert_close_scaled, bf16_round, to_device, to_host,
                     worst_scaled)

pytestmark = pytest.mark.gpu

T, N_LAYOUT = kernels.LAYOUT_TRANSPOSED, kernels.LAYOUT_NO_TRANSPOSE

# Term-scaled tolerances (relative to sum_k |a_k b_k|):
FP32_RTOL = 1.0e-6  # the reference's own (tests/gemm_test.cu:83-87)
TF32_RTOL = 4.0e-3  # two 10-bit-mantissa roundings per product: <= 2 * 2^-10 + accumulation
BF16_RTOL = 1.0e-5  # operands exact in bf16 on both sides; accumulation order only


def run(a, b, bias, c0, problem: GemmProblem, math, torch, c_dtype=kernels.DTYPE_F32):
    in_dtype = torch.bfloat16 if math == kernels.MATH_BF16 else torch.float32
    out_dtype = torch.bfloat16 if c_dtype == kernels.DTYPE_BF16 else torch.float32
    da = to_device(a, in_dtype)
    db = to_device(b, in_dtype)
    dbias = None if bias is None else to_device(bias)
    dc = to_device(c0, out_dtype)
    kernels.launch_gemm_ex(da, db, dbias, dc, problem, c_dtype=c_dtype, math=math)
    torch.cuda.synchronize()
    return to_host(dc)


def check_case(m, n, k, layout, with_bias, alpha, math, torch, seed=None, rtol=None):
    rng = np.random.default_rng(seed if seed is not None else m * 31 + n * 7 + k)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    if math == kernels.MATH_BF16:
        a, b = bf16_round(a), bf16_round(b)
    transposed = layout == T
    want = oracle.gemm(a, b, bias if with_bias else None, np.zeros(m * n, np.float32), m, n, k,
                       transposed, alpha=alpha)
    scale = oracle.gemm_term_magnitudes(a, b, m, n, k, transposed, alpha)
    problem = gemm_problem(m, n, k, layout)
    problem.alpha = alpha
    got = run(a, b, bias if with_bias else None, np.full(m * n, np.nan, np.float32), problem,
              math, torch)
    tol = rtol if rtol is not None else {kernels.MATH_FP32: FP32_RTOL,
                                         kernels.MATH_TF32: TF32_RTOL,
                                         kernels.MATH_BF16: BF16_RTOL}[math]
    assert_close_scaled(got, want, scale, tol, 1e-6, f"{m}x{n}x{k} layout {layout} math {math}")
    return worst_scaled(got, want, scale)


# Every shape of tests/gemm_test.cu:93-106 plus tile edges of this kernel (128-row tiles,
# 64/128/256-column tiles, 32/64-element K stages).
SHAPES = [(1, 1, 1), (1, 1000, 192), (17, 33, 7), (63, 63, 63), (64, 64, 64), (65, 65, 65),
          (197, 576, 192), (197, 192, 192), (197, 768, 192), (197, 192, 768), (197, 197, 64),
          (197, 64, 197), (127, 129, 33), (128, 256, 64), (129, 257, 65), (256, 128, 128)]


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32, kernels.MATH_BF16],
                         ids=["fp32", "tf32", "bf16"])
@pytest.mark.parametrize("layout", [N_LAYOUT, T], ids=["kN", "kT"])
def test_shapes_and_layouts(math, layout, cuda):
    for m, n, k in SHAPES:
        for with_bias in (False, True):
            check_case(m, n, k, layout, with_bias, 1.0, math, cuda)


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32, kernels.MATH_BF16],
                         ids=["fp32", "tf32", "bf16"])
def test_alpha_scales_the_product(math, cuda):
    check_case(197, 197, 64, T, False, 0.125, math, cuda)
    check_case(32, 48, 16, N_LAYOUT, True, -2.5, math, cuda)


def test_fp32_mode_is_the_default_and_uses_reference_tolerance(cuda):
    assert kernels.get_math_mode() == kernels.MATH_FP32
    rng = np.random.default_rng(1)
    m, n, k = 197, 576, 192
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    da, db, dc = to_device(a), to_device(b), to_device(np.zeros(m * n))
    kernels.launch_gemm(da, db, None, dc, gemm_problem(m, n, k, T))
    cuda.cuda.synchronize()
    want = oracle.gemm(a, b, None, np.zeros(m * n, np.float32), m, n, k, True)
    scale = oracle.gemm_term_magnitudes(a, b, m, n, k, True)
    assert_close_scaled(to_host(dc), want, scale, FP32_RTOL, 1e-6, "default FP32 launch_gemm")


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32, kernels.MATH_BF16],
                         ids=["fp32", "tf32", "bf16"])
def test_attention_layout_split_batch(math, cuda):
    """Q.K^T and P.V exactly as src/model/vit.cu:205-242 issues them: column slices of the
    packed [T, 3E] projection reached through lda = 3E and an (image, head) split batch."""
    images, heads, tokens, d = 2, 3, 197, 64
    e = heads * d
    rng = np.random.default_rng(7)
    qkv = rng.standard_normal(images * tokens * 3 * e).astype(np.float32)
    if math == kernels.MATH_BF16:
        qkv = bf16_round(qkv)
    per_image = tokens * 3 * e
    logits = GemmProblem(m=tokens, n=tokens, k=d, layout=T, alpha=0.125, lda=3 * e, ldb=3 * e,
                         ldc=tokens)
    logits.batch = kernels.GemmBatch(count=images * heads, stride_a=d, stride_b=d,
                                     stride_c=tokens * tokens, inner=heads,
                                     outer_stride_a=per_image, outer_stride_b=per_image,
                                     outer_stride_c=heads * tokens * tokens)
    in_dtype = cuda.bfloat16 if math == kernels.MATH_BF16 else cuda.float32
    dq = to_device(qkv, in_dtype)
    element = dq.element_size()
    dout = to_device(np.zeros(images * heads * tokens * tokens, np.float32))
    kernels.launch_gemm_ex(dq.data_ptr(), dq.data_ptr() + e * element, None, dout, logits,
                           math=math)
    cuda.cuda.synchronize()
    got = to_host(dout)
    want = oracle.gemm(qkv, qkv[e:], None, np.zeros(images * heads * tokens * tokens),
                       tokens, tokens, d, True, alpha=0.125, lda=3 * e, ldb=3 * e, ldc=tokens,
                       count=images * heads, inner=heads, stride_a=d, stride_b=d,
                       stride_c=tokens * tokens, outer_a=per_image, outer_b=per_image,
                       outer_c=heads * tokens * tokens)
    tol = {kernels.MATH_FP32: FP32_RTOL, kernels.MATH_TF32: TF32_RTOL,
           kernels.MATH_BF16: BF16_RTOL}[math]
    # Term magnitudes for every (image, head) slice.
    q = np.abs(qkv.reshape(images, tokens, 3, heads, d))
    scale = 0.125 * np.einsum("bqhd,bkhd->bhqk", q[:, :, 0], q[:, :, 1]).reshape(-1)
    assert_close_scaled(got, want, scale, tol, 1e-6, "split-batch attention logits")


def test_zero_stride_shares_an_operand(cuda):
    batch, m, n, k = 4, 40, 24, 32
    rng = np.random.default_rng(77)
    a = rng.standard_normal(batch * m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    problem = gemm_problem(m, n, k, N_LAYOUT)
    problem.batch = kernels.GemmBatch(count=batch, stride_a=m * k, stride_b=0, stride_c=m * n)
    got = run(a, b, None, np.zeros(batch * m * n), problem, kernels.MATH_FP32, cuda)
    for i in range(batch):
        slice_a = a[i * m * k:(i + 1) * m * k]
        want = oracle.gemm(slice_a, b, None, np.zeros(m * n), m, n, k, False)
        scale = oracle.gemm_term_magnitudes(slice_a, b, m, n, k, False)
        assert_close_scaled(got[i * m * n:(i + 1) * m * n], want, scale, FP32_RTOL, 1e-6,
                            "shared weight across a batch")


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_BF16], ids=["fp32", "bf16"])
def test_accumulate_epilogue_adds_into_the_destination(math, cuda):
    m, n, k = 70, 40, 24
    rng = np.random.default_rng(404)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    existing = rng.standard_normal(m * n).astype(np.float32)
    if math == kernels.MATH_BF16:
        a, b = bf16_round(a), bf16_round(b)
    product = oracle.gemm(a, b, bias, np.zeros(m * n), m, n, k, False)
    scale = oracle.gemm_term_magnitudes(a, b, m, n, k, False)
    tol = FP32_RTOL if math == kernels.MATH_FP32 else BF16_RTOL
    problem = gemm_problem(m, n, k, N_LAYOUT)
    problem.epilogue.accumulate = True
    got = run(a, b, bias, existing, problem, math, cuda)
    assert_close_scaled(got, existing + product, scale, tol, 1e-5, "accumulate epilogue")
    got = run(a, b, bias, existing, gemm_problem(m, n, k, N_LAYOUT), math, cuda)
    assert_close_scaled(got, product, scale, tol, 1e-5, "default epilogue overwrites")


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32], ids=["fp32", "tf32"])
def test_gelu_epilogue_and_bias_order(math, cuda):
    m, n, k = 33, 96, 48
    rng = np.random.default_rng(505)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    want = oracle.gemm(a, b, bias, np.zeros(m * n), m, n, k, False, gelu=True)
    problem = gemm_problem(m, n, k, N_LAYOUT)
    problem.epilogue.gelu = True
    got = run(a, b, bias, np.zeros(m * n), problem, math, cuda)
    if math == kernels.MATH_FP32:
        assert_close(got, want, 1e-4, 1e-5, "GELU epilogue")  # tests/gemm_test.cu:310-311
    else:
        assert_close(got, want, 1e-2, 2e-2, "GELU epilogue (TF32)")
    wrong = oracle.gelu(oracle.gemm(a, b, None, np.zeros(m * n), m, n, k, False))
    wrong = wrong + np.tile(bias, m)
    diff = np.abs(got - wrong) > 1e-3 + 1e-3 * np.abs(wrong)
    assert diff.any(), "the GELU epilogue applied the bias in the wrong order"


def test_gelu_epilogue_with_bf16_output(cuda):
    """FC1's form: bf16 operands, bias + GELU, bf16 output (the epilogue evaluates erf with
    Abramowitz-Stegun 7.1.26 here): within bf16 rounding of the erf-form oracle."""
    m, n, k = 200, 768, 192
    rng = np.random.default_rng(606)
    a = bf16_round(rng.standard_normal(m * k))
    b = bf16_round(0.2 * rng.standard_normal(n * k))
    bias = rng.standard_normal(n).astype(np.float32)
    want = oracle.gemm(a, b, bias, np.zeros(m * n), m, n, k, True, gelu=True)
    problem = gemm_problem(m, n, k, T)
    problem.epilogue.gelu = True
    got = run(a, b, bias, np.zeros(m * n), problem, kernels.MATH_BF16, cuda,
              c_dtype=kernels.DTYPE_BF16)
    assert_close(got, want, 2 ** -8, 1e-3, "bf16 GELU epilogue")
    # the approximation itself, away from bf16 rounding: FP32-output path vs bf16-output
    # path differ only by the final rounding
    got32 = run(a, b, bias, np.zeros(m * n), problem, kernels.MATH_BF16, cuda)
    np.testing.assert_allclose(got, bf16_round(got32), rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("layout", [N_LAYOUT, T], ids=["kN", "kT"])
def test_fp32_split_handles_huge_and_non_finite_operands(layout, cuda):
    """The 3xTF32 splitter rounds with integer adds, exact below 2^127; operands at or above
    it and infinities / NaNs take its checked rounding. Huge finite operands stay within the
    reference tolerance; a row with an infinity or a NaN gives non-finite results exactly
    where the FP32 oracle does, and every other output is unaffected."""
    m, n, k = 160, 136, 96
    rng = np.random.default_rng(29)
    a = rng.uniform(-1, 1, m * k).astype(np.float32)
    b = (1e-3 * rng.uniform(-1, 1, k * n)).astype(np.float32)
    a[5 * k + 3] = 3.0e38         # exponent 254
    a[7 * k + 90] = -2.9e38
    a[9 * k + 11] = 1.7014e38     # exactly 2^127-ish
    a[20 * k + 4] = np.inf
    a[30 * k + 40] = np.nan
    transposed = layout == T
    want = oracle.gemm(a, b, None, np.zeros(m * n, np.float32), m, n, k, transposed)
    got = run(a, b, None, np.full(m * n, np.nan, np.float32), gemm_problem(m, n, k, layout),
              kernels.MATH_FP32, cuda)
    np.testing.assert_array_equal(np.isfinite(got), np.isfinite(want))
    finite = np.isfinite(want)
    with np.errstate(invalid="ignore", over="ignore"):
        scale = oracle.gemm_term_magnitudes(np.nan_to_num(a, posinf=0.0), b, m, n, k, transposed)
    assert_close_scaled(got[finite], want[finite], scale[finite], FP32_RTOL, 1e-6,
                        f"huge operands layout {layout}")


def test_zero_k_produces_the_bias_exactly(cuda):
    m, n = 8, 8
    bias = np.random.default_rng(5).standard_normal(n).astype(np.float32)
    for math in (kernels.MATH_FP32, kernels.MATH_TF32, kernels.MATH_BF16):
        got = run(np.zeros(1), np.zeros(1), bias, np.full(m * n, np.nan), gemm_problem(m, n, 0, 0),
                  math, cuda)
        np.testing.assert_array_equal(got.reshape(m, n), np.tile(bias, (m, 1)))


def test_unaligned_leading_dimension_takes_the_general_path(cuda):
    """lda = ldc = 197 floats (788 bytes) cannot be a TMA stride; results must still hold the
    FP32 tolerance (the reference's .V GEMM reads its logits this way, vit.cu:229-242)."""
    m, n, k = 50, 64, 197
    rng = np.random.default_rng(12)
    a_full = rng.standard_normal(m * 197).astype(np.float32)
    b = rng.standard_normal(k * n).astype(np.float32)
    problem = GemmProblem(m=m, n=n, k=k, layout=N_LAYOUT, lda=197, ldc=197)
    got = run(a_full, b, None, np.zeros(m * 197), problem, kernels.MATH_FP32, cuda)
    got = got.reshape(m, 197)[:, :n]
    want = oracle.gemm(a_full, b, None, np.zeros(m * n), m, n, k, False, lda=197)
    a = a_full.reshape(m, 197)[:, :k].copy()
    scale = oracle.gemm_term_magnitudes(a, b, m, n, k, False)
    assert_close_scaled(got, want, scale, FP32_RTOL, 1e-6, "unaligned lda")


@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32, kernels.MATH_BF16],
                         ids=["fp32", "tf32", "bf16"])
def test_persistent_tiles_and_pipeline_wraparound(math, cuda):
    """More output tiles than SMs and more K stages than the smem ring holds: every CTA walks
    several tiles and every stage barrier goes through several phases. Rows sampled."""
    m, n, k = 4100, 1024, 640
    rng = np.random.default_rng(99)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(n * k).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    if math == kernels.MATH_BF16:
        a, b = bf16_round(a), bf16_round(b)
    got = run(a, b, bias, np.zeros(m * n), gemm_problem(m, n, k, T), math, cuda).reshape(m, n)
    rows = np.array([0, 1, 127, 128, 129, 2047, 2048, 4095, 4096, 4099])
    a_rows = a.reshape(m, k)[rows]
    want = oracle.gemm(a_rows, b, bias, np.zeros(rows.size * n), rows.size, n, k, True)
    scale = oracle.gemm_term_magnitudes(a_rows, b, rows.size, n, k, True)
    tol = {kernels.MATH_FP32: FP32_RTOL, kernels.MATH_TF32: TF32_RTOL,
           kernels.MATH_BF16: BF16_RTOL}[math]
    assert_close_scaled(got[rows], want, scale, tol, 1e-6, "persistent GEMM sampled rows")


def test_bf16_output_and_bf16_accumulate(cuda):
    m, n, k = 300, 384, 256
    rng = np.random.default_rng(8)
    a = bf16_round(rng.standard_normal(m * k))
    b = bf16_round(rng.standard_normal(n * k))
    existing = bf16_round(rng.standard_normal(m * n))
    product = oracle.gemm(a, b, None, np.zeros(m * n), m, n, k, True)
    got = run(a, b, None, np.zeros(m * n), gemm_problem(m, n, k, T), kernels.MATH_BF16, cuda,
              c_dtype=kernels.DTYPE_BF16)
    np.testing.assert_array_equal(got, bf16_round(got))
    assert_close(got, product, 2 ** -8, 1e-3, "bf16 output")
    problem = gemm_problem(m, n, k, T)
    problem.epilogue.accumulate = True
    got = run(a, b, None, existing, problem, kernels.MATH_BF16, cuda, c_dtype=kernels.DTYPE_BF16)
    assert_close(got, existing + product, 2 ** -7, 1e-2, "bf16 accumulate")


@pytest.mark.parametrize("math,c_dtype,n,ldc,accumulate", [
    (kernels.MATH_BF16, kernels.DTYPE_F32, 384, 400, False),    # TMA store, padded rows
    (kernels.MATH_BF16, kernels.DTYPE_F32, 384, 387, True),     # ldc not 16-byte: direct
    (kernels.MATH_BF16, kernels.DTYPE_BF16, 192, 192, False),   # 64-wide tiles: direct
    (kernels.MATH_BF16, kernels.DTYPE_BF16, 512, 520, False),   # TMA store of bf16
    (kernels.MATH_TF32, kernels.DTYPE_TF32, 320, 320, False),   # TF32-rounded storage
    (kernels.MATH_TF32, kernels.DTYPE_TF32, 320, 320, True),    # rounded after the add
    (kernels.MATH_FP32, kernels.DTYPE_F32, 96, 100, True),      # reduce-add, 3xTF32
])
def test_output_paths(math, c_dtype, n, ldc, accumulate, cuda):
    """Every way the epilogue writes C: TMA store, TMA reduce-add, direct stores; FP32,
    BF16 and TF32-rounded storage; padded rows left untouched."""
    m, k = 300, 256
    rng = np.random.default_rng(n + ldc)
    a = rng.standard_normal(m * k).astype(np.float32)
    b = rng.standard_normal(n * k).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    if math == kernels.MATH_BF16:
        a, b = bf16_round(a), bf16_round(b)
    existing = rng.standard_normal(m * ldc).astype(np.float32)
    if c_dtype == kernels.DTYPE_BF16:
        existing = bf16_round(existing)
    problem = GemmProblem(m=m, n=n, k=k, layout=T, ldc=ldc)
    problem.epilogue.accumulate = accumulate
    out_dtype = {kernels.DTYPE_F32: cuda.float32, kernels.DTYPE_TF32: cuda.float32,
                 kernels.DTYPE_BF16: cuda.bfloat16}[c_dtype]
    in_dtype = cuda.bfloat16 if math == kernels.MATH_BF16 else cuda.float32
    dc = to_device(existing, out_dtype)
    kernels.launch_gemm_ex(to_device(a, in_dtype), to_device(b, in_dtype), to_device(bias), dc,
                           problem, c_dtype=c_dtype, math=math)
    cuda.cuda.synchronize()
    got = to_host(dc).reshape(m, ldc)
    product = oracle.gemm(a, b, bias, np.zeros(m * n), m, n, k, True).reshape(m, n)
    want = product + existing.reshape(m, ldc)[:, :n] if accumulate else product
    np.testing.assert_array_equal(got[:, n:], existing.reshape(m, ldc)[:, n:])
    if c_dtype == kernels.DTYPE_TF32:
        bits = got[:, :n].view(np.uint32)
        assert not (bits & 0x1FFF).any(), "TF32 storage holds more than 10 mantissa bits"
    tol = {kernels.MATH_FP32: 1e-5, kernels.MATH_TF32: 4e-3, kernels.MATH_BF16: 1e-5}[math]
    if c_dtype == kernels.DTYPE_BF16:
        assert_close(got[:, :n], want, 2 ** -7, 1e-2, "bf16 output")
    else:
        scale = oracle.gemm_term_magnitudes(a, b, m, n, k, True).reshape(m, n)
        assert_close_scaled(got[:, :n], want, scale, tol, 1e-5, "output path")


@pytest.mark.parametrize("label", ["config1 qkv", "config1 gelu", "config1 accumulate"])
@pytest.mark.parametrize("math", [kernels.MATH_FP32, kernels.MATH_TF32], ids=["fp32", "tf32"])
def test_baseline_config1_against_reference_golden(label, math, golden, cuda):
    """The single-GEMM benchmark case (ViT-Tiny QKV shape, U(-1,1) seed 0; GELU N=768;
    accumulate K=768) against the outputs of the reference's own CPU code."""
    import make_golden as mg

    case = next(c for c in mg.GEMM_CASES if c[0] == label)
    _, m, n, k, transposed, alpha, with_bias, epilogue, dist, seed = case
    a, b, bias, existing = mg.gemm_inputs(m, n, k, seed, dist)
    problem = gemm_problem(m, n, k, T)
    problem.epilogue.gelu = epilogue == "gelu"
    problem.epilogue.accumulate = epilogue == "accumulate"
    got = run(a, b, bias, existing if epilogue == "accumulate" else np.zeros(m * n), problem,
              math, cuda).reshape(m, n)
    key = f"gemm/{label}"
    rows = golden[key + "/rows"]
    rtol = FP32_RTOL if math == kernels.MATH_FP32 else TF32_RTOL
    if epilogue == "gelu":
        # GELU's slope is at most ~1.13, so the pre-activation bound carries over.
        rtol *= 1.2
    assert_close_scaled(got[rows], golden[key + "/c"], golden[key + "/scale"], rtol, 1e-6, label)


def test_device_timeout_is_reported_and_the_context_survives(cuda):
    """A kernel whose wait can never complete gives up after 1 ms, flags the status word and
    returns; the host sees CUVIT_DEVICE_TIMEOUT and the next launch works."""
    from cuvit import _lib
    from cuvit.errors import DeviceTimeout, check

    check(_lib.library().cuvit_selftest_bounded_wait(1_000_000))
    with pytest.raises(DeviceTimeout):
        kernels.device_status()
    assert kernels.device_status() == 0
    check_case(64, 64, 64, T, True, 1.0, kernels.MATH_BF16, cuda)


# Large BF16 GEMMs with the weights' [N, K] layout and no GELU run on the CTA-pair kernel
# (256-row tiles over two SMs) once there are at least as many 256-row tiles as SMs; these
# shapes all get there. Reference: the same bfloat16 operands multiplied in FP32 by PyTorch
# (TF32 off).
PAIR_CASES = [
    # m, n, k, count, c_dtype, gelu, accumulate, with_bias
    (4261, 2304, 768, 1, kernels.DTYPE_F32, False, False, True),     # ragged last tile
    (4261, 2304, 768, 1, kernels.DTYPE_BF16, False, False, True),    # bf16 output
    (50432, 768, 768, 1, kernels.DTYPE_F32, False, True, True),      # residual reduce-add
    (2048, 2560, 64, 2, kernels.DTYPE_F32, False, False, False),     # one k-block, batched
    (4096, 2560, 8000, 1, kernels.DTYPE_F32, False, False, True),    # long K, ragged k-block
]


@pytest.mark.parametrize("m,n,k,count,c_dtype,gelu,accumulate,with_bias", PAIR_CASES,
                         ids=[f"{c[0]}x{c[1]}x{c[2]}x{c[3]}" + ("-gelu" if c[5] else "") +
                              ("-acc" if c[6] else "") for c in PAIR_CASES])
def test_cta_pair_gemm_against_torch_fp32(m, n, k, count, c_dtype, gelu, accumulate, with_bias,
                                          cuda):
    torch = cuda
    assert not torch.backends.cuda.matmul.allow_tf32
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(count, m, k, device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn(count, n, k, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g) if with_bias else None
    c0 = torch.randn(count, m, n, device="cuda", generator=g)
    out_dtype = torch.bfloat16 if c_dtype == kernels.DTYPE_BF16 else torch.float32
    c = c0.to(out_dtype, copy=True) if accumulate else torch.full(
        (count, m, n), float("nan"), device="cuda", dtype=out_dtype)
    problem = gemm_problem(m, n, k, T)
    problem.batch.count = count
    problem.batch.stride_a = m * k
    problem.batch.stride_b = n * k
    problem.batch.stride_c = m * n
    problem.epilogue.gelu = gelu
    problem.epilogue.accumulate = accumulate
    kernels.launch_gemm_ex(a, b, bias, c, problem, c_dtype=c_dtype, math=kernels.MATH_BF16)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0

    af, bf = a.float(), b.float()
    want = torch.bmm(af, bf.transpose(1, 2))
    scale = torch.bmm(af.abs(), bf.abs().transpose(1, 2))
    if bias is not None:
        want = want + bias
    if gelu:
        want = torch.nn.functional.gelu(want)
    if accumulate:
        want = want + c0.to(out_dtype).float()
    got = c.float()
    assert torch.isfinite(got).all(), "rows or columns were left unwritten"
    if c_dtype == kernels.DTYPE_BF16:
        # one bf16 rounding of the result (2^-8 relative) on top of the accumulation
        tol = want.abs() * 2.0 ** -8 + scale * 1e-5 + 1e-6
    else:
        tol = scale * 1e-5 + 1e-6
    excess = ((got - want).abs() - tol).max().item()
    assert excess <= 0, f"error exceeds the bound by {excess:.3g}"
