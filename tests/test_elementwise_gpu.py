"""Memory-bound operators on the GPU against the oracle, following the reference's
tests/elementwise_test.cu (shapes, tolerances, landmark values) plus the patch gather
(bit-exact) and the broadcasts, which the reference only reaches through vit_test."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from cuvit import kernels
from cuvit.errors import InvalidArgument
from helpers import assert_close, bf16_round, to_device, to_host

pytestmark = pytest.mark.gpu


def test_gelu_matches_the_erf_form(cuda):
    rng = np.random.default_rng(31)
    x = (3.0 * rng.standard_normal(4099)).astype(np.float32)
    x[:13] = [-30.0, -8.0, -2.7, -2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0, 2.7, 8.0, 30.0]
    dx, dy = to_device(x), to_device(np.zeros_like(x))
    kernels.launch_gelu(dx, dy, x.size)
    assert_close(to_host(dy), oracle.gelu(x), 1e-5, 1e-6, "GELU")
    # unaligned views take the scalar path
    kernels.launch_gelu(dx[1:], dy[1:], x.size - 1)
    assert_close(to_host(dy)[1:], oracle.gelu(x[1:]), 1e-5, 1e-6, "GELU unaligned")


def test_residual_add_is_exact(cuda):
    rng = np.random.default_rng(9)
    acc = rng.standard_normal(1027).astype(np.float32)
    addend = rng.standard_normal(1027).astype(np.float32)
    dacc, dadd = to_device(acc), to_device(addend)
    kernels.launch_add(dacc, dadd, acc.size)
    np.testing.assert_array_equal(to_host(dacc), acc + addend)


@pytest.mark.parametrize("rows,columns", [(1, 192), (197, 192), (197, 768), (3, 1), (5, 31),
                                          (2, 1024), (7, 1536), (300, 384)])
def test_layer_norm(rows, columns, cuda):
    rng = np.random.default_rng(rows * 101 + columns)
    x = rng.standard_normal(rows * columns).astype(np.float32)
    gamma = (1.0 + 0.2 * rng.standard_normal(columns)).astype(np.float32)
    beta = (0.2 * rng.standard_normal(columns)).astype(np.float32)
    want = oracle.layer_norm(x, gamma, beta, rows, columns)
    dy = to_device(np.zeros_like(x))
    kernels.launch_layer_norm(to_device(x), to_device(gamma), to_device(beta), dy, rows, columns)
    assert_close(to_host(dy), want, 1e-5, 2e-6, f"layer norm {rows}x{columns}")


def test_layer_norm_tolerates_a_large_offset(cuda):
    rows, columns = 197, 192
    x = (np.random.default_rng(7).standard_normal(rows * columns) + 1000.0).astype(np.float32)
    gamma = np.ones(columns, np.float32)
    beta = np.zeros(columns, np.float32)
    want = oracle.layer_norm(x, gamma, beta, rows, columns)
    dy = to_device(np.zeros_like(x))
    kernels.launch_layer_norm(to_device(x), to_device(gamma), to_device(beta), dy, rows, columns)
    assert_close(to_host(dy), want, 1e-5, 5e-5, "layer norm at offset 1000")


def test_layer_norm_normalizes(cuda):
    rows, columns = 8, 192
    x = (5.0 + 3.0 * np.random.default_rng(3).standard_normal(rows * columns)).astype(np.float32)
    dy = to_device(np.zeros_like(x))
    kernels.launch_layer_norm(to_device(x), to_device(np.ones(columns)),
                              to_device(np.zeros(columns)), dy, rows, columns)
    y = to_host(dy).reshape(rows, columns).astype(np.float64)
    assert np.all(np.abs(y.mean(1)) < 1e-4)
    assert np.all(np.abs((y * y).mean(1) - 1.0) < 1e-3)


def test_layer_norm_strided_rows_and_bf16_output(cuda):
    """The runner's final norm: class-token rows only (row stride T*E), bf16 out."""
    images, tokens, e = 5, 197, 384
    rng = np.random.default_rng(17)
    x = rng.standard_normal(images * tokens * e).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(e)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(e)).astype(np.float32)
    want = oracle.layer_norm(x, gamma, beta, images, e, in_stride=tokens * e)
    out = cuda.zeros(images * e, dtype=cuda.bfloat16, device="cuda")
    kernels.launch_layer_norm_ex(to_device(x), tokens * e, to_device(gamma), to_device(beta),
                                 out, kernels.DTYPE_BF16, e, images, e)
    got = to_host(out)
    assert_close(got, want, 2 ** -8, 1e-5, "strided bf16 layer norm")
    out32 = to_device(np.zeros(images * e))
    kernels.launch_layer_norm_ex(to_device(x), tokens * e, to_device(gamma), to_device(beta),
                                 out32, kernels.DTYPE_F32, e, images, e)
    assert_close(to_host(out32), want, 1e-5, 2e-6, "strided fp32 layer norm")


@pytest.mark.parametrize("rows,columns", [(1, 2), (197, 197), (4, 1), (3, 1000), (8, 33),
                                          (2, 5000)])
def test_softmax(rows, columns, cuda):
    x = (4.0 * np.random.default_rng(rows * 17 + columns).standard_normal(rows * columns)
         ).astype(np.float32)
    want = oracle.softmax(x, rows, columns)
    dx = to_device(x)
    kernels.launch_softmax(dx, dx, rows, columns)  # in place, as the model calls it
    got = to_host(dx)
    assert_close(got, want, 1e-4, 1e-6, f"softmax {rows}x{columns}")
    sums = got.reshape(rows, columns).astype(np.float64).sum(1)
    assert np.all((got >= 0) & (got <= 1)) and np.all(np.abs(sums - 1) < 1e-4)


def test_softmax_survives_large_logits(cuda):
    rows, columns = 4, 64
    x = np.full((rows, columns), -500.0, np.float32)
    x[np.arange(rows), np.arange(rows)] = 500.0
    dx, dy = to_device(x), to_device(np.zeros_like(x))
    kernels.launch_softmax(dx, dy, rows, columns)
    y = to_host(dy).reshape(rows, columns)
    assert np.isfinite(y).all()
    np.testing.assert_allclose(y, np.eye(rows, columns), atol=1e-5)


def test_softmax_row_stride(cuda):
    rows, columns, stride = 6, 197, 200
    x = np.random.default_rng(4).standard_normal(rows * stride).astype(np.float32)
    dx = to_device(x)
    kernels.launch_softmax_ex(dx, dx, rows, columns, stride)
    got = to_host(dx).reshape(rows, stride)
    want = oracle.softmax(x.reshape(rows, stride)[:, :columns].copy(), rows, columns)
    assert_close(got[:, :columns], want, 1e-4, 1e-6, "strided softmax")
    np.testing.assert_array_equal(got[:, columns:], x.reshape(rows, stride)[:, columns:])


# The strip kernel's block shapes (row groups of 4, 2, 16 and 1, a patch of 4 rows capping
# them, and a width past its 1024-group limit, which takes the per-element kernel) and the
# unaligned fallbacks.
@pytest.mark.parametrize("batch,channels,size,patch", [(2, 3, 224, 16), (3, 3, 32, 8),
                                                       (1, 1, 12, 3), (4, 2, 10, 5),
                                                       (2, 3, 384, 16), (1, 3, 64, 32),
                                                       (2, 4, 48, 4), (1, 3, 1024, 16),
                                                       (1, 1, 4112, 16)])
def test_extract_patches_is_bit_exact(batch, channels, size, patch, cuda):
    images = np.random.default_rng(size).standard_normal(
        batch * channels * size * size).astype(np.float32)
    want = oracle.extract_patches(images, batch, channels, size, size, patch)
    out = to_device(np.zeros_like(want))
    kernels.launch_extract_patches(to_device(images), out, batch, channels, size, size, patch)
    np.testing.assert_array_equal(to_host(out), want)
    out16 = cuda.zeros(want.size, dtype=cuda.bfloat16, device="cuda")
    kernels.launch_extract_patches_ex(to_device(images), out16, kernels.DTYPE_BF16, batch,
                                      channels, size, size, patch)
    np.testing.assert_array_equal(to_host(out16), bf16_round(want))


def test_broadcasts_and_token_initialisation(cuda):
    rng = np.random.default_rng(21)
    batch, tokens, e = 3, 197, 192
    cls = rng.standard_normal(e).astype(np.float32)
    pos = rng.standard_normal(tokens * e).astype(np.float32)
    stream = rng.standard_normal(batch * tokens * e).astype(np.float32)
    # reference pair: broadcast the class token into row 0, then add pos to every image
    d = to_device(stream)
    kernels.launch_broadcast(d, to_device(cls), e, tokens * e, batch)
    kernels.launch_add_broadcast(d, to_device(pos), tokens * e, batch)
    want = oracle.add_broadcast(oracle.broadcast(stream, cls, e, tokens * e, batch), pos,
                                tokens * e, batch)
    np.testing.assert_array_equal(to_host(d), want)
    # the fused initialisation the runner uses
    init = to_device(np.zeros(batch * tokens * e))
    kernels.launch_init_tokens(init, to_device(cls), to_device(pos), batch, tokens, e)
    expected = np.tile(pos, batch).reshape(batch, tokens, e)
    expected[:, 0, :] = cls + pos[:e]
    np.testing.assert_array_equal(to_host(init).reshape(batch, tokens, e), expected)


def test_conversion_rounds_to_nearest_even(cuda):
    x = np.random.default_rng(2).standard_normal(10001).astype(np.float32)
    out = cuda.zeros(x.size, dtype=cuda.bfloat16, device="cuda")
    kernels.launch_convert_f32_to_bf16(to_device(x), out, x.size)
    np.testing.assert_array_equal(to_host(out), bf16_round(x))


def tf32_round(x):
    """Round to nearest TF32 value (ties away from zero in magnitude), float32 storage."""
    bits = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return rounded.view(np.float32)


def test_tf32_storage_outputs(cuda):
    """CUVIT_DTYPE_TF32: float storage holding round-to-nearest TF32 values."""
    rng = np.random.default_rng(23)
    x = rng.standard_normal(4097).astype(np.float32)
    out = to_device(np.zeros_like(x))
    kernels.launch_round_to_tf32(to_device(x), out, x.size)
    np.testing.assert_array_equal(to_host(out), tf32_round(x))
    rows, columns = 9, 192
    x = rng.standard_normal(rows * columns).astype(np.float32)
    g = np.ones(columns, np.float32)
    b = np.zeros(columns, np.float32)
    full = to_device(np.zeros(rows * columns))
    rounded = to_device(np.zeros(rows * columns))
    kernels.launch_layer_norm_ex(to_device(x), 0, to_device(g), to_device(b), full,
                                 kernels.DTYPE_F32, 0, rows, columns)
    kernels.launch_layer_norm_ex(to_device(x), 0, to_device(g), to_device(b), rounded,
                                 kernels.DTYPE_TF32, 0, rows, columns)
    np.testing.assert_array_equal(to_host(rounded), tf32_round(to_host(full)))
    images = rng.standard_normal(2 * 3 * 32 * 32).astype(np.float32)
    patches = to_device(np.zeros(images.size))
    kernels.launch_extract_patches_ex(to_device(images), patches, kernels.DTYPE_TF32, 2, 3, 32,
                                      32, 8)
    np.testing.assert_array_equal(to_host(patches),
                                  tf32_round(oracle.extract_patches(images, 2, 3, 32, 32, 8)))


@pytest.mark.parametrize("batch,classes,k", [(37, 1000, 5), (1, 1000, 1), (9, 33, 33),
                                             (300, 10, 3)])
def test_logits_top_k_matches_the_report(batch, classes, k, cuda):
    """report_top (src/main.cpp:90-114) on the device: the same classes and logits as the
    oracle, bitwise; probabilities within 1e-5 relative of its double-precision softmax."""
    rng = np.random.default_rng(batch * 7 + classes)
    logits = (3.0 * rng.standard_normal((batch, classes))).astype(np.float32)
    logits[0, : min(4, classes)] = logits[0].max() + 1.0  # ties at the top
    want_i, want_v, want_p = oracle.top_k(logits, k)
    indices = cuda.zeros((batch, k), dtype=cuda.int32, device="cuda")
    values = cuda.zeros((batch, k), device="cuda")
    probabilities = cuda.zeros((batch, k), device="cuda")
    kernels.launch_logits_top_k(to_device(logits), indices, values, probabilities, batch,
                                classes, k)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(indices.cpu().numpy(), want_i)
    np.testing.assert_array_equal(values.cpu().numpy(), want_v)
    np.testing.assert_allclose(probabilities.cpu().numpy(), want_p, rtol=1e-5, atol=1e-30)
    with pytest.raises(InvalidArgument):
        kernels.launch_logits_top_k(to_device(logits), indices, values, probabilities, batch,
                                    classes, classes + 1)


def test_logits_top_k_skips_nan(cuda):
    """NaN logits take no part in the report: not in the maximum (a NaN in column 0 used to
    seed it), not in the sum of exponentials, never picked; a row with fewer than k finite
    logits pads with index -1, value NaN, probability 0."""
    rng = np.random.default_rng(5)
    batch, classes, k = 4, 50, 5
    logits = rng.standard_normal((batch, classes)).astype(np.float32)
    logits[0, 0] = np.nan
    logits[1, 25] = np.nan
    logits[1, 26] = logits[1].max() + 2.0 if np.isfinite(logits[1]).all() else 10.0
    logits[2, :] = np.nan
    logits[2, 7] = 1.5
    logits[2, 9] = -0.5
    logits[3, ::2] = np.nan
    want_i, want_v, want_p = oracle.top_k(logits, k)
    assert want_i[2, 2] == -1 and want_p[2, 2] == 0.0
    assert np.isfinite(want_p).all() and np.isfinite(want_v[0]).all()
    indices = cuda.zeros((batch, k), dtype=cuda.int32, device="cuda")
    values = cuda.zeros((batch, k), device="cuda")
    probabilities = cuda.zeros((batch, k), device="cuda")
    kernels.launch_logits_top_k(to_device(logits), indices, values, probabilities, batch,
                                classes, k)
    cuda.cuda.synchronize()
    np.testing.assert_array_equal(indices.cpu().numpy(), want_i)
    np.testing.assert_array_equal(values.cpu().numpy(), want_v)
    np.testing.assert_allclose(probabilities.cpu().numpy(), want_p, rtol=1e-6, atol=1e-30)


def test_invalid_arguments_on_device_buffers(cuda):
    buffer = to_device(np.zeros(16))
    kernels.launch_gelu(buffer, buffer, 0)
    with pytest.raises(InvalidArgument):
        kernels.launch_gelu(None, buffer, 4)
    with pytest.raises(InvalidArgument):
        kernels.launch_layer_norm(buffer, None, buffer, buffer, 2, 4)
