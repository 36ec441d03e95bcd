"""The fused attention kernel against the oracle's restatement of the reference's attention
(tests/reference/vit.hpp:149-183: Q.K^T * scale -> softmax -> .V per head).

BF16 runs on bf16-rounded projections, so the remaining error is P rounded to bf16 (2^-9
relative) plus the bf16 output store (2^-9): bounded by 1e-2 of the largest |V| of the head.
TF32 rounds Q, K, P and V to 10-bit mantissas: the same bound holds with room to spare.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from cuvit import kernels
from helpers import bf16_round, to_device, to_host

pytestmark = pytest.mark.gpu


def run_attention(qkv, batch, tokens, heads, dtype, torch):
    e = heads * 64
    torch_dtype = torch.bfloat16 if dtype == kernels.DTYPE_BF16 else torch.float32
    dq = to_device(qkv, torch_dtype)
    out = torch.full((batch * tokens * e,), float("nan"), dtype=torch_dtype, device="cuda")
    kernels.launch_attention(dq, out, dtype, batch, tokens, heads, 64, 0.125)
    torch.cuda.synchronize()
    return to_host(out).reshape(batch, tokens, e)


def expected(qkv, batch, tokens, heads):
    e = heads * 64
    per_image = qkv.reshape(batch, tokens * 3 * e)
    return np.stack([oracle.attention(per_image[b], tokens, e, heads).reshape(tokens, e)
                     for b in range(batch)])


@pytest.mark.parametrize("dtype", [kernels.DTYPE_BF16, kernels.DTYPE_F32], ids=["bf16", "tf32"])
@pytest.mark.parametrize("batch,tokens,heads", [(1, 1, 1), (2, 17, 2), (2, 33, 2), (1, 64, 3),
                                                (1, 97, 2), (3, 128, 2), (2, 129, 1),
                                                (2, 197, 3), (1, 197, 12), (2, 225, 2),
                                                (1, 241, 1), (1, 256, 2), (4, 50, 16)])
def test_fused_attention_matches_reference_attention(dtype, batch, tokens, heads, cuda):
    rng = np.random.default_rng(tokens * 13 + heads + batch)
    qkv = rng.standard_normal(batch * tokens * 3 * heads * 64).astype(np.float32)
    if dtype == kernels.DTYPE_BF16:
        qkv = bf16_round(qkv)
    got = run_attention(qkv, batch, tokens, heads, dtype, cuda)
    want = expected(qkv, batch, tokens, heads)
    assert np.isfinite(got).all(), "rows beyond the token count leaked into the output"
    v_max = np.abs(qkv.reshape(batch, tokens, 3, heads * 64)[:, :, 2]).max()
    err = np.abs(got - want).max()
    assert err <= 1e-2 * v_max, f"max error {err:.3g} vs bound {1e-2 * v_max:.3g}"


@pytest.mark.parametrize("batch,tokens,heads", [(26, 197, 12), (50, 80, 8), (40, 128, 8),
                                                (60, 129, 5), (2, 224, 100)])
def test_fused_attention_several_pairs_per_cta(batch, tokens, heads, cuda):
    """More (image, head) pairs than SMs, so each persistent CTA walks two or three pairs and
    reuses its shared-memory and tensor-memory buffers; shapes with one query tile (every TMEM
    lane quarter idle past 80 tokens), two tiles, a one-row second tile, and 224 tokens (the
    widest score buffer)."""
    rng = np.random.default_rng(batch * 7 + tokens + heads)
    qkv = bf16_round(rng.standard_normal(batch * tokens * 3 * heads * 64).astype(np.float32))
    got = run_attention(qkv, batch, tokens, heads, kernels.DTYPE_BF16, cuda)
    want = expected(qkv, batch, tokens, heads)
    assert np.isfinite(got).all()
    v_max = np.abs(qkv.reshape(batch, tokens, 3, heads * 64)[:, :, 2]).max()
    err = np.abs(got - want).max()
    assert err <= 1e-2 * v_max, f"max error {err:.3g} vs bound {1e-2 * v_max:.3g}"


def test_fused_attention_sharp_and_flat_rows(cuda):
    """Large logits (near one-hot softmax) and all-equal keys (uniform softmax)."""
    batch, tokens, heads = 1, 197, 2
    e = heads * 64
    rng = np.random.default_rng(3)
    qkv = rng.standard_normal((batch, tokens, 3, e)).astype(np.float32)
    qkv[:, :, 0] *= 6.0  # logits of order 6*sqrt(64)/8 * |k|: sharp
    qkv[:, :60, 1] = qkv[:, 0:1, 1]  # 60 identical keys
    qkv = bf16_round(qkv.reshape(-1))
    for dtype in (kernels.DTYPE_BF16, kernels.DTYPE_F32):
        got = run_attention(qkv, batch, tokens, heads, dtype, cuda)
        want = expected(qkv, batch, tokens, heads)
        v_max = np.abs(qkv.reshape(batch, tokens, 3, e)[:, :, 2]).max()
        assert np.abs(got - want).max() <= 1.5e-2 * v_max


def test_fused_attention_is_deterministic_and_batch_invariant(cuda):
    batch, tokens, heads = 4, 197, 3
    qkv = bf16_round(np.random.default_rng(11).standard_normal(batch * tokens * 3 * heads * 64))
    first = run_attention(qkv, batch, tokens, heads, kernels.DTYPE_BF16, cuda)
    second = run_attention(qkv, batch, tokens, heads, kernels.DTYPE_BF16, cuda)
    np.testing.assert_array_equal(first, second)
    per_image = qkv.reshape(batch, -1)
    for b in range(batch):
        alone = run_attention(per_image[b], 1, tokens, heads, kernels.DTYPE_BF16, cuda)
        np.testing.assert_array_equal(alone[0], first[b])


@pytest.mark.parametrize("late_block,boost", [(2, 12.0), (3, 9.0), (1, 14.0), (2, 4.0)])
def test_fused_attention_row_maximum_in_a_later_key_block(late_block, boost, cuda):
    """Rows whose maximum sits in one narrow group of keys far from the first ones: a few keys
    of the 64-key block `late_block` score `boost` (natural-log units) above all others, so
    the exponentials span up to 2^20, and each row's maximum lies in the part of the keys the
    second softmax warpgroup (or the first, for block 1) reads; against the oracle's exact
    softmax."""
    batch, tokens, heads = 2, 197, 2
    e = heads * 64
    rng = np.random.default_rng(int(boost * 10) + late_block)
    qkv = 0.3 * rng.standard_normal((batch, tokens, 3, e)).astype(np.float32)
    direction = rng.standard_normal(64).astype(np.float32)
    direction /= np.linalg.norm(direction)
    first = late_block * 64 + 3
    keys = slice(first, min(first + 5, tokens))
    for h in range(heads):
        cols = slice(h * 64, (h + 1) * 64)
        qkv[:, :, 0, cols] = 4.0 * direction          # every query along `direction`
        # s = 4 * a for these keys: 0.125 * s = boost  ->  a = 2 * boost
        qkv[:, keys, 1, cols] = (2.0 * boost) * direction
    qkv = bf16_round(qkv.reshape(-1))
    got = run_attention(qkv, batch, tokens, heads, kernels.DTYPE_BF16, cuda)
    want = expected(qkv, batch, tokens, heads)
    assert np.isfinite(got).all()
    v_max = np.abs(qkv.reshape(batch, tokens, 3, e)[:, :, 2]).max()
    err = np.abs(got - want).max()
    assert err <= 1e-2 * v_max, f"max error {err:.3g} vs bound {1e-2 * v_max:.3g}"
