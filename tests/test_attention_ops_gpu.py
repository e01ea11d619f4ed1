"""xinfer::flash_attention and xinfer::batched_flash_attention backed by this library's sm_100a
attention kernel, checked the way the reference checks its operators
(compiler/common/tests/test_attention.py): against fp32 scaled-dot-product attention with the
lower-right causal mask and grouped-query heads (relative L2 < 1 % and peak relative error
<= 5 % per row), bit-for-bit repeatable, blind to cache slots outside the valid prefix and to
other rows' caches, zeros for inactive queries, never aliasing or modifying its inputs."""

import pytest
import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from xinfer_b200 import torch_ops

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    torch_ops.load()
    return torch.ops.xinfer


def row_errors(actual, expected):
    delta = actual - expected
    return dict(
        relative_l2=(delta.norm(dim=-1) / expected.norm(dim=-1).clamp_min(1e-12)).max().item(),
        peak_relative=(delta.abs().amax(dim=-1) / expected.abs().amax(dim=-1).clamp_min(1e-12)).max().item())


def extent(length):
    """Only this CPU tensor's size is read (compiler/common/attention.py:19-24)."""
    return torch.empty(length + 1, dtype=torch.uint8)


def inputs(heads, kv_heads, dim, tokens, capacity=1024, batch=1, feature_stride=1, device="cuda"):
    o = dict(device=device, dtype=torch.bfloat16)
    q = torch.randn(batch, heads, tokens, dim * feature_stride, **o)[..., ::feature_stride]
    k = torch.randn(batch, kv_heads, capacity, dim * feature_stride, **o)[..., ::feature_stride]
    v = torch.randn(batch, kv_heads, capacity, dim * feature_stride, **o)[..., ::feature_stride]
    return q, k, v


def reference(q, k, v, count, length, scale):
    """fp32 attention of the first `count` queries over the first `length` slots."""
    positions = torch.arange(length - count, length, device=q.device)
    mask = torch.arange(length, device=q.device)[None, :] <= positions[:, None]
    with sdpa_kernel(SDPBackend.MATH):
        return F.scaled_dot_product_attention(q[:, :, :count].float(), k[:, :, :length].float(),
                                              v[:, :, :length].float(), attn_mask=mask,
                                              enable_gqa=True, scale=scale)


def assert_close(actual, expected):
    err = row_errors(actual.float().flatten(1), expected.flatten(1))
    assert err["relative_l2"] < 0.01 and err["peak_relative"] <= 0.05, err


@pytest.mark.parametrize("heads,kv_heads,dim", [(16, 8, 128), (8, 2, 256), (4, 4, 64), (8, 4, 40)])
@pytest.mark.parametrize("tokens,length", [(1, 1), (1, 129), (1, 1024), (2, 3), (16, 129),
                                           (510, 1022), (512, 512), (512, 1024)])
@torch.inference_mode()
def test_prefix_attention(ops, heads, kv_heads, dim, tokens, length):
    torch.manual_seed(35)
    q, k, v = inputs(heads, kv_heads, dim, tokens)
    before = [t.clone() for t in (q, k, v)]
    out = ops.flash_attention(q, k, v, extent(length), dim ** -0.5)
    assert out.shape == q.shape and out.is_contiguous()
    assert out.data_ptr() not in [t.data_ptr() for t in (q, k, v)]
    assert all(torch.equal(t, b) for t, b in zip((q, k, v), before))
    assert_close(out, reference(q, k, v, tokens, length, dim ** -0.5))
    # slots beyond the valid prefix are never read
    k[:, :, length:].fill_(100)
    v[:, :, length:].fill_(-100)
    assert torch.equal(out, ops.flash_attention(q, k, v, extent(length), dim ** -0.5))


@torch.inference_mode()
def test_lower_right_causality_kat(ops):
    """compiler/common/tests/test_attention.py:293-307: q = k = 0, v[slot] = slot, extent 5, two
    queries: they average slots 0..3 (1.5) and 0..4 (2.0)."""
    for heads, kv_heads, dim in ((16, 8, 128), (8, 2, 256)):
        q, k, v = inputs(heads, kv_heads, dim, 2)
        q.zero_()
        k.zero_()
        v.copy_(torch.arange(1024, device="cuda", dtype=torch.bfloat16)[None, None, :, None])
        out = ops.flash_attention(q, k, v, extent(5), dim ** -0.5)
        expected = torch.tensor([1.5, 2.0], device="cuda", dtype=torch.bfloat16)
        assert torch.equal(out, expected[None, None, :, None].expand_as(out))


@torch.inference_mode()
def test_long_prefix(ops):
    for heads, kv_heads, dim in ((16, 8, 128), (16, 4, 256)):
        for length in (8192, 8193, 16384):
            q, k, v = inputs(heads, kv_heads, dim, 2, capacity=16384)
            out = ops.flash_attention(q, k, v, extent(length), dim ** -0.5)
            assert_close(out, reference(q, k, v, 2, length, dim ** -0.5))
    with pytest.raises(RuntimeError, match="Invalid valid-prefix length"):
        ops.flash_attention(q, k, v, extent(16385), dim ** -0.5)


@torch.inference_mode()
def test_feature_strides_and_rows(ops):
    torch.manual_seed(3)
    q, k, v = inputs(8, 2, 256, 2, feature_stride=2, batch=2)
    out = ops.flash_attention(q, k, v, extent(3), 256 ** -0.5)
    dense = ops.flash_attention(q.contiguous(), k.contiguous(), v.contiguous(), extent(3), 256 ** -0.5)
    assert torch.equal(out, dense)
    k[0].fill_(5)
    v[0].fill_(7)
    assert torch.equal(out[1], ops.flash_attention(q, k, v, extent(3), 256 ** -0.5)[1])


@torch.inference_mode()
def test_invalid_arguments(ops):
    q, k, v = inputs(8, 2, 256, 2)
    for length in (0, 1, 1025):
        with pytest.raises(RuntimeError, match="Invalid valid-prefix length"):
            ops.flash_attention(q, k, v, extent(length), 256 ** -0.5)
    with pytest.raises(RuntimeError, match="Query heads must be a positive multiple"):
        ops.flash_attention(q[:, :3], k, v, extent(3), 256 ** -0.5)
    for dim in (7, 264):
        bad = inputs(8, 2, dim, 2)
        with pytest.raises(RuntimeError, match="Flash head dimension"):
            ops.flash_attention(*bad, extent(3), dim ** -0.5)


def metadata(kv_lengths, query_lengths, device):
    """batched_attention_metadata of compiler/common/attention.py:27-40."""
    lengths = torch.stack((query_lengths, kv_lengths))
    offsets = torch.cat((torch.zeros((2, 1), dtype=torch.int32), lengths.cumsum(1, dtype=torch.int32)), dim=1)
    blocks = torch.arange(kv_lengths.shape[0], device=device, dtype=torch.int32)[:, None]
    return offsets, offsets.to(device), blocks


@torch.inference_mode()
def test_batched_ragged_rows(ops):
    """Rows with full, single and no queries and different prefixes in one call (the shapes of
    compiler/common/tests/test_attention.py:39-129)."""
    torch.manual_seed(18)
    for batch in (1, 3, 8):
        for width, start, capacity in ((1, 17, 1024), (2, 511, 513), (17, 7, 1024), (512, 1, 1024),
                                       (512, 2048, 4096)):
            counts = [width if r % 3 == 0 else (0 if r % 3 == 1 else 1) for r in range(batch)]
            starts = [start - r if start >= batch else start for r in range(batch)]
            lengths = [s + c for s, c in zip(starts, counts)]
            q, k, v = inputs(16, 8, 128, width, capacity=capacity, batch=batch)
            host, cu, blocks = metadata(torch.tensor(lengths, dtype=torch.int32),
                                        torch.tensor(counts, dtype=torch.int32), q.device)
            out = ops.batched_flash_attention(q, k, v, host, cu, blocks, 128 ** -0.5)
            assert out.shape == q.shape and out.stride() == torch.empty(q.shape).stride()
            for row, (count, length) in enumerate(zip(counts, lengths)):
                assert torch.count_nonzero(out[row, :, count:]) == 0
                if count:
                    assert_close(out[row:row + 1, :, :count],
                                 reference(q[row:row + 1], k[row:row + 1], v[row:row + 1], count, length,
                                           128 ** -0.5))
                q[row, :, count:] = float("nan")
                k[row, :, length:] = float("nan")
                v[row, :, length:] = float("nan")
            assert torch.equal(out, ops.batched_flash_attention(q, k, v, host, cu, blocks, 128 ** -0.5))
            if batch > 1:
                k[0].fill_(5)
                v[0].fill_(7)
                assert torch.equal(out[1:], ops.batched_flash_attention(q, k, v, host, cu, blocks, 128 ** -0.5)[1:])


@torch.inference_mode()
def test_opcheck(ops):
    q, k, v = inputs(16, 8, 128, 4, capacity=64)
    torch.library.opcheck(ops.flash_attention.default, (q, k, v, extent(9), 128 ** -0.5),
                          test_utils=("test_schema", "test_faketensor"))
    host, cu, blocks = metadata(torch.tensor([9], dtype=torch.int32), torch.tensor([4], dtype=torch.int32), q.device)
    torch.library.opcheck(ops.batched_flash_attention.default, (q, k, v, host, cu, blocks, 128 ** -0.5),
                          test_utils=("test_schema", "test_faketensor"))
