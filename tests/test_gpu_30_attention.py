"""Flash attention (tcgen05 for head_dim 32/64/128, the CUDA-core kernel for
other multiples of 8 up to 256) against the reference's own attention math (gpu).

Cases are the reference's scripts/verify_kernel.py:39-55 set (shapes, causal,
padded, causal+padded folded into a [B,1,S,S] mask) plus the packed-view
bit-identity check (:110-129, :241-249) and the fp16 tolerance it uses for the
tensor-core kernel (3e-3, :171-182). The reference here is
reference_attention_f64 (:74-91): the baseline's arithmetic in float64 with
fully masked rows mapped to 0.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

# (label, batch, heads, seq_len, head_dim, causal, padded)
# scripts/verify_kernel.py:39-55, all 15 cases as the reference lists them
CASES = [
    ("tiny", 1, 1, 8, 8, False, False),
    ("tiny causal", 1, 1, 8, 8, True, False),
    ("tiny padded", 2, 1, 8, 8, False, True),
    ("tiny causal+pad", 2, 1, 8, 8, True, True),
    ("default", 8, 8, 128, 64, False, False),
    ("default causal", 8, 8, 128, 64, True, False),
    ("default padded", 8, 8, 128, 64, False, True),
    ("default caus+pad", 8, 8, 128, 64, True, True),
    ("long seq", 1, 8, 2048, 64, False, False),
    ("long seq causal", 1, 8, 2048, 64, True, False),
    ("odd shape", 3, 5, 37, 32, True, True),
    ("wide head_dim", 2, 4, 64, 128, False, False),
    ("wide caus+pad", 2, 4, 128, 128, True, True),
    ("head_dim 256", 2, 4, 64, 256, False, False),
    ("head_dim 256 caus", 2, 4, 128, 256, True, True),
    # further cases of this build: the tcgen05 tiny and odd shapes, packed
    # short sequences, and more head dims of the CUDA-core kernel
    ("tiny hd32", 1, 1, 8, 32, False, False),
    ("tiny hd32 causal+pad", 2, 1, 8, 32, True, True),
    ("odd hd128", 3, 2, 200, 128, True, False),
    ("short packed", 64, 4, 32, 64, False, False),
    ("hd 8", 4, 4, 64, 8, False, False),
    ("hd 8 caus+pad", 3, 4, 70, 8, True, True),
    ("hd 16 causal", 2, 3, 100, 16, True, False),
    ("hd 24", 1, 2, 33, 24, False, False),
    ("hd 16 long causal", 2, 2, 300, 16, True, False),
    ("hd 24 caus+pad", 2, 3, 257, 24, True, True),
    ("hd 8 padded", 3, 2, 200, 8, False, True),
    ("hd 48 padded", 2, 2, 90, 48, False, True),
    ("hd 256 caus+pad", 2, 2, 130, 256, True, True),
]

TOL = 3e-3


def reference_attention_f64(q, k, v, attn_mask, is_causal, scale):
    q, k, v = q.double(), k.double(), v.double()
    S = q.shape[2]
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if is_causal:
        blocked = torch.ones(S, S, device=q.device, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(blocked, float("-inf"))
    if attn_mask is not None:
        scores = scores.masked_fill(~attn_mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.nan_to_num(torch.matmul(probs, v), nan=0.0)


def build_case(b, h, s, d, causal, padded, seed=0):
    """scripts/verify_kernel.py:93-107: padding folds causal into the mask."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(b, h, s, d, generator=g, device="cuda")
    k = torch.randn(b, h, s, d, generator=g, device="cuda")
    v = torch.randn(b, h, s, d, generator=g, device="cuda")
    attn_mask, is_causal = None, causal
    if padded:
        lengths = torch.randint(1, s + 1, (b,), generator=g, device="cuda")
        valid = torch.arange(s, device="cuda")[None, :] < lengths[:, None]
        key_mask = valid[:, None, None, :]
        if causal:
            attn_mask = key_mask & torch.ones(s, s, device="cuda", dtype=torch.bool).tril()
            is_causal = False
        else:
            attn_mask = key_mask.expand(b, 1, s, s).contiguous()
    return q, k, v, attn_mask, is_causal


def as_packed_views(q, k, v):
    """q/k/v as strided views of one [B,S,3,H,hd] buffer (the fused QKV layout)."""
    b, h, s, d = q.shape
    packed = torch.empty(b, s, 3, h, d, device=q.device, dtype=q.dtype)
    for i, t in enumerate((q, k, v)):
        packed[:, :, i] = t.permute(0, 2, 1, 3)
    return packed.permute(2, 0, 3, 1, 4).unbind(0)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_attention_cases(kernels, case):
    _, b, h, s, d, causal, padded = case
    q, k, v, mask, is_causal = build_case(b, h, s, d, causal, padded)
    scale = d ** -0.5
    out = kernels.fused_attention_forward(q, k, v, mask, is_causal, scale, 0, 0, 0)
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = reference_attention_f64(q, k, v, mask, is_causal, scale)
    err = (out.double() - ref).abs().max().item()
    assert err <= TOL, err
    assert torch.isfinite(out).all()
    # layout 1 is the same values as [B,S,H*hd]
    out1 = kernels.fused_attention_forward(q, k, v, mask, is_causal, scale, 0, 1, 0)
    assert torch.equal(out1, out.transpose(1, 2).reshape(b, s, h * d))
    # The fused-QKV strided views give the same bits as contiguous inputs
    # whenever both take the same tiling. Sequences of 128 or more always do
    # (each gets tiles of its own); shorter ones are packed several to a tile
    # when the layout allows it (the fused buffer does, a contiguous
    # [B,H,S,hd] with H > 1 does not), which moves keys to other tile columns
    # and so can change the last bit of an fp32 sum.
    q16, k16, v16 = (t.half() for t in (q, k, v))
    qp, kp, vp = as_packed_views(q16, k16, v16)
    a = kernels.fused_attention_forward(q16, k16, v16, mask, is_causal, scale, 0, 0, 0)
    p = kernels.fused_attention_forward(qp, kp, vp, mask, is_causal, scale, 0, 0, 0)
    if s >= 128:
        assert torch.equal(a, p)
    else:
        assert (a.float() - p.float()).abs().max().item() <= 1e-3


@pytest.mark.parametrize("d", [64, 8, 16, 24, 256])
def test_key_mask_with_causal_unfolded(kernels, d):
    """A [B,1,1,S] key mask plus is_causal (the model's call), not folded."""
    b, h, s = 3, 4, 256
    q, k, v, _, _ = build_case(b, h, s, d, False, False, seed=4)
    lengths = torch.tensor([256, 130, 1], device="cuda")
    valid = torch.arange(s, device="cuda")[None, :] < lengths[:, None]
    mask = valid[:, None, None, :]
    out = kernels.fused_attention_forward(q, k, v, mask, True, d ** -0.5, 0, 0, 0)
    ref = reference_attention_f64(q, k, v, mask, True, d ** -0.5)
    assert (out.double() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("d", [128, 64, 32])
def test_mixed_short_and_long_key_ranges(kernels, d):
    """Batch rows of 100 and of 512 valid keys, many work items per CTA: one-
    key-tile items (handled by one softmax group) interleave with four-tile
    items (both groups), so an S/P buffer's uses alternate between the groups
    in every pattern, and each group must still wait on its own S tiles'
    phases, not a phase of the other group's."""
    b, h, s = 96, 4, 512
    q, k, v, _, _ = build_case(b, h, s, d, False, False, seed=8)
    lengths = torch.tensor([100 if i % 2 == 0 else 512 for i in range(b)], device="cuda")
    lengths[5::7] = 129   # two key tiles, one of them nearly empty
    valid = torch.arange(s, device="cuda")[None, :] < lengths[:, None]
    mask = valid[:, None, None, :]
    out = kernels.fused_attention_forward(q, k, v, mask, False, d ** -0.5, 0, 0, 0)
    again = kernels.fused_attention_forward(q, k, v, mask, False, d ** -0.5, 0, 0, 0)
    assert torch.equal(out, again)
    ref = reference_attention_f64(q, k, v, mask, False, d ** -0.5)
    assert (out.double() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("d", [64, 8])
def test_fully_masked_rows_are_zero(kernels, d):
    b, h, s = 2, 2, 64
    q, k, v, _, _ = build_case(b, h, s, d, False, False, seed=5)
    mask = torch.zeros(b, 1, 1, s, dtype=torch.bool, device="cuda")
    mask[0, ..., :10] = True
    out = kernels.fused_attention_forward(q, k, v, mask, False, d ** -0.5, 0, 0, 0)
    assert torch.all(out[1] == 0)
    ref = reference_attention_f64(q, k, v, mask, False, d ** -0.5)
    assert (out.double() - ref).abs().max().item() <= TOL


@pytest.mark.parametrize("hd", [4, 12, 264])
def test_uncovered_head_dims_raise(kernels, hd):
    q = torch.randn(1, 1, 16, hd, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        kernels.fused_attention_forward(q, q, q, None, False, hd ** -0.5, 0, 0, 0)


def test_uncovered_precision_raises(kernels):
    q = torch.randn(1, 1, 16, 64, device="cuda")
    with pytest.raises(RuntimeError, match="not covered"):
        kernels.fused_attention_forward(q, q, q, None, False, 0.125, 1, 0, 0)
    with pytest.raises(RuntimeError, match="not covered"):
        kernels.fused_attention_forward(q, q, q, None, False, 0.125, 0, 0, 4)


# Split-KV: shapes with fewer (batch, head, query tile) items than SMs and long
# key ranges, where dotl_attention cuts each tile's keys into runs and a
# combine kernel folds them (the reference's split path and combine,
# attention_wmma.cuh:662-759, 1783-1826). (batch, heads, seq, head_dim,
# causal, per-row valid key counts or None)
SPLIT_CASES = [
    (1, 2, 2048, 64, True, None),
    (1, 1, 4096, 128, False, None),
    (2, 1, 1536, 32, True, [1536, 300]),
    (2, 2, 1024, 64, False, [1024, 0]),      # a row with no valid key: zeros
]


@pytest.mark.parametrize("case", SPLIT_CASES)
def test_split_kv_matches_one_pass(kernels, case):
    b, h, s, d, causal, lengths = case
    assert kernels.attention_workspace_bytes(b, h, s, d, causal, torch.device("cuda")) > 0, \
        "the plan must split this shape"
    g = torch.Generator(device="cuda").manual_seed(s + d)
    q, k, v = (torch.randn(b, h, s, d, device="cuda", generator=g).half() for _ in range(3))
    key_mask = None
    if lengths is not None:
        key_mask = torch.arange(s, device="cuda")[None, :] < torch.tensor(lengths, device="cuda")[:, None]
    scale = d ** -0.5
    one = kernels.attention_packed(q, k, v, causal, scale, key_mask=key_mask, split_kv=False)
    split = kernels.attention_packed(q, k, v, causal, scale, key_mask=key_mask)
    again = kernels.attention_packed(q, k, v, causal, scale, key_mask=key_mask)
    assert torch.equal(split, again), "split-KV must give the same bits on every call"
    # the runs fold in another order than one pass: within fp16 output rounding
    assert (split.float() - one.float()).abs().max().item() <= 2e-3
    mask4 = key_mask[:, None, None, :] if key_mask is not None else None
    ref = reference_attention_f64(q, k, v, mask4, causal, scale).transpose(1, 2).reshape(b, s, h * d)
    err = (split.double() - ref).abs().max().item()
    assert err <= TOL, err
    pair = kernels.attention_packed(q, k, v, causal, scale, key_mask=key_mask, out_pair=True)
    assert torch.equal(pair[0], split)
    if lengths is not None and 0 in lengths:
        assert torch.all(split[lengths.index(0)] == 0)


@pytest.mark.parametrize("S,d,causal,padded", [(32, 64, False, False), (32, 64, True, True), (64, 32, False, True),
                                                (16, 128, True, False), (128, 64, False, True)])
def test_single_tile_items_overlapped(kernels, S, d, causal, padded):
    """Every work item one key tile (packed sequences that divide 128, or
    sequences of 128) and more items than SMs, so CTAs take several: the MMA
    thread then issues the next item's S before this item's P.V and both
    softmax groups work at once. Checked against float64, and bit for bit
    against the same sequences run 128 items at a time (one item per CTA,
    the kernel without the overlap)."""
    H = 4
    B = 1024 * 32 // S if S < 128 else 64          # 1024 or 256 items
    g = torch.Generator(device="cuda").manual_seed(S + d)
    qkv = torch.randn(B, S, 3, H, d, device="cuda", generator=g).half()
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    mask = None
    if padded:
        lengths = torch.randint(1, S + 1, (B,), device="cuda", generator=g)
        mask = torch.arange(S, device="cuda")[None, :] < lengths[:, None]
    scale = d ** -0.5
    out = kernels.attention_packed(q, k, v, causal, scale, key_mask=mask)
    # each chunk: 128 items (128 // H batch rows of one tile row block each)
    per = 128 * 128 // (S * H) if S < 128 else 128 // H
    for lo in range(0, B, per):
        hi = min(lo + per, B)
        part = kernels.attention_packed(q[lo:hi], k[lo:hi], v[lo:hi], causal, scale,
                                        key_mask=mask[lo:hi] if mask is not None else None)
        assert torch.equal(part, out[lo:hi]), f"batch rows {lo}:{hi} differ from the whole batch"
    n = min(B, 64)
    am = mask[:n, None, None, :] if mask is not None else None
    ref = reference_attention_f64(q[:n].float(), k[:n].float(), v[:n].float(), am, causal, scale)
    ref = ref.transpose(1, 2).reshape(n, S, H * d)
    assert (out[:n].double() - ref).abs().max().item() <= TOL
