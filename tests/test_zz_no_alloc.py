"""dotl_attention_static_scratch through the C ABI (gpu).

The entry point serves callers that cannot allocate device memory themselves
(a binding that owns no CUDA allocator, or code that must not grow device
memory): the split-KV scratch of the attention is a static array inside the
library instead of a workspace the caller passes. Checked here, on a shape
whose split plan uses that scratch: two calls in a row each give the same
output as dotl_attention with a torch-allocated workspace (the same plan, so
the same bits) and meet the float64 reference within the attention tests'
3e-3; and a shape whose plan needs more than the array holds is rejected.

This file is collected last on purpose, so a run that stops at its first
failure has run every other test first.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 3e-3
F16 = 1


def _strides(t):
    return (ctypes.c_int64 * 3)(*[int(v) for v in t.stride()[:3]])


def _call(lib, fn, q, k, v, causal, out, extra):
    B, H, S, hd = q.shape
    no_mask = (ctypes.c_int64 * 4)(0, 0, 0, 0)
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, S, hd, _strides(q), _strides(k), _strides(v),
              None, 0, no_mask, 1 if causal else 0, float(hd ** -0.5), out.data_ptr(), 1, F16, *extra, stream)


def test_static_scratch_matches_workspace_path(kernels):
    import dotl_ops

    lib = dotl_ops.lib()
    B, H, S, hd, causal = 1, 2, 2048, 64, True
    need = kernels.attention_workspace_bytes(B, H, S, hd, causal, torch.device("cuda"))
    assert 0 < need <= 16 << 20, "the shape must take the split path within the static array"
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(B, H, S, hd, device="cuda", generator=g).half() for _ in range(3))

    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    want = torch.empty(B, S, H * hd, dtype=torch.float16, device="cuda")
    assert _call(lib, lib.dotl_attention, q, k, v, causal, want, (ws.data_ptr(), need)) == 0

    s = (q.double() @ k.double().transpose(-1, -2)) * hd ** -0.5
    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device="cuda").triu(1), float("-inf"))
    ref = (torch.softmax(s, -1) @ v.double()).transpose(1, 2).reshape(B, S, H * hd)

    for _ in range(2):   # the second call finds the array holding the first call's runs
        got = torch.full_like(want, float("nan"))
        rc = _call(lib, lib.dotl_attention_static_scratch, q, k, v, causal, got, ())
        assert rc == 0, lib.dotl_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert (got.double() - ref).abs().max().item() <= TOL


def test_static_scratch_rejects_plans_over_its_size(kernels):
    import dotl_ops

    lib = dotl_ops.lib()
    B, H, S, hd, causal = 1, 1, 4736, 128, True
    need = kernels.attention_workspace_bytes(B, H, S, hd, causal, torch.device("cuda"))
    assert need > 16 << 20
    q, k, v = (torch.zeros(B, H, S, hd, device="cuda", dtype=torch.float16) for _ in range(3))
    out = torch.empty(B, S, H * hd, dtype=torch.float16, device="cuda")
    assert _call(lib, lib.dotl_attention_static_scratch, q, k, v, causal, out, ()) == 2
    assert "static array" in lib.dotl_last_error().decode()
