"""dotl_allreduce_ln on one GPU (gpu).

One launch stands in for one rank. The "peers'" buffers are further local
buffers, and their start/end flags are written beforehand, so nothing waits on
another kernel. That covers the sum over ranks (in rank order, bit-exact), the
bias / residual / row masks, the LayerNorm, and both modes: one-shot (every row,
own outputs) and push (this rank's rows, every rank's outputs). A flag that
nothing sets checks the bounded wait: the call gives up, sets the device error
bit and the context stays usable. The cross-GPU path runs in
test_gpu_50_tensor_parallel.py.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

PEER_MAX = 8
TIMEOUT_BIT = 4


def _signals(k, world, rank, preset):
    """Zeroed signal areas; with preset, this rank's flags from every peer are
    already far ahead, so both handshakes pass at once."""
    blocks = k.peer_blocks()
    words = k.peer_signal_bytes(blocks) // 4
    sig = [torch.zeros(words, dtype=torch.int32, device="cuda") for _ in range(world)]
    if preset:
        sig[rank][blocks:] = 1 << 30
    return blocks, sig


def _ref(x, parts, bias, valid, w, b, eps, keep):
    s = parts[0].clone()
    for p in parts[1:]:
        s = s + p
    if bias is not None:
        s = s + bias
    x_new = torch.where(valid[:, None], x + s, x) if valid is not None else x + s
    y = torch.nn.functional.layer_norm(x_new.double(), (x.shape[1],), w.double(), b.double(), eps)
    if keep is not None:
        y = y * keep[:, None]
    return x_new, y


def _run(k, world, rank, push, rows, D, half, with_bias, masks, seed, preset=True, timeout_ms=2000):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, D, device="cuda", generator=g)
    parts = [torch.randn(rows, D, device="cuda", generator=g) for _ in range(world)]
    bias = torch.randn(D, device="cuda", generator=g) * 0.1 if with_bias else None
    w = torch.randn(D, device="cuda", generator=g) * 0.2 + 1.0
    b = torch.randn(D, device="cuda", generator=g) * 0.1
    valid = torch.rand(rows, device="cuda", generator=g) > 0.3 if masks else None
    keep = torch.rand(rows, device="cuda", generator=g) > 0.3 if masks else None
    blocks, sig = _signals(k, world, rank, preset)
    x_new = [torch.full((rows, D), float("nan"), device="cuda") for _ in range(world)]
    normed = [torch.full((rows, D), float("nan"), device="cuda", dtype=torch.float16 if half else torch.float32)
              for _ in range(world)]
    dst = range(world) if push else [rank]
    k.allreduce_ln(world, rank, [p.data_ptr() for p in parts], [s.data_ptr() for s in sig],
                   [t.data_ptr() if i in dst else None for i, t in enumerate(x_new)],
                   [t.data_ptr() if i in dst else None for i, t in enumerate(normed)], half, push,
                   x, bias, w, b, 1e-5, valid, keep, rows, D, blocks, timeout_ms)
    torch.cuda.synchronize()
    return x, parts, bias, valid, w, b, keep, x_new, normed


@pytest.mark.parametrize("D", [4, 128, 256, 1000, 2048])
@pytest.mark.parametrize("half", [False, True])
def test_single_rank(kernels, D, half):
    rows = 777
    x, parts, bias, valid, w, b, keep, x_new, normed = _run(kernels, 1, 0, False, rows, D, half, True, True, D)
    ref_x, ref_y = _ref(x, parts, bias, valid, w, b, 1e-5, keep)
    assert torch.equal(x_new[0], ref_x)
    tol = 2 ** -10 if half else 1e-5
    err = (normed[0].double() - ref_y).abs() / (ref_y.abs() + 1.0)
    assert err.max().item() < tol


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("push", [False, True])
def test_sum_over_ranks(kernels, world, push):
    rows, D, rank = 1000, 512, world - 1
    x, parts, bias, valid, w, b, keep, x_new, normed = _run(kernels, world, rank, push, rows, D, True, True,
                                                            True, 100 + world)
    ref_x, ref_y = _ref(x, parts, bias, valid, w, b, 1e-5, keep)
    if push:
        chunk = -(-rows // world)
        lo, hi = min(rows, chunk * rank), min(rows, chunk * (rank + 1))
        for i in range(world):   # every rank's buffers get this rank's rows, nothing else
            assert torch.equal(x_new[i][lo:hi], ref_x[lo:hi])
            err = (normed[i][lo:hi].double() - ref_y[lo:hi]).abs() / (ref_y[lo:hi].abs() + 1.0)
            assert err.max().item() < 2 ** -10
            assert torch.isnan(x_new[i][:lo]).all() and torch.isnan(x_new[i][hi:]).all()
    else:
        assert torch.equal(x_new[rank], ref_x)   # rank-order sum, bit-exact
        err = (normed[rank].double() - ref_y).abs() / (ref_y.abs() + 1.0)
        assert err.max().item() < 2 ** -10
        for i in range(world):
            if i != rank:
                assert torch.isnan(x_new[i]).all()


def test_no_bias_no_masks_and_x_new_not_stored(kernels):
    k = kernels
    rows, D = 300, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(rows, D, device="cuda", generator=g)
    part = torch.randn(rows, D, device="cuda", generator=g)
    w, b = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    blocks, sig = _signals(k, 1, 0, True)
    out = torch.empty(rows, D, device="cuda")
    k.allreduce_ln(1, 0, [part.data_ptr()], [sig[0].data_ptr()], None, [out.data_ptr()], False, False,
                   x, None, w, b, 1e-5, None, None, rows, D, blocks, 2000)
    ref = torch.nn.functional.layer_norm((x + part).double(), (D,), eps=1e-5)
    assert (out.double() - ref).abs().max().item() < 1e-5


def test_graph_replay_advances_the_call_counter(kernels):
    """The flags carry a per-CTA counter kept on the device, so a captured call
    replays correctly (each replay is a new call for the handshake)."""
    k = kernels
    rows, D, world = 512, 256, 2
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(rows, D, device="cuda", generator=g)
    parts = [torch.randn(rows, D, device="cuda", generator=g) for _ in range(world)]
    w, b = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    blocks, sig = _signals(k, world, 0, True)
    out = torch.empty(rows, D, device="cuda")
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            k.allreduce_ln(world, 0, [p.data_ptr() for p in parts], [s.data_ptr() for s in sig], None,
                           [out.data_ptr(), None], False, False, x, None, w, b, 1e-5, None, None, rows, D,
                           blocks, 2000)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert k.device_error(clear=True) == 0
    assert torch.equal(sig[0][:blocks], torch.full((blocks,), 3, dtype=torch.int32, device="cuda"))
    # rank 0 told "rank 1" (slot [b][0] of its area) that it reached call 3
    start = sig[1][blocks: blocks + blocks * PEER_MAX].view(blocks, PEER_MAX)[:, 0]
    assert torch.equal(start, torch.full((blocks,), 3, dtype=torch.int32, device="cuda"))
    ref = torch.nn.functional.layer_norm((x + (parts[0] + parts[1])).double(), (D,), eps=1e-5)
    assert (out.double() - ref).abs().max().item() < 1e-5


def test_missing_peer_times_out_and_context_survives(kernels):
    """A peer that never arrives: every CTA gives up after timeout_ms, sets the
    device error bit, does no work, and the GPU stays usable."""
    k = kernels
    k.device_error(clear=True)
    x, parts, bias, valid, w, b, keep, x_new, normed = _run(k, 2, 0, False, 256, 128, False, False, False, 5,
                                                            preset=False, timeout_ms=50)
    assert k.device_error(clear=True) & TIMEOUT_BIT
    assert torch.isnan(x_new[0]).all() and torch.isnan(normed[0]).all()
    y = k.linear_fp16(torch.ones(128, 64, device="cuda").half(), torch.ones(64, 64, device="cuda").half(),
                      torch.zeros(64, device="cuda"))
    assert torch.all(y == 64)
    assert k.device_error(clear=True) == 0


def test_rejects(kernels):
    k = kernels
    rows, D = 16, 128
    x = torch.zeros(rows, D, device="cuda")
    w, b = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    blocks, sig = _signals(k, 1, 0, True)
    out = torch.full((rows, D), float("nan"), device="cuda")

    def call(world=1, rank=0, D_=D, blocks_=blocks, timeout=2000, parts=None):
        parts = parts if parts is not None else [x.data_ptr()] * world
        k.allreduce_ln(world, rank, parts, [sig[0].data_ptr()] * world, None, [out.data_ptr()] * world,
                       False, False, x, None, w, b, 1e-5, None, None, rows, D_, blocks_, timeout)

    with pytest.raises(RuntimeError, match="world"):
        call(world=9)
    with pytest.raises(RuntimeError, match="world"):
        call(rank=1)
    with pytest.raises(RuntimeError, match="multiple of 4"):
        call(D_=126)
    with pytest.raises(RuntimeError, match="multiple of 4"):
        call(D_=4096)
    with pytest.raises(RuntimeError, match="blocks"):
        call(blocks_=blocks + 1)
    with pytest.raises(RuntimeError, match="timeout_ms"):
        call(timeout=0)
    with pytest.raises(RuntimeError, match="aligned"):
        call(parts=[x.data_ptr() + 4])
    with pytest.raises(RuntimeError, match="NULL"):
        call(parts=[None])
    torch.cuda.synchronize()
    assert torch.isnan(out).all()   # a rejected call enqueues nothing


@pytest.mark.parametrize("world", [1, 2, 4])
def test_gemm_scatters_tiles_to_row_owners(kernels, world):
    """dotl_linear_peer with every "rank's" receive slot a local buffer: rows
    [r R, (r+1) R) land in slot r at offset 0, with the bits of dotl_linear."""
    k = kernels
    R, K, N = 256, 512, 384
    g = torch.Generator(device="cuda").manual_seed(world)
    a = torch.randn(world * R, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).half()
    slots = [torch.full((R, N), float("nan"), device="cuda") for _ in range(world)]
    k.linear_peer(a, w, None, [t.data_ptr() for t in slots], R, N)
    ref = k.linear_fp16(a, w, torch.zeros(N, device="cuda"))
    torch.cuda.synchronize()
    for r in range(world):
        assert torch.equal(slots[r] + 0.0, ref[r * R:(r + 1) * R] + 0.0), r


def test_reduction_from_owner_slots(kernels):
    """parts_local: the partial sums of this rank's rows come from its own
    slots (row lo at offset 0), results pushed to every rank's buffers."""
    k = kernels
    world, rank, rows, D = 2, 1, 512, 256
    lo, hi = 256, 512
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(rows, D, device="cuda", generator=g)
    slots = [torch.randn(hi - lo, D, device="cuda", generator=g) for _ in range(world)]
    bias = torch.randn(D, device="cuda", generator=g) * 0.1
    w, b = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    blocks, sig = _signals(k, world, rank, True)
    x_new = [torch.full((rows, D), float("nan"), device="cuda") for _ in range(world)]
    normed = [torch.full((rows, D), float("nan"), device="cuda", dtype=torch.float16) for _ in range(world)]
    k.allreduce_ln(world, rank, [t.data_ptr() for t in slots], [s.data_ptr() for s in sig],
                   [t.data_ptr() for t in x_new], [t.data_ptr() for t in normed], True, True, x, bias, w, b,
                   1e-5, None, None, rows, D, blocks, 2000, parts_local=True)
    torch.cuda.synchronize()
    ref_x = x[lo:hi] + ((slots[0] + slots[1]) + bias)
    ref_y = torch.nn.functional.layer_norm(ref_x.double(), (D,), eps=1e-5)
    for i in range(world):
        assert torch.equal(x_new[i][lo:hi], ref_x)
        assert (normed[i][lo:hi].double() - ref_y).abs().max().item() < 4e-3
        assert torch.isnan(x_new[i][:lo]).all()


def _phantom_allreduce_ln(phantom):
    """PeerGroup.allreduce_ln as if the group had a second rank that never
    calls: the real kernel, one-shot, with rank 1's partial sums and signal
    area as local buffers whose flags nothing sets."""
    from optimized.peer import PeerTimeoutError

    def call(self, x, bias, ln_w, ln_b, eps, x_new, normed, rows, sum_row_valid=None,
             normed_row_valid=None, from_owners=False):
        if self.poisoned:
            raise PeerTimeoutError("poisoned")
        if not phantom:
            phantom["sig"] = torch.zeros(self.signal_bytes // 4, dtype=torch.int32, device=x.device)
            phantom["part"] = torch.zeros(self.rows, self.d, device=x.device)
        self.k.allreduce_ln(2, 0, [self.ptrs["part"][0], phantom["part"].data_ptr()],
                            [self.ptrs["signal"][0], phantom["sig"].data_ptr()],
                            None if x_new is None else [self.ptrs[x_new][0], None],
                            [self.ptrs[normed][0], None], normed == "n16", False, x, bias, ln_w, ln_b, eps,
                            sum_row_valid, normed_row_valid, rows, self.d, self.blocks, self.timeout_ms,
                            signal_bytes=self.signal_bytes, status=self.status.data_ptr())
    return call


@pytest.mark.parametrize("error_check", ["sync", "deferred"])
def test_tp_forward_raises_when_a_peer_never_arrives(kernels, monkeypatch, error_check):
    """Through TensorParallelTransformer.forward: the fused reduction waits for
    a peer that never calls, gives up after 50 ms, and the forward raises
    PeerTimeoutError (at its end with error_check="sync", at the next check
    with "deferred") instead of returning the invalid output. The group is then
    poisoned; the next forward rebuilds it and is correct again."""
    import datetime
    import socket

    import torch.distributed as dist
    from oracle import layer as O
    from optimized import peer as peer_mod
    from optimized.tensor_parallel import TensorParallelTransformer

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    store = dist.TCPStore("127.0.0.1", port, 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        cfg = O.TransformerConfig(2, 128, 256, 4, 512, 1, True)
        params = O.init_params(cfg, 31)
        x, _ = O.generate_random_case(cfg, 32, 0.0, 1.0)
        x = x.cuda()
        tp = TensorParallelTransformer(cfg, params, timeout_ms=50, error_check=error_check)
        try:
            with torch.inference_mode():
                good = tp(x).clone()
                torch.cuda.synchronize()
                tp.check()
                phantom = {}
                monkeypatch.setattr(peer_mod.PeerGroup, "allreduce_ln", _phantom_allreduce_ln(phantom))
                if error_check == "sync":
                    with pytest.raises(peer_mod.PeerTimeoutError):
                        tp(x)
                else:
                    tp(x)                               # returns; the failure is seen afterwards
                    torch.cuda.synchronize()
                    with pytest.raises(peer_mod.PeerTimeoutError):
                        tp.check()
                assert tp.peer.poisoned
                assert kernels.device_error(clear=True) & TIMEOUT_BIT
                monkeypatch.undo()
                old = tp.peer
                again = tp(x).clone()
                torch.cuda.synchronize()
                tp.check()
                assert tp.peer is not old and not tp.peer.poisoned
                assert torch.equal(again, good)
        finally:
            tp.close()
    finally:
        dist.destroy_process_group()
