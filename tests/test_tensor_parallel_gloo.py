"""Tensor-parallel sharding (optimized/tensor_parallel.py) on CPU ranks.

Two gloo ranks each take their TPShardPlan slice of a full state_dict, run the
layer's per-rank arithmetic in plain fp32 torch with an all-reduce after the
output projection and after the second FFN GEMM (the decomposition the GPU
path uses), and must reproduce the unsharded oracle forward.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import layer as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_cpu_forward(w, cfg, plan, x, mask):
    B, S, d = x.shape
    hl, hd = plan.local_heads, plan.head_dim
    ln = lambda t, n: F.layer_norm(t, (d,), w[n + ".weight"], w[n + ".bias"], 1e-5)
    normed = ln(x, "layers.0.norm1")
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        qkv = F.linear(normed, w[p + "wqkv"], w[p + "bqkv"])
        q, k, v = qkv.view(B, S, 3, hl, hd).permute(2, 0, 3, 1, 4).unbind(0)
        ctx = O.attention_reference(q.contiguous(), k.contiguous(), v.contiguous(),
                                    mask[:, None, None, :] if mask is not None else None,
                                    cfg.causal, hd ** -0.5)
        ctx = ctx.transpose(1, 2).reshape(B, S, hl * hd)
        part = F.linear(ctx, w[p + "wo"], w[p + "bo"])
        if mask is not None:
            part = part.masked_fill(~mask[..., None], 0)
        dist.all_reduce(part)
        x1 = x + part
        h = F.gelu(F.linear(ln(x1, p + "norm2"), w[p + "w1"], w[p + "b1"]), approximate="none")
        part2 = F.linear(h, w[p + "w2"], w[p + "b2"])
        if mask is not None:
            part2 = part2.masked_fill(~mask[..., None], 0)
        dist.all_reduce(part2)
        x = x1 + part2
        last = i == cfg.num_layers - 1
        normed = ln(x, "final_norm" if last else f"layers.{i + 1}.norm1")
    if mask is not None:
        normed = normed.masked_fill(~mask[..., None], 0)
    return normed


def _worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from optimized.tensor_parallel import TPShardPlan

        cfg = O.TransformerConfig(2, 20, 64, 4, 128, 2, True)
        params = O.init_params(cfg, 8)
        x, mask = O.generate_random_case(cfg, 9, 0.5, 1.0)
        plan = TPShardPlan(cfg.d_model, cfg.num_heads, cfg.ffn_dim, world, rank)
        w = plan.shard(params, cfg.num_layers)
        out = _tp_cpu_forward(w, cfg, plan, x, mask)
        if rank == 0:
            torch.save({"tp": out, "full": O.baseline_forward(params, cfg, x, mask)}, path)
    finally:
        dist.destroy_process_group()


def test_tp_decomposition_matches_oracle(tmp_path):
    path = str(tmp_path / "tp.pt")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, start_method="spawn", join=True)
    r = torch.load(path)
    assert (r["tp"] - r["full"]).abs().max().item() < 1e-4


def test_shard_plan_slices():
    from optimized.tensor_parallel import TPShardPlan

    plan = TPShardPlan(2048, 16, 8192, 8, 3)
    assert plan.local_heads == 2 and plan.head_dim == 128
    assert plan.d_slice == slice(768, 1024) and plan.f_slice == slice(3072, 4096)
    with pytest.raises(ValueError, match="divide"):
        TPShardPlan(2048, 16, 8192, 3, 0)
