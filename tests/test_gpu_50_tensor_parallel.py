"""Tensor-parallel layer on 2 GPUs against the oracle (gpu), with each
all-reduce + add + LayerNorm either fused over peer memory (push mode, the
row-parallel GEMMs scattering their tiles to the row owners where the rows
allow it, or not; one-shot mode) or as NCCL all-reduce + the LayerNorm kernel.

Runs only where at least two GPUs are visible; the CPU decomposition test in
test_tensor_parallel_gloo.py covers the sharding everywhere, and
test_gpu_55_allreduce_ln.py the fused kernel's arithmetic on one GPU."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path, case, mode):
    import sys
    import datetime

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "distraction-optimizedtransformerlayer_b200"))
    import torch.distributed as dist
    from oracle import layer as O
    from optimized.tensor_parallel import TensorParallelTransformer

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        B, S, d, H, Fd, L, causal, pad = case
        cfg = O.TransformerConfig(B, S, d, H, Fd, L, causal)
        params = O.init_params(cfg, 21)
        x, mask = O.generate_random_case(cfg, 22, pad, 1.0)
        tp = TensorParallelTransformer(cfg, params, fused=mode != "nccl", push=mode.startswith("push"),
                                       scatter=False if mode == "push_noscatter" else None)
        try:
            with torch.inference_mode():
                out = tp(x.cuda(), mask.cuda() if pad > 0 else None).cpu()
                out2 = tp(x.cuda(), mask.cuda() if pad > 0 else None).cpu()
            torch.cuda.synchronize()
            word = tp._kernels().device_error(clear=True)
        finally:
            tp.close()
        torch.save({"out": out, "out2": out2, "word": word}, f"{path}.{rank}")
        if rank == 0:
            ref = O.baseline_forward(params, cfg, x, mask if pad > 0 else None, query_block=256)
            torch.save({"ref": ref}, path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["push", "push_noscatter", "oneshot", "nccl"])
@pytest.mark.parametrize("case", [(2, 256, 512, 8, 1024, 1, True, 0.0),
                                  (2, 192, 256, 4, 512, 2, False, 0.5),
                                  (1, 512, 1024, 8, 2048, 1, True, 0.0)])
def test_tp2_matches_oracle(kernels, tmp_path, case, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    from oracle import layer as O

    path = str(tmp_path / "tp.pt")
    mp.start_processes(_worker, args=(2, _free_port(), path, case, mode), nprocs=2, start_method="spawn",
                       join=True)
    ref = torch.load(path)["ref"]
    r0, r1 = torch.load(f"{path}.0"), torch.load(f"{path}.1")
    assert r0["word"] == 0 and r1["word"] == 0
    assert torch.equal(r0["out"], r0["out2"])
    assert torch.equal(r0["out"], r1["out"]), "every rank must hold the same bits"
    res = O.compare_outputs(ref, r0["out"])
    assert res.passed, (res.failed_elements, res.max_abs_error)
