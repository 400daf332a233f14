#!/usr/bin/env python3
"""Layer-forward throughput of the B200 build, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

A step is one forward of one BASELINE config's layer through the public API
`optimized.OptimizedTransformer.forward`, on synthetic seeded data of that
shape (x ~ N(0,1), the reference's generate_random_case masks, Xavier-uniform
weights), with inputs already in HBM. The headline workload is config 5
(B=16 S=1024 d=2048 16x128 heads FFN 8192 causal), the largest that fits one
GPU. Under torchrun (one process per GPU) the config's batch is split across
the ranks (strong scaling: B/N rows each; rows never interact, so there is no
data-path collective; NCCL carries only barriers and the max-over-ranks time).

The line also carries `per_config`: every BASELINE config measured the same
way (configs whose batch does not split over N ranks are marked so), each with
device tokens/s, e2e tokens/s, the dominant kernel's roofline fraction and, at
N=1, the reference CPU layer's tokens/s on this host, plus the geometric mean
of the GPU/CPU speed-ups over the five configs (the metric's second half).

Timing: W warm-up steps (the first may capture the CUDA graph), about a second
of untimed steps, then exactly K steps, each bracketed by CUDA events on the
launching stream, with a 256 MiB write between steps to flush the 126 MB L2.
`value` = tokens processed by all ranks / max over ranks of the summed step
time. `e2e` repeats the steps through optimized.HostPipeline: each step's
input is copied in from pinned host memory and its output copied back, with
step i+1's copy-in and step i-1's copy-out overlapping step i's forward; the
time runs from the first copy-in to the last copy-out. `roofline` is the
dominant kernel of the layer, timed alone with CUDA events around CUDA-graph
replays of 20 back-to-back launches (best of 5), its DRAM traffic read from
the committed ncu summary table profiles/dram_traffic.md. `cpu_baseline` is the
reference's CPU layer (the oracle port of BaselineTransformer) on this host's
cores, rank 0 at N=1 only, on a bounded sample of batch rows.

--impl reference times that CPU layer alone on the same config and prints the
same JSON line with "impl": "reference" (rank 0 only; other ranks exit 0).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "distraction-optimizedtransformerlayer_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "layer-forward tokens/sec per config at 1/2/4/8 B200; geomean speedup vs CPU ref"

# (B, S, d_model, heads, ffn, causal, padding_ratio)
CONFIGS = {
    1: (2, 128, 256, 4, 1024, False, 0.5),
    2: (4, 512, 512, 8, 2048, True, 0.0),
    3: (8, 2048, 1024, 16, 4096, False, 0.5),
    4: (8192, 32, 256, 4, 1024, False, 0.0),
    5: (16, 1024, 2048, 16, 8192, True, 0.0),
}
FLUSH_BYTES = 256 << 20
SEED = 1234


def _describe(cid):
    B, S, d, H, F, causal, pad = CONFIGS[cid]
    mask = "causal" if causal else ("key-padding, lengths U[S/2,S]" if pad > 0 else "no mask")
    return f"cfg{cid}: B={B} S={S} d_model={d} heads={H}x{d // H} ffn={F} {mask}, 1 layer, fp32 I/O"


class _Cfg:
    def __init__(self, cid, layers):
        B, S, d, H, F, causal, pad = CONFIGS[cid]
        self.batch_size, self.seq_len, self.d_model, self.num_heads = B, S, d, H
        self.ffn_dim, self.num_layers, self.causal, self.padding_ratio = F, layers, causal, pad


def _synthetic_case(cfg, seed, rows):
    """x ~ N(0,1) and a prefix key-padding mask (lengths U[round(S(1-p)), S]),
    padded rows of x zeroed: the reference's generate_random_case
    (torch_transformer_benchmark.py:500-540) drawn on the CPU."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(rows, cfg.seq_len, cfg.d_model, generator=g)
    if cfg.padding_ratio <= 0:
        return x, None
    lo = max(1, int(round(cfg.seq_len * (1.0 - cfg.padding_ratio))))
    lengths = torch.randint(lo, cfg.seq_len + 1, (rows,), generator=g)
    mask = torch.arange(cfg.seq_len)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


def _init_model(model, seed):
    """The benchmark init: Xavier-uniform weights, U(-0.02,0.02) biases, LN 1/0."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.fill_(1.0 if name.endswith("weight") else 0.0)
            elif name.endswith("weight"):
                bound = math.sqrt(6.0 / (p.shape[0] + p.shape[1]))
                p.copy_((torch.rand(p.shape, generator=g) * 2 - 1) * bound)
            else:
                p.copy_((torch.rand(p.shape, generator=g) * 2 - 1) * 0.02)


def shard_rows(batch, world, rank, strong):
    """Batch rows [lo, hi) this rank runs. Weak scaling: every rank runs the
    config's whole batch (a global batch of batch * world). Strong scaling:
    the config's batch is split evenly across ranks (rows never interact)."""
    if not strong:
        return 0, batch
    if batch % world != 0:
        raise ValueError(f"--strong needs the batch ({batch}) divisible by the {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def settle(step, seconds, dist, device):
    """Runs step() until `seconds` have passed, deciding after every call
    together with the other ranks (an all-reduce of "keep going"), so every
    rank runs the same number of steps: a step with collectives inside (tensor
    parallel) would otherwise pair up different collectives across ranks."""
    t_end = time.perf_counter() + seconds
    while True:
        step()
        more = torch.tensor([1 if time.perf_counter() < t_end else 0], dtype=torch.int32, device=device)
        if dist is not None:
            dist.all_reduce(more, op=dist.ReduceOp.MAX)
        if not int(more.item()):
            return


def max_over_ranks(values, dist, device):
    """Elementwise max of a list of floats over all ranks (the slowest rank's
    time is the job's time)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- CPU side --

class _CpuLayer:
    """The reference's CPU layer (oracle port of BaselineTransformer) on a
    bounded sample of batch rows: one row first, then as many rows (up to
    the config's batch) as make one forward take about a second."""

    def __init__(self, cfg, target_s=1.0):
        from oracle import layer as O

        self.O = O
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.cfg = cfg
        ocfg = O.TransformerConfig(cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads,
                                   cfg.ffn_dim, cfg.num_layers, cfg.causal)
        self.params = O.init_params(ocfg, SEED)
        self.qb = 256 if cfg.seq_len > 512 else 0
        self._prepare(1)
        self.forward_s()                     # the first forward pays one-off setup
        one = self.forward_s()
        rows = int(max(1, min(cfg.batch_size, target_s / max(one, 1e-4))))
        if rows > 1:
            self._prepare(rows)

    def _prepare(self, rows):
        O, cfg = self.O, self.cfg
        self.rows = rows
        self.sub = O.TransformerConfig(rows, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim,
                                       cfg.num_layers, cfg.causal)
        x, mask = O.generate_random_case(self.sub, SEED, cfg.padding_ratio, 1.0)
        self.x, self.mask = x, (mask if cfg.padding_ratio > 0 else None)

    def forward_s(self):
        t0 = time.perf_counter_ns()
        self.O.baseline_forward(self.params, self.sub, self.x, self.mask, query_block=self.qb)
        return (time.perf_counter_ns() - t0) / 1e9

    def sample(self, med, n):
        return (f"{self.rows} of {self.cfg.batch_size} batch rows x {self.cfg.seq_len} tokens per "
                f"forward, median of {n} fp32 CPU forwards ({med * 1e3:.1f} ms each), "
                f"torch {torch.__version__} on {self.threads} threads")


def _cpu_layer_tokens_per_s(cfg, budget_s=10.0):
    layer = _CpuLayer(cfg)
    samples = []
    t_end = time.perf_counter() + budget_s
    while (time.perf_counter() < t_end and len(samples) < 200) or len(samples) < 3:
        samples.append(layer.forward_s())
    med = statistics.median(samples)
    return {"value": layer.rows * cfg.seq_len / med, "unit": "tokens/s", "cores": layer.threads,
            "kind": "port", "sample": layer.sample(med, len(samples))}


def _config_dict(cid, world, layers):
    """The workload description both arms print (identical for the same
    config, N and layer count)."""
    B, S = CONFIGS[cid][0], CONFIGS[cid][1]
    per = B // world if B % world == 0 else None
    return {"workload": _describe(cid), "global_batch": B, "batch_per_gpu": per, "seq_len": S,
            "layers": layers, "parallelism": f"dp{world} (batch rows split across GPUs)",
            "l2": "flushed between steps (256 MiB write)"}


def run_reference(args, rank, world):
    """The reference CPU layer on the arm's config (rank 0 only)."""
    if rank != 0:
        return 0
    cfg = _Cfg(args.config, args.layers)
    layer = _CpuLayer(cfg)
    for _ in range(args.warmup):
        layer.forward_s()
    per_step = [layer.forward_s() for _ in range(args.steps)]
    med = statistics.median(per_step)
    value = layer.rows * cfg.seq_len / med
    cpu = {"value": value, "unit": "tokens/s", "cores": layer.threads, "kind": "port",
           "sample": layer.sample(med, len(per_step))}
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": med * 1e3,
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": _config_dict(args.config, world, cfg.num_layers),
        "reference_run": {"device": "cpu", "step": "one fp32 CPU forward of the sample below, timed on the host",
                          "threads": layer.threads},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU side --

class _ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled while the GPU works."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = None
        self.gpu_index = gpu_index

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu_index)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self):
        if self.proc is None:
            if getattr(self, "f", None) is not None:
                self.f.close()
            os.unlink(self.path)
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _attention_pairs(cfg, mask, batch=None):
    """Allowed (query, key) pairs per head, summed over the batch rows run
    (`batch` rows without a mask; the mask's rows with one)."""
    S = cfg.seq_len
    if mask is not None:
        total = 0
        for n in (int(v) for v in mask.sum(dim=1).tolist()):
            # every query row (padded ones too) sees keys < n, and j <= i if causal
            total += (n * (n + 1) // 2 + (S - n) * n) if cfg.causal else S * n
        return total
    rows = cfg.batch_size if batch is None else batch
    return rows * (S * (S + 1) // 2 if cfg.causal else S * S)


def _layer_ops(model, x, mask, kernels, cfg):
    """The kernels of one layer forward as separate calls on preallocated
    buffers: (name, bound, algorithmic work per launch, call)."""
    from optimized.kernels import _f32_param

    B, S, d = x.shape
    T, F, H, hd = B * S, cfg.ffn_dim, cfg.num_heads, d // cfg.num_heads
    layer = model.layers[0]
    use_mask = mask is not None
    row_valid = mask.reshape(-1) if use_mask else None
    qkv_w, qkv_b = layer.attention._get_qkv_weight()
    n1 = kernels.layernorm_rows(x, _f32_param(layer.norm1, "weight"), _f32_param(layer.norm1, "bias"),
                                1e-5, out_half=True)
    qkv = kernels.linear_fp16(n1, qkv_w, qkv_b, out_half=True)
    q, k, v = qkv.view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4).unbind(0)
    ctx = kernels.attention_packed(q, k, v, cfg.causal, hd ** -0.5, key_mask=mask)
    x1 = kernels.linear_fp16(ctx, layer.attention.out_proj.half_weight(),
                             _f32_param(layer.attention.out_proj, "bias"), resid=x,
                             row_valid=row_valid, resid_mode=2 if use_mask else 1)
    n2 = kernels.layernorm_rows(x1, _f32_param(layer.norm2, "weight"), _f32_param(layer.norm2, "bias"),
                                1e-5, out_half=True)
    h = kernels.linear_fp16(n2, layer.ffn_in.half_weight(), _f32_param(layer.ffn_in, "bias"), act=1,
                            out_half=True)
    x2 = kernels.linear_fp16(h, layer.ffn_out.half_weight(), _f32_param(layer.ffn_out, "bias"), resid=x1,
                             row_valid=row_valid, resid_mode=3 if use_mask else 1)
    pairs = _attention_pairs(cfg, mask.cpu() if use_mask else None, batch=B)
    lnw2, lnb2 = _f32_param(layer.norm2, "weight"), _f32_param(layer.norm2, "bias")
    lnwf, lnbf = _f32_param(model.final_norm, "weight"), _f32_param(model.final_norm, "bias")
    out_f = torch.empty_like(x)
    # the layer's own kernel list (optimized/layers.py MyTransformerBlock)
    ln_fused = kernels.linear_ln_preferred(T, d)
    ops = [
        ("layernorm_entry", "hbm", T * d * 6,
         lambda: kernels.layernorm_rows(x, _f32_param(layer.norm1, "weight"),
                                        _f32_param(layer.norm1, "bias"), 1e-5, out_half=True, out=n1)),
        ("gemm_qkv", "tensor", 2 * T * 3 * d * d,
         lambda: kernels.linear_fp16(n1, qkv_w, qkv_b, out_half=True, out=qkv)),
        ("attention", "tensor", 4 * hd * H * pairs,
         lambda: kernels.attention_packed(q, k, v, cfg.causal, hd ** -0.5, key_mask=mask, out=ctx)),
    ]
    if ln_fused:
        ops.append(("gemm_out_proj_ln", "tensor", 2 * T * d * d,
                    lambda: kernels.linear_ln(ctx, layer.attention.out_proj.half_weight(),
                                              _f32_param(layer.attention.out_proj, "bias"), lnw2, lnb2, 1e-5,
                                              resid=x, row_valid=row_valid, resid_mode=2 if use_mask else 1,
                                              out=x1, normed=n2)))
    else:
        ops += [
            ("gemm_out_proj_residual", "tensor", 2 * T * d * d,
             lambda: kernels.linear_fp16(ctx, layer.attention.out_proj.half_weight(),
                                         _f32_param(layer.attention.out_proj, "bias"), resid=x,
                                         row_valid=row_valid, resid_mode=2 if use_mask else 1, out=x1)),
            ("layernorm_2", "hbm", T * d * 6,
             lambda: kernels.layernorm_rows(x1, lnw2, lnb2, 1e-5, out_half=True, out=n2)),
        ]
    if kernels.ffn_preferred(T, d, F):
        ops.append(("ffn_fused", "tensor", 4 * T * d * F,
                    lambda: kernels.ffn(n2, layer.ffn_in.half_weight(), _f32_param(layer.ffn_in, "bias"),
                                        layer.ffn_out.half_weight(), _f32_param(layer.ffn_out, "bias"),
                                        lnwf, lnbf, 1e-5, resid=x1, row_valid=row_valid,
                                        resid_mode=3 if use_mask else 1, normed_row_valid=row_valid,
                                        normed=out_f)))
        return ops
    ops.append(("gemm_ffn_in_gelu", "tensor", 2 * T * d * F,
                lambda: kernels.linear_fp16(n2, layer.ffn_in.half_weight(), _f32_param(layer.ffn_in, "bias"),
                                            act=1, out_half=True, out=h)))
    if ln_fused:
        ops.append(("gemm_ffn_out_ln", "tensor", 2 * T * F * d,
                    lambda: kernels.linear_ln(h, layer.ffn_out.half_weight(), _f32_param(layer.ffn_out, "bias"),
                                              lnwf, lnbf, 1e-5, resid=x1, row_valid=row_valid,
                                              resid_mode=3 if use_mask else 1, store_x=False, normed_half=False,
                                              normed_row_valid=row_valid, normed=out_f)))
    else:
        ops += [
            ("gemm_ffn_out_residual", "tensor", 2 * T * F * d,
             lambda: kernels.linear_fp16(h, layer.ffn_out.half_weight(), _f32_param(layer.ffn_out, "bias"),
                                         resid=x1, row_valid=row_valid, resid_mode=3 if use_mask else 1,
                                         out=x2)),
            ("layernorm_final", "hbm", T * d * 8,
             lambda: kernels.layernorm_rows(x2, lnwf, lnbf, 1e-5, row_valid=row_valid)),
        ]
    return ops


def _op_breakdown(model, x, mask, reps, kernels, cfg):
    """Each kernel of one layer forward timed alone: `reps` back-to-back
    launches captured in a CUDA graph (no host launch cost in the timing),
    replayed between CUDA events on the launching stream, best of 5."""
    ops = _layer_ops(model, x, mask, kernels, cfg)
    out = []
    for name, bound, work, fn in ops:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                fn()
        stream = torch.cuda.current_stream()
        best = float("inf")
        for _ in range(5):
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
            best = min(best, ev0.elapsed_time(ev1) / reps)
        graph.reset()
        out.append({"kernel": name, "bound": bound, "work": work, "ms": best})
    return out


def _allreduce_roofline(dist, dev, numel, world, reps=20):
    """One layer's all-reduce (an fp32 [T, d_model] partial sum) timed alone:
    bus bandwidth 2 (P-1)/P * bytes / time against the measured 8-rank
    NVLink all-reduce bus bandwidth of this pool (725 GB/s at 1 GiB)."""
    buf = torch.ones(numel, dtype=torch.float32, device=dev)
    for _ in range(3):
        dist.all_reduce(buf)
    torch.cuda.synchronize(dev)
    dist.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(reps):
        dist.all_reduce(buf)
    ev1.record()
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / reps
    ms = max_over_ranks([ms], dist, dev)[0]
    achieved = 2.0 * (world - 1) / world * numel * 4 / (ms / 1e3) / 1e9
    return {"kernel": "nccl_allreduce_fp32_partials", "bound": "nvlink", "achieved": achieved,
            "peak": 725.0, "unit": "GB/s", "frac": achieved / 725.0,
            "peak_source": "measured 8-rank all-reduce bus bandwidth of this pool", "traffic": None,
            "ms_per_allreduce": ms, "allreduces_per_step": 2}


def _fused_allreduce_roofline(model, dist, dev, T, d, world, reps=20):
    """One dotl_allreduce_ln launch (the layer's out_proj reduction + add +
    LayerNorm) timed alone on the group's own buffers. NVLink bytes each GPU
    sends per launch: one-shot, every peer reads its whole fp32 partial sum,
    (P-1) T d 4; push, peers read 1/P of it from each rank and each rank
    stores its 1/P of x_new (fp32) and normed (fp16) into every peer,
    (P-1)/P T d (4 + 6); push with the GEMMs scattering their tiles to the
    row owners, only the stores, (P-1)/P T d 6. Against the measured 770 GB/s per direction of a peer
    copy on this pool."""
    pg = model.peer
    w = model.w
    x = pg.view("xa", T)
    local = model.scatter is not False and pg.scatter_ok(T)

    def once():
        pg.allreduce_ln(x, w["layers.0.bo_full"], w["layers.0.norm2.weight"], w["layers.0.norm2.bias"],
                        model.eps, "xb", "n16", T, from_owners=local)

    for _ in range(3):
        once()
    torch.cuda.synchronize(dev)
    dist.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(reps):
        once()
    ev1.record()
    torch.cuda.synchronize(dev)
    ms = max_over_ranks([ev0.elapsed_time(ev1) / reps], dist, dev)[0]
    if local:
        nbytes = (world - 1) / world * T * d * 6    # the partial sums crossed inside the GEMMs
    elif pg.push:
        nbytes = (world - 1) / world * T * d * 10
    else:
        nbytes = (world - 1) * T * d * 4
    achieved = nbytes / (ms / 1e3) / 1e9
    kind = "push_from_owner_slots" if local else ("push" if pg.push else "oneshot")
    return {"kernel": "allreduce_ln_" + kind, "bound": "nvlink",
            "achieved": achieved, "peak": 770.0, "unit": "GB/s", "frac": achieved / 770.0,
            "peak_source": "measured peer copy of this pool, per direction per GPU", "traffic": None,
            "nvlink_bytes_per_gpu": nbytes, "ms_per_launch": ms, "launches_per_step": 2}


def _traffic_table():
    """DRAM bytes (read + write) per launch of each layer kernel, from the
    committed ncu summaries: the rows `| cfg | kernel | read | write | ... |`
    of profiles/dram_traffic.md (one ncu capture each; the file gives the
    commands)."""
    path = os.path.join(REPO, "profiles", "dram_traffic.md")
    table = {}
    try:
        with open(path) as f:
            for line in f:
                cells = [c.strip() for c in line.strip().strip("|").split("|")]
                if len(cells) >= 4 and cells[0].isdigit():
                    try:
                        table[(int(cells[0]), cells[1].strip("`"))] = int(cells[2].replace(",", "")) + \
                            int(cells[3].replace(",", ""))
                    except ValueError:
                        continue
    except OSError:
        pass
    return table


def _init_dist(world, dev):
    if world <= 1:
        return None
    import datetime

    import torch.distributed as dist
    # NCCL prints a version banner on stdout when the communicator comes up
    # (eagerly here, device_id is bound): send it to stderr, so rank 0's
    # stdout carries only the JSON line.
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        dist.barrier()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    return dist


def _measure(cid, args, kernels, dist, dev, rank, world, steps, cpu_budget_s):
    """One config measured the bench's way. Returns a dict (rank 0's view,
    times already maxed over ranks), or None where the config's batch does not
    split over the ranks."""
    from optimized import HostPipeline, OptimizedTransformer

    cfg = _Cfg(cid, args.layers)
    strong = world > 1 and not args.weak
    if strong and cfg.batch_size % world != 0:
        return None
    model = OptimizedTransformer(cfg)
    _init_model(model, SEED)
    model = model.to(dev).eval()
    lo, hi = shard_rows(cfg.batch_size, world, rank, strong)
    if strong or world == 1:
        x_all, mask_all = _synthetic_case(cfg, SEED, cfg.batch_size)
        x_cpu = x_all[lo:hi].contiguous()
        mask_cpu = mask_all[lo:hi].contiguous() if mask_all is not None else None
    else:
        x_cpu, mask_cpu = _synthetic_case(cfg, SEED + 17 * rank, cfg.batch_size)
    x = x_cpu.to(dev)
    mask = mask_cpu.to(dev) if mask_cpu is not None else None
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    tokens_per_rank = (hi - lo) * cfg.seq_len
    job_tokens = world * tokens_per_rank
    stream = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    sampler = _ClockSampler(dev.index)
    sampler.start()
    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x, mask)
        # a wait that ran out would make every later step wait out its limit too
        word = kernels.device_error(clear=False)
        if word:
            raise RuntimeError(f"device error word {word:#x} after the warm-up steps (config {cid})")
        # about a second of untimed steps so the clocks settle before timing
        settle(lambda: model(x, mask), args.settle, dist, dev)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier()
        torch.cuda.nvtx.range_push("timed_steps")    # the launch-list profile selects this range
        for i in range(steps):
            flush.zero_()
            starts[i].record(stream)
            model(x, mask)
            ends[i].record(stream)
        torch.cuda.nvtx.range_pop()
        barrier()
    clocks = sampler.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))

    # e2e: pinned host input -> forward -> pinned host output, every step,
    # through optimized.HostPipeline (copy-in of step i+1 and copy-out of step
    # i-1 overlap step i's forward; every step still copies its own input in
    # and its output out). The L2 flush runs on the compute stream before each
    # forward and counts toward the time.
    x_host = x_cpu.pin_memory()
    mask_host = mask_cpu.pin_memory() if mask_cpu is not None else None
    out_hosts = [torch.empty(x_cpu.shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    pipe = HostPipeline(model, dev, before_compute=flush.zero_)

    def masks(n):
        return [mask_host] * n if mask_host is not None else None

    with torch.inference_mode():
        # W warm-up steps, then about a second more: the first pipelined
        # copies out of freshly pinned buffers run well below steady state
        pipe.run([x_host] * args.warmup, masks(args.warmup), [out_hosts[i & 1] for i in range(args.warmup)])
        settle(lambda: pipe.run([x_host] * 8, masks(8), [out_hosts[i & 1] for i in range(8)]),
               args.settle, dist, dev)
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        barrier()
        pipe.run([x_host] * steps, masks(steps), [out_hosts[i & 1] for i in range(steps)],
                 start_event=e_start, end_event=e_end)
        barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    h2d = x_cpu.numel() * 4 + (mask_cpu.numel() if mask_cpu is not None else 0)
    d2h = x_cpu.numel() * 4
    link_in_ms, link_out_ms = _pcie_duplex_ms(x_host, out_hosts[0], dev)
    total_ms, e2e_ms, link_in_ms, link_out_ms = max_over_ranks([total_ms, e2e_ms, link_in_ms, link_out_ms], dist, dev)
    link_ms = max(link_in_ms, link_out_ms)

    res = {"config": cid, "tokens_per_rank": tokens_per_rank, "job_tokens": job_tokens,
           "ms_per_step": total_ms / steps, "value": job_tokens * steps / (total_ms / 1e3),
           "e2e": {"value": job_tokens * steps / (e2e_ms / 1e3), "unit": "tokens/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                   # the copies alone, both directions at once: the e2e ceiling
                   "pcie": {"h2d_gbs": x_host.numel() * 4 / link_in_ms / 1e6,
                            "d2h_gbs": d2h / link_out_ms / 1e6, "concurrent": True,
                            "bound_value": job_tokens / (link_ms / 1e3),
                            "frac": (link_ms * steps) / e2e_ms}},
           "clocks": clocks, "batch_per_gpu": hi - lo, "strong": strong,
           "cuda_graph": len(model._graphs) > 0,
           "l2": "inputs " + ("larger" if x.numel() * 4 > 126 * 2 ** 20 else "smaller") + " than L2"}
    if rank == 0:
        with torch.inference_mode():
            breakdown = _op_breakdown(model, x, mask, 20, kernels, cfg)
        res["launches_per_step"] = 1 + (len(breakdown) - 1) * cfg.num_layers
        hbm, tflops, _tsus, peak_kind = _peaks()
        dom = max(breakdown, key=lambda r: r["ms"])
        if dom["bound"] == "tensor":
            achieved, peak, unit = dom["work"] / (dom["ms"] / 1e3) / 1e12, tflops, "TFLOP/s"
        else:
            achieved, peak, unit = dom["work"] / (dom["ms"] / 1e3) / 1e9, hbm, "GB/s"
        res["roofline"] = {
            "kernel": dom["kernel"], "bound": dom["bound"], "achieved": achieved, "peak": peak, "unit": unit,
            "frac": achieved / peak,
            "peak_source": f"{peak_kind} ({'bf16_tflops burst' if unit == 'TFLOP/s' else 'hbm_gbs'})",
            "work_per_launch": dom["work"], "launch_us": dom["ms"] * 1e3,
            "traffic": _traffic_table().get((cid, dom["kernel"]))}
        res["kernels"] = [{"kernel": r["kernel"], "us": round(r["ms"] * 1e3, 2),
                           ("tflops" if r["bound"] == "tensor" else "gbs"):
                               round(r["work"] / (r["ms"] / 1e3) / (1e12 if r["bound"] == "tensor" else 1e9), 1)}
                          for r in breakdown]
        if world == 1 and cpu_budget_s > 0:
            res["cpu_baseline"] = _cpu_layer_tokens_per_s(cfg, budget_s=cpu_budget_s)
    word = kernels.device_error(clear=True)
    if word:
        raise RuntimeError(f"device error word {word:#x} after config {cid}")
    model.release_graphs()
    del model, x, mask, flush, pipe, x_host, out_hosts
    torch.cuda.empty_cache()
    return res


def _pcie_duplex_ms(x_host, out_host, dev, reps=5):
    """Best-of-reps times (ms) of one host->device copy of x_host and one
    device->host copy into out_host (both pinned, the e2e step's buffers),
    issued together on two streams as the e2e pipeline overlaps them: the
    link's ceiling for the e2e number."""
    d_in = torch.empty(x_host.shape, dtype=x_host.dtype, device=dev)
    d_out = torch.zeros(out_host.shape, dtype=out_host.dtype, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    best_in = best_out = float("inf")
    for _ in range(reps):
        torch.cuda.synchronize(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        with torch.cuda.stream(s_in):
            ev[0].record(s_in)
            d_in.copy_(x_host, non_blocking=True)
            ev[1].record(s_in)
        with torch.cuda.stream(s_out):
            ev[2].record(s_out)
            out_host.copy_(d_out, non_blocking=True)
            ev[3].record(s_out)
        torch.cuda.synchronize(dev)
        best_in = min(best_in, ev[0].elapsed_time(ev[1]))
        best_out = min(best_out, ev[2].elapsed_time(ev[3]))
    return best_in, best_out


def _per_config_entry(r):
    e = {"value": r["value"], "unit": "tokens/s", "ms_per_step": r["ms_per_step"],
         "batch_per_gpu": r["batch_per_gpu"], "e2e": r["e2e"]["value"],
         "e2e_pcie_frac": round(r["e2e"]["pcie"]["frac"], 3), "cuda_graph": r["cuda_graph"],
         "sm_mhz": r["clocks"].get("sm_mhz"), "throttle": r["clocks"].get("reasons")}
    if "roofline" in r:
        rf = r["roofline"]
        e["roofline"] = {"kernel": rf["kernel"], "bound": rf["bound"], "frac": round(rf["frac"], 4),
                         "achieved": round(rf["achieved"], 1), "unit": rf["unit"]}
    if "cpu_baseline" in r:
        e["cpu_baseline"] = r["cpu_baseline"]
        e["speedup_vs_cpu"] = r["value"] / r["cpu_baseline"]["value"]
        e["e2e_speedup_vs_cpu"] = r["e2e"]["value"] / r["cpu_baseline"]["value"]
    return e


def run_ours(args, rank, world, local_rank):
    import kernel_ext
    from optimized import config as oconfig

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = _init_dist(world, dev)
    kernels = kernel_ext.get_kernels()
    if kernels is None:
        raise RuntimeError(f"libdotl failed to load: {kernel_ext.load_error()}")
    if args.no_graph:
        oconfig.CUDA_GRAPH = "off"
    if args.profile_kernel:
        return _profile_kernel(args, kernels, dev)
    if args.tp:
        return run_tp(args, rank, world, dev, dist, kernels)

    cpu_budget = 0.0 if args.no_cpu_baseline else args.cpu_budget
    head = _measure(args.config, args, kernels, dist, dev, rank, world, args.steps, cpu_budget)
    if head is None:
        raise SystemExit(f"config {args.config}'s batch ({CONFIGS[args.config][0]}) does not split over "
                         f"{world} ranks; use --weak or another --config")
    per_config = {}
    for cid in args.configs:
        r = head if cid == args.config else _measure(cid, args, kernels, dist, dev, rank, world,
                                                      max(3, min(args.steps, args.per_config_steps)), cpu_budget)
        per_config[str(cid)] = (_per_config_entry(r) if r is not None else
                                {"skipped": f"batch {CONFIGS[cid][0]} does not split over {world} GPUs"})

    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            # the run's mode (the config's batch split over the ranks unless
            # --weak), the same label at every N of a scaling sweep
            "higher_is_better": True, "scaling": "weak" if args.weak else "strong",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": _config_dict(args.config, world, args.layers),
            "impl_notes": {"cuda_graph": head["cuda_graph"], "l2": head["l2"],
                           "arithmetic": "fp16 tensor-core operands, fp32 accumulate, fp32 I/O and LN"},
            "clocks": head["clocks"],
            "e2e": head["e2e"],
            "gpu_launches": head["launches_per_step"] * args.steps,
            "roofline": head["roofline"],
            "kernels": head["kernels"],
        }
        if "cpu_baseline" in head:
            line["cpu_baseline"] = head["cpu_baseline"]
        line["per_config"] = per_config
        sp = [v["speedup_vs_cpu"] for v in per_config.values() if "speedup_vs_cpu" in v]
        sp_e2e = [v["e2e_speedup_vs_cpu"] for v in per_config.values() if "e2e_speedup_vs_cpu" in v]
        if sp:
            line["geomean_vs_cpu"] = {
                "device": math.exp(sum(math.log(v) for v in sp) / len(sp)),
                "e2e": math.exp(sum(math.log(v) for v in sp_e2e) / len(sp_e2e)),
                "configs": [int(c) for c, v in per_config.items() if "speedup_vs_cpu" in v]}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_tp(args, rank, world, dev, dist, kernels):
    """Config 5's tensor-parallel layer over all ranks (--tp): one global
    batch per step, heads and FFN columns sharded."""
    from optimized import HostPipeline, OptimizedTransformer
    from optimized.tensor_parallel import TensorParallelTransformer

    if world < 2:
        raise SystemExit("--tp needs torchrun with at least 2 ranks")
    cfg = _Cfg(args.config, args.layers)
    full = OptimizedTransformer(cfg)
    _init_model(full, SEED)
    state = {k: v.detach() for k, v in full.state_dict().items()}
    model = TensorParallelTransformer(cfg, state, device=dev,
                                      fused=None if args.tp_impl == "auto" else args.tp_impl == "fused",
                                      push=not args.tp_oneshot,
                                      scatter=False if args.tp_no_scatter else None, error_check="deferred")
    x_cpu, mask_cpu = _synthetic_case(cfg, SEED, cfg.batch_size)
    x = x_cpu.to(dev)
    mask = mask_cpu.to(dev) if mask_cpu is not None else None
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    job_tokens = cfg.batch_size * cfg.seq_len
    stream = torch.cuda.current_stream(dev)

    def barrier():
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)

    sampler = _ClockSampler(dev.index)
    sampler.start()
    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x, mask)
        torch.cuda.synchronize(dev)
        model.check()
        settle(lambda: model(x, mask), args.settle, dist, dev)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            model(x, mask)
            ends[i].record(stream)
        barrier()
        model.check()
    clocks = sampler.stop()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    x_host = x_cpu.pin_memory()
    mask_host = mask_cpu.pin_memory() if mask_cpu is not None else None
    out_hosts = [torch.empty(x_cpu.shape, dtype=torch.float32).pin_memory() for _ in range(2)]
    pipe = HostPipeline(model, dev, before_compute=flush.zero_)

    def masks(n):
        return [mask_host] * n if mask_host is not None else None

    with torch.inference_mode():
        pipe.run([x_host] * args.warmup, masks(args.warmup), [out_hosts[i & 1] for i in range(args.warmup)])
        settle(lambda: pipe.run([x_host] * 8, masks(8), [out_hosts[i & 1] for i in range(8)]),
               args.settle, dist, dev)
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        barrier()
        pipe.run([x_host] * args.steps, masks(args.steps), [out_hosts[i & 1] for i in range(args.steps)],
                 start_event=e_start, end_event=e_end)
        barrier()
        model.check()
    e2e_ms = e_start.elapsed_time(e_end)
    total_ms, e2e_ms = max_over_ranks([total_ms, e2e_ms], dist, dev)
    if model.fused:
        allreduce = _fused_allreduce_roofline(model, dist, dev, x.numel() // cfg.d_model, cfg.d_model, world)
    else:
        allreduce = _allreduce_roofline(dist, dev, x.numel(), world)
    word = kernels.device_error(clear=True)
    if word:
        raise RuntimeError(f"device error word {word:#x} after the timed run")
    if rank == 0:
        line = {
            "metric": METRIC, "value": job_tokens * args.steps / (total_ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": dict(_config_dict(args.config, world, cfg.num_layers),
                           parallelism=f"tp{world} (heads and FFN columns split across GPUs)"),
            "impl_notes": {
                "cuda_graph": False, "arithmetic": "fp16 tensor-core operands, fp32 accumulate, fp32 partial sums",
                "allreduce": ("dotl_allreduce_ln over peer memory, " + ("push" if model.peer.push else "one-shot")
                              + (", GEMM tiles scattered to the row owners by dotl_linear_peer"
                                 if model.scatter is not False and model.peer.scatter_ok(x.numel() // cfg.d_model)
                                 else ""))
                if model.fused else "NCCL all_reduce + LayerNorm kernel"},
            "clocks": clocks,
            "e2e": {"value": job_tokens * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_cpu.numel() * 4 + (mask_cpu.numel() if mask_cpu is not None else 0),
                    "d2h_bytes_per_step": x_cpu.numel() * 4},
            "gpu_launches": (1 + 7 * cfg.num_layers) * args.steps,
            "roofline": allreduce,
        }
        print(json.dumps(line), flush=True)
    model.close()   # collective: unmaps and frees the peer buffers
    dist.barrier()
    dist.destroy_process_group()
    return 0


def _profile_allreduce_ln(args, kernels, dev):
    """dotl_allreduce_ln as one rank of config C's tensor-parallel layer runs it
    (push mode, fp16 normed rows), 3 times inside "dotl_profile", with the
    --profile-ranks ranks stood in for by local buffers: rank P-1 reduces its
    T/P rows from P fp32 partial sums, adds bias and residual, normalises, and
    writes x_new and normed into all P ranks' buffers. The peers' flags are
    preset far ahead, so no wait ever spins."""
    B, S, d = CONFIGS[args.config][:3]
    T, P = B * S, args.profile_ranks
    rank = P - 1
    g = torch.Generator(device=dev).manual_seed(SEED)
    parts = [torch.randn(T, d, device=dev, generator=g) for _ in range(P)]
    x = torch.randn(T, d, device=dev, generator=g)
    bias, w, b = (torch.randn(d, device=dev, generator=g) * 0.1 for _ in range(3))
    x_new = [torch.empty(T, d, device=dev) for _ in range(P)]
    normed = [torch.empty(T, d, device=dev, dtype=torch.float16) for _ in range(P)]
    blocks = kernels.peer_blocks()
    words = kernels.peer_signal_bytes(blocks) // 4
    sig = [torch.zeros(words, dtype=torch.int32, device=dev) for _ in range(P)]
    sig[rank][blocks:] = 1 << 30
    torch.cuda.synchronize(dev)
    torch.cuda.nvtx.range_push("dotl_profile")
    for _ in range(3):
        kernels.allreduce_ln(P, rank, [t.data_ptr() for t in parts], [t.data_ptr() for t in sig],
                             [t.data_ptr() for t in x_new], [t.data_ptr() for t in normed], True, True,
                             x, bias, w, b, 1e-5, None, None, T, d, blocks, 2000)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    if kernels.device_error(clear=True):
        raise SystemExit("allreduce_ln profile: the device error word is set")
    print(f"profiled allreduce_ln x3: rank {rank} of {P}, {T // P} of {T} rows, d_model {d}")
    return 0


def _profile_kernel(args, kernels, dev):
    """Runs one kernel of the layer 3 times inside the NVTX range
    "dotl_profile" (for ncu --nvtx --nvtx-include dotl_profile/), nothing else
    timed. --profile-shape B,S,d,H,F replaces the config's shape (causal)."""
    from optimized import OptimizedTransformer

    if args.profile_kernel == "allreduce_ln":
        return _profile_allreduce_ln(args, kernels, dev)
    cfg = _Cfg(args.config, args.layers)
    if args.profile_shape:
        B, S, d, H, F = (int(v) for v in args.profile_shape.split(","))
        cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim = B, S, d, H, F
        cfg.causal, cfg.padding_ratio = True, 0.0
    model = OptimizedTransformer(cfg)
    _init_model(model, SEED)
    model = model.to(dev).eval()
    x_cpu, mask_cpu = _synthetic_case(cfg, SEED, cfg.batch_size)
    x = x_cpu.to(dev)
    mask = mask_cpu.to(dev) if mask_cpu is not None else None
    with torch.inference_mode():
        ops = {name: fn for name, _b, _w, fn in _layer_ops(model, x, mask, kernels, cfg)}
        if args.profile_kernel not in ops:
            raise SystemExit(f"--profile-kernel must be one of {sorted(ops)}")
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("dotl_profile")
        for _ in range(3):
            ops[args.profile_kernel]()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
    shape = (f"B={cfg.batch_size} S={cfg.seq_len} d_model={cfg.d_model} heads={cfg.num_heads} "
             f"ffn={cfg.ffn_dim} causal" if args.profile_shape else _describe(args.config))
    print(f"profiled {args.profile_kernel} x3 on {shape}")
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[1])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=5, choices=sorted(CONFIGS),
                    help="the headline workload (default: config 5, the largest on one GPU)")
    ap.add_argument("--configs", default="1,2,3,4,5",
                    help="configs measured for per_config ('none' for the headline only)")
    ap.add_argument("--per-config-steps", type=int, default=30,
                    help="timed steps of each per_config entry other than the headline")
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-graph", action="store_true", help="time the eager path (no CUDA graph)")
    ap.add_argument("--tp", action="store_true",
                    help="tensor parallel across all ranks (heads and FFN columns sharded, two reductions "
                         "per layer); one global batch per step")
    ap.add_argument("--tp-impl", choices=("auto", "fused", "nccl"), default="auto",
                    help="--tp: each all-reduce + add + LayerNorm as one peer-memory kernel, or NCCL + LN "
                         "(auto: the model's default, fused at 2 ranks)")
    ap.add_argument("--tp-oneshot", action="store_true",
                    help="--tp fused: one-shot mode (every rank reduces every row)")
    ap.add_argument("--tp-no-scatter", action="store_true",
                    help="--tp fused push: row-parallel GEMMs write locally (no scatter to the row owners)")
    ap.add_argument("--weak", action="store_true",
                    help="every rank runs the config's whole batch (weak scaling) instead of splitting it")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=6.0,
                    help="seconds of CPU reference forwards per config for cpu_baseline (N=1, rank 0)")
    ap.add_argument("--settle", type=float, default=1.0, help="seconds of untimed steps before timing")
    ap.add_argument("--profile-kernel", default=None,
                    help="run only this kernel of the layer 3x in an NVTX range (for ncu); "
                         "'allreduce_ln' runs one rank's fused tensor-parallel reduction")
    ap.add_argument("--profile-shape", default=None,
                    help="B,S,d_model,heads,ffn: profile the kernel on this causal shape instead of the config")
    ap.add_argument("--profile-ranks", type=int, default=8,
                    help="ranks emulated by --profile-kernel allreduce_ln")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    args.configs = [] if args.configs == "none" else [int(c) for c in args.configs.split(",")]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world != args.gpus:
        print(f"[bench] note: --gpus {args.gpus} but WORLD_SIZE={world}; using {world}", file=sys.stderr)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    raise SystemExit(main())
