"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference project is mounted (it is read, never
modified):

    python tests/golden/make_golden.py /path/to/reference

For each case it builds the reference's own `BaselineTransformer`
(torch_transformer_benchmark.py:248-272), loads the benchmark parameter
initialisation from `oracle.init_params` with strict=True, draws inputs with the
reference's own `generate_random_case` (:500-540) on the CPU and runs the
reference forward in fp32. It stores the inputs, the mask, the reference output
and a fingerprint of the parameters in `tests/golden/<case>.npz`.

The parameters themselves are not stored: `oracle.init_params(cfg, seed)`
regenerates them bit-for-bit from the seed (the fingerprint proves it).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import layer as oracle  # noqa: E402

# (name, B, S, d, H, F, layers, causal, padding_ratio, seed)
CASES = [
    ("cfg1", 2, 128, 256, 4, 1024, 1, False, 0.5, 1234),
    ("small_causal", 2, 64, 128, 2, 256, 1, True, 0.0, 11),
    ("odd_causal_pad", 3, 37, 64, 2, 128, 1, True, 0.5, 12),
    ("short_seq", 16, 32, 256, 4, 1024, 1, False, 0.0, 13),
    ("hd128_causal", 2, 128, 256, 2, 512, 1, True, 0.0, 14),
    ("two_layer_pad", 2, 64, 128, 4, 256, 2, False, 0.5, 15),
    ("hd8_two_layer_causal_pad", 3, 40, 32, 4, 64, 2, True, 0.5, 16),
    ("hd256_causal", 2, 48, 512, 2, 512, 1, True, 0.0, 17),
]


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch_transformer_benchmark as ref  # the unmodified reference harness

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, B, S, d, H, F, L, causal, pad, seed in CASES:
        rcfg = ref.TransformerConfig(B, S, d, H, F, L, causal)
        ocfg = oracle.TransformerConfig(B, S, d, H, F, L, causal)
        model = ref.BaselineTransformer(rcfg).eval()
        params = oracle.init_params(ocfg, seed)
        model.load_state_dict(params, strict=True)
        x, mask = ref.generate_random_case(
            rcfg, torch.device("cpu"), torch.float32, seed=seed + 1000,
            padding_ratio=pad, input_scale=1.0)
        with torch.inference_mode():
            out = model(x, mask)
        # The restatement must reproduce the reference bit-for-bit on the CPU.
        ox, om = oracle.generate_random_case(ocfg, seed + 1000, pad, 1.0)
        assert torch.equal(ox, x) and torch.equal(om, mask), name
        oout = oracle.baseline_forward(params, ocfg, x, mask)
        diff = (oout - out).abs().max().item()
        print(f"{name}: out {tuple(out.shape)} oracle-vs-reference max|d|={diff:.3e}")
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"),
            x=x.numpy(), mask=mask.numpy(), out=out.numpy(),
            cfg=np.array([B, S, d, H, F, L, int(causal)], dtype=np.int64),
            padding_ratio=np.array(pad), seed=np.array(seed),
            input_seed=np.array(seed + 1000),
            param_checksum=np.array(oracle.param_checksum(params)),
            torch_version=np.array(torch.__version__),
        )


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python make_golden.py <reference project root>  "
                         "(the directory holding torch_transformer_benchmark.py)")
    main(sys.argv[1])
