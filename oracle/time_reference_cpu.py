"""Time the reference package's own CPU path beside the numpy oracle, on the same
sample, in a container where the reference is importable (it is pure Python):

    python oracle/time_reference_cpu.py --src <checkout>/src [--layers 2]

The sample is layers of the Qwen2.5-7B-shaped 32k cache (K and V [1, 4, 32768,
128] bf16, profile "graphkv" with importance scores): the reference's
quantize_kv_layer then QuantizedKvLayer.dequantize (src/graphkv/core.py:647-772,
265-307), and the oracle's quantize_layer then dequantize_layer.  Both use the
host's threads (torch's intra-op pool for the reference; numpy's for the
oracle).  The printed ratio relates the oracle, which is what the GPU box can
time as its CPU baseline (the reference cannot be installed there), to the
reference itself.  Test infrastructure: nothing in the package imports this.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import graphkv_oracle as orc  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", required=True, help="the reference checkout's src directory")
    ap.add_argument("--layers", type=int, default=2)
    args = ap.parse_args()
    sys.path.insert(0, args.src)
    import graphkv as ref  # noqa: E402
    from graphkv import core as ref_core  # noqa: E402

    T, H, D = 32768, 4, 128
    gen = torch.Generator().manual_seed(0)
    cfg = ref.get_profile("graphkv").config
    pol = orc.POLICIES["graphkv"]
    t_ref = t_orc = 0.0
    nbytes = 0
    for _ in range(args.layers):
        k = (torch.randn(1, H, T, D, generator=gen) * torch.exp(torch.randn(H, 1, D, generator=gen))).to(torch.bfloat16)
        v = torch.randn(1, H, T, D, generator=gen).to(torch.bfloat16)
        s = torch.exp(2 * torch.randn(T, generator=gen))
        nbytes += 2 * k.numel() * k.element_size()
        t0 = time.perf_counter()
        layer = ref_core.quantize_kv_layer(k, v, cfg, importance_scores=s)
        layer.dequantize()
        t1 = time.perf_counter()
        ql = orc.quantize_layer(k.float().numpy(), v.float().numpy(), "bf16", pol, s.numpy())
        orc.dequantize_layer(ql)
        t2 = time.perf_counter()
        t_ref += t1 - t0
        t_orc += t2 - t1
    print(f"sample: {args.layers} layers of K+V [1, {H}, {T}, {D}] bf16 ({nbytes / 1e6:.0f} MB), profile graphkv")
    print(f"host threads: torch {torch.get_num_threads()}, cpu count {os.cpu_count()}")
    print(f"reference quantize_kv_layer + dequantize: {t_ref:.2f} s = {nbytes / t_ref / 1e9:.4f} GB/s")
    print(f"oracle quantize_layer + dequantize_layer: {t_orc:.2f} s = {nbytes / t_orc / 1e9:.4f} GB/s")
    print(f"oracle / reference throughput: {t_ref / t_orc:.3f}")


if __name__ == "__main__":
    main()
