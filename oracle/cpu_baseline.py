"""Timed CPU baseline: the oracle's quantized matmul in float32 on the host cores.

TEST / BASELINE INFRASTRUCTURE ONLY (see oracle/__init__.py).  MLX's CPU backend is not
installable on this image, so the CPU path of the reference (mx.quantized_matmul on mx.cpu,
skinny_mlx/qmm.py:183) is timed through this port: dequantize q * s + b per 64-group
(the same math as oracle.quant.qmm_ref) and a float32 GEMM, multithreaded through torch's CPU
BLAS.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch


def threads() -> int:
    return torch.get_num_threads()


def qmm_cpu(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor) -> torch.Tensor:
    """x [M, K] float32, packed int32 [N, K/8], scales/biases bf16 [N, K/64] (CPU tensors)."""
    n, kw = packed.shape
    words = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, dtype=torch.int64) * 4
    q = ((words.unsqueeze(-1) >> shifts) & 0xF).to(torch.float32).reshape(n, kw * 8 // 64, 64)
    w = q * scales.float().unsqueeze(-1) + biases.float().unsqueeze(-1)
    return x @ w.reshape(n, kw * 8).T


def time_stack(shapes, m: int, budget_s: float = 12.0, seed: int = 0) -> dict:
    """Run qmm_cpu over the (N, K) shapes in order (cycling) until `budget_s` of work is done.

    Weights are quantized-random packs generated on the host; only the qmm calls are timed.
    Returns bytes/s of the algorithmic traffic (packed weights + activations in/out).
    """
    gen = torch.Generator().manual_seed(seed)
    done_bytes = 0
    spent = 0.0
    calls = 0
    cache = {}
    i = 0
    while spent < budget_s and calls < 10_000:
        n, k = shapes[i % len(shapes)]
        i += 1
        key = (n, k)
        if key not in cache:
            packed = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=gen, dtype=torch.int64).to(torch.int32)
            s = (torch.rand(n, k // 64, generator=gen) * 0.01).to(torch.bfloat16)
            b = (-torch.rand(n, k // 64, generator=gen) * 0.05).to(torch.bfloat16)
            x = torch.randn(m, k, generator=gen)
            cache = {key: (packed, s, b, x)}  # keep one matrix resident at a time
        packed, s, b, x = cache[key]
        t0 = time.perf_counter()
        y = qmm_cpu(x, packed, s, b)
        spent += time.perf_counter() - t0
        del y
        done_bytes += n * k // 2 + n * (k // 64) * 4 + 2 * m * (n + k)
        calls += 1
    return {"bytes_per_s": done_bytes / spent, "seconds": spent, "calls": calls,
            "cores": threads(), "host_cpus": os.cpu_count()}


def baseline_rows(stack_shapes, budget_s: float = 16.0) -> dict:
    """CPU rows beside the B200 numbers, all through qmm_cpu on the host cores, about budget_s of
    work: config 1 (one 9728 x 2560 matrix) at M = 1, 8, 16; the config-2 stack at M = 1 and 8,
    from which the config-3 step's projection cost at M = 1 and 8 and the config-4 greedy rate
    follow (the step's 129 projections only: the mixers' recurrence and attention are left out,
    so these CPU step times are lower bounds)."""
    out = {"config1_gbs": {}}
    for m in (1, 8, 16):
        r = time_stack([(9728, 2560)], m, budget_s=budget_s * 0.08)
        out["config1_gbs"][str(m)] = round(r["bytes_per_s"] / 1e9, 3)
    stack_bytes = sum(n * k // 2 + n * (k // 64) * 4 for n, k in stack_shapes)
    steps = {}
    for m, frac in ((1, 0.3), (8, 0.46)):
        r = time_stack(stack_shapes, m, budget_s=budget_s * frac, seed=m)
        w_bytes_s = r["bytes_per_s"] * stack_bytes / (stack_bytes + 2 * m * sum(n + k for n, k in stack_shapes))
        steps[str(m)] = round(stack_bytes / w_bytes_s * 1e3, 1)
        if m == 8:
            out["config2_stack_gbs"] = round(r["bytes_per_s"] / 1e9, 3)
    out["config3_projection_ms"] = steps
    out["config3_cost_m8_vs_m1"] = round(steps["8"] / steps["1"], 3)
    out["config4_greedy_tok_s"] = round(1e3 / steps["1"], 3)
    out["cores"] = threads()
    out["host_cpus"] = os.cpu_count()
    return out


if __name__ == "__main__":
    print(time_stack([(9728, 2560)], 8, budget_s=3.0))
    _ = np
