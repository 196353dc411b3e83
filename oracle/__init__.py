"""CPU oracle for the B200 verify path.  TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU in numpy, the arithmetic of rachittshah/skinny-mlx's flat
multi-token verify path and of the MLX / mlx-lm code it calls.  Only `tests/`,
`__graft_entry__.smoke()` and `bench.py` (its `cpu_baseline` leg and `--impl reference` arm)
may import it, and only as the checker or the timed CPU baseline.  The product package
`skinny_mlx_b200` never imports it: there is no CPU fallback.

Third-party boundary.  The reference's arithmetic lives in MLX `quantized_matmul` / `quantize`
(mlx >= 0.32, README pins 0.32.1) and mlx-lm's Qwen3.5 code (mlx-lm >= 0.31), neither of which
is installed here or on the GPU box, and the reference ships no golden vectors.  Parity is
pinned two ways:
  * the packing convention is pinned against the reference's own `repack_for_skinny`
    (skinny_mlx/qmm.py:96-115), executed in this container over a numpy stand-in for
    `mlx.core` (tests/golden/make_golden.py), which also pins the reference kernel's decode
    order and affine identity (skinny_mlx/qmm.py:21-86) through `qmm_metal_order` below;
  * the decode-loop protocol is pinned by running the reference's own `greedy` and
    `speculative` loops (skinny_mlx/spec.py:98-156), its `MTPDrafter` and `PromptLookupDrafter`
    and its `HybridRollback` (skinny_mlx/rollback.py:19-73) over this oracle's float64 model
    (oracle/model.py), through numpy stand-ins for mlx.core / mlx_lm; the token streams are the
    fixture tests/golden/spec_streams.json (tests/golden/make_golden.py), which
    tests/test_spec_golden.py holds this repository's loops to on the CPU and on the GPU.
`qmm_small.npz` is oracle-generated (oracle.quant.qmm_ref), not reference output.
The MLX CPU accumulation order itself is unpinned; every float comparison therefore uses the
reference's own relative-error metric (skinny_mlx/qmm.py:185) with the tolerance BASELINE
states (1.5e-2), never bit equality.
"""
