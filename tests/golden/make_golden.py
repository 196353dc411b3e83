"""Generate the committed golden fixtures under tests/golden/.

Run in the build container (it reads the reference checkout, which the GPU box does not have):

    python tests/golden/make_golden.py /path/to/skinny-mlx

qmm_repack_ref.npz   seeded MLX packs and the output of the reference's own
                     `repack_for_skinny` (skinny_mlx/qmm.py:96-115), executed over a numpy
                     stand-in for mlx.core; pins the nibble order every other layout derives from.
config_for_ref.json  the reference's `config_for(m, k)` (skinny_mlx/qmm.py:118-126).
qmm_small.npz        seeded config-1-style case (N=384, K=512, M in {1,3,8,16}): x (bf16 bits),
                     packs, scales/biases (bf16 bits) and the float64 MLX-semantics product.
"""

from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))

from oracle import quant  # noqa: E402

import _mlx_stub  # noqa: E402


def load_reference_module(ref_root: Path, name: str):
    _mlx_stub.install()
    sys.path.insert(0, str(ref_root))
    try:
        return importlib.import_module(name)
    finally:
        sys.path.remove(str(ref_root))


def make_repack(ref_qmm) -> None:
    rng = np.random.default_rng(1234)
    cases = {}
    for idx, (n, k) in enumerate([(8, 64), (16, 128), (64, 256)]):
        packed = rng.integers(0, 2**32, size=(n, k // 8), dtype=np.uint64).astype(np.uint32)
        out = np.asarray(ref_qmm.repack_for_skinny(packed.view(_mlx_stub.array)), dtype=np.uint32)
        cases[f"w{idx}"] = packed
        cases[f"r{idx}"] = out
    np.savez_compressed(HERE / "qmm_repack_ref.npz", **cases)


def make_config(ref_qmm) -> None:
    table = {f"{m},{k}": list(ref_qmm.config_for(m, k)) for m in (1, 2, 4, 6, 8, 12, 16)
             for k in (2048, 2560, 4096, 9728, 9216)}
    (HERE / "config_for_ref.json").write_text(json.dumps(table, indent=0, sort_keys=True) + "\n")


def make_qmm_small() -> None:
    rng = np.random.default_rng(7)
    n, k = 384, 512
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, s_bits, b_bits = quant.quantize(w)
    out = {"packed": packed, "s_bits": s_bits, "b_bits": b_bits}
    for m in (1, 3, 8, 16):
        x_bits = quant.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
        x = quant.bf16_bits_to_f32(x_bits)
        out[f"x{m}"] = x_bits
        out[f"y{m}"] = quant.qmm_ref(x, packed, s_bits, b_bits).astype(np.float32)
    np.savez_compressed(HERE / "qmm_small.npz", **out)


def main() -> None:
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <checkout of the reference skinny-mlx>")
    ref_root = Path(sys.argv[1])
    ref_qmm = load_reference_module(ref_root, "skinny_mlx.qmm")
    make_repack(ref_qmm)
    make_config(ref_qmm)
    make_qmm_small()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
