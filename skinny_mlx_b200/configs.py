"""Model shapes of the benchmark configurations (synthetic, seeded; no checkpoints).

HYBRID_4B: the Qwen3.5-4B-like hybrid decoder the reference measures (skinny_mlx/patch.py:5-9,
bench/step_cost_curve.py): 32 layers, hidden 2560, every 4th layer full attention, the rest
Gated DeltaNet, SwiGLU MLP 9728, tied 151936-token head, 4-bit group-64 weights.

The projection shapes listed for the benchmark stack (fused as skinny_mlx/patch.py:23-27 fuses
them) are:
  attention layer: fused q/k/v 2560 -> 5120, o_proj 4096 -> 2560
  GDN layer:       fused qkv/z + b/a 2560 -> 8192 + 32, out 2048 -> 2560
  every layer:     fused gate/up 2560 -> 19456, down 9728 -> 2560
  head:            2560 -> 151936
"""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass(frozen=True)
class HybridConfig:
    name: str = "hybrid-4b"
    hidden: int = 2560
    layers: int = 32
    attn_every: int = 4           # layers 3, 7, ..., 31 are full attention
    vocab: int = 151936
    intermediate: int = 9728
    # full attention (gated query, as Qwen3.5 / Qwen3-Next): q + gate 16 x 128 x 2, k/v 4 x 128
    n_heads: int = 16
    n_kv_heads: int = 4
    head_dim: int = 128
    attn_qkv_out: int = 5120      # listed fused QKV width
    attn_o_in: int = 4096         # listed o_proj input width
    # Gated DeltaNet
    gdn_heads: int = 16
    gdn_k_dim: int = 128
    gdn_v_dim: int = 128
    gdn_qkvz_out: int = 8192
    gdn_ba_out: int = 32
    gdn_out_in: int = 2048
    conv_kernel: int = 4
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    weight_std: float = 0.02

    def is_attention(self, i: int) -> bool:
        return i % self.attn_every == self.attn_every - 1


HYBRID_4B = HybridConfig()


def hybrid_stack_shapes(cfg: HybridConfig = HYBRID_4B) -> list[tuple[str, int, int]]:
    """(name, N, K) of the 129 fused projections of one verify step, in execution order."""
    out = []
    for i in range(cfg.layers):
        if cfg.is_attention(i):
            out.append((f"layers.{i}.attn.qkv", cfg.attn_qkv_out, cfg.hidden))
            out.append((f"layers.{i}.attn.o", cfg.hidden, cfg.attn_o_in))
        else:
            out.append((f"layers.{i}.gdn.qkvz_ba", cfg.gdn_qkvz_out + cfg.gdn_ba_out, cfg.hidden))
            out.append((f"layers.{i}.gdn.out", cfg.hidden, cfg.gdn_out_in))
        out.append((f"layers.{i}.mlp.gate_up", 2 * cfg.intermediate, cfg.hidden))
        out.append((f"layers.{i}.mlp.down", cfg.hidden, cfg.intermediate))
    out.append(("lm_head", cfg.vocab, cfg.hidden))
    return out


def packed_bytes(n: int, k: int) -> int:
    """Bytes of one MLX 4-bit group-64 matrix: nibbles + bf16 scale + bf16 bias per group."""
    return n * k // 2 + n * (k // 64) * 4


@dataclass(frozen=True)
class DenseConfig:
    """64-layer dense decoder, hidden 5120, 40 q / 8 kv heads x 128,
    SwiGLU 25600, vocab 151936."""

    name: str = "dense-64l"
    hidden: int = 5120
    layers: int = 64
    n_heads: int = 40
    n_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 25600
    vocab: int = 151936
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    weight_std: float = 0.02
    extra: dict = field(default_factory=dict)


DENSE_64L = DenseConfig()
