"""Generate the committed golden fixtures under tests/golden/.

Run in the build container (it reads the reference checkout, which the GPU box does not have):

    python tests/golden/make_golden.py /path/to/skinny-mlx

qmm_repack_ref.npz   seeded MLX packs and the output of the reference's own
                     `repack_for_skinny` (skinny_mlx/qmm.py:96-115), executed over a numpy
                     stand-in for mlx.core; pins the nibble order every other layout derives from.
config_for_ref.json  the reference's `config_for(m, k)` (skinny_mlx/qmm.py:118-126).
qmm_small.npz        ORACLE-GENERATED (not reference output): a seeded config-1-style case
                     (N=384, K=512, M in {1,3,8,16}): x (bf16 bits), packs, scales/biases (bf16
                     bits) and oracle.quant.qmm_ref's float64 MLX-semantics product.
spec_streams.json    token streams of the reference's OWN decode loops -- skinny_mlx/spec.py
                     `greedy` and `speculative` with skinny_mlx/rollback.py `HybridRollback`, its
                     `MTPDrafter` and `PromptLookupDrafter`, and a scripted drafter whose
                     acceptance varies -- executed over the float64 oracle model (oracle/model.py)
                     built from the seeded small hybrid model (skinny_mlx_b200.model.SMALL, seed 0,
                     weights drawn on the CPU generator) and its MTP head (seed 13), through numpy
                     stand-ins for mlx.core and mlx_lm (_mlx_stub.py).  Each stream comes with the
                     oracle's per-token (top1 - top2, top1) logit gaps for the near-tie check.
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


SPEC_PROMPT_SEED, SPEC_PROMPT_LEN, SPEC_TOKENS = 5, 24, 32


class ScriptDrafter:
    """Drafts the known greedy continuation `ref`; proposal i of draft call c is replaced by a
    wrong token when (c + i) % bad == 0, so verify steps accept a varying prefix (the drafter
    protocol of skinny_mlx/spec.py: begin / draft / update)."""

    def __init__(self, ref, bad, vocab, array):
        self.ref, self.bad, self.vocab, self.array, self.calls = ref, bad, vocab, array, 0

    def begin(self, prompt, h, first):
        self.pos = 1

    def draft(self, k):
        self.calls += 1
        toks = []
        for i in range(k):
            j = self.pos + i
            t = self.ref[j] if j < len(self.ref) else 0
            if (self.calls + i) % self.bad == 0:
                t = (t + 1) % self.vocab
            toks.append(t)
        return self.array(toks, dtype=np.int32)

    def update(self, h_kept, new_tokens):
        self.pos += len(new_tokens)


class GapTrace:
    """Wraps the model for the reference's `greedy`: records (top1 - top2, top1) of the last row
    of every call's logits (call j chooses token j)."""

    def __init__(self, model):
        self.model, self.gaps = model, []

    def __getattr__(self, name):
        return getattr(self.model, name)

    def __call__(self, inputs, cache=None):
        from oracle.checks import top2_gap

        logits = self.model(inputs, cache)
        self.gaps.append(top2_gap(np.asarray(logits)[0, -1]))
        return logits


def make_spec_streams(ref_root: Path) -> None:
    import torch

    from oracle import model as om
    from skinny_mlx_b200.model import SMALL, HybridModel
    from skinny_mlx_b200.mtp import MTPHead

    core = _mlx_stub.install(quantized_matmul=om.quantized_matmul)
    _mlx_stub.install_mlx_lm(om, om.gated_delta_update)
    sys.path.insert(0, str(ref_root))
    try:
        spec = importlib.import_module("skinny_mlx.spec")
    finally:
        sys.path.remove(str(ref_root))
    torch.manual_seed(0)
    tm = HybridModel(SMALL, seed=0, device="cpu")
    th = MTPHead(tm, seed=13)
    q35 = sys.modules["mlx_lm.models.qwen3_5"]
    model = om.HybridModel(om.weights_from_torch(tm), gdu=q35)
    head = om.MTPHead(om.head_weights_from_torch(th))
    prompt = [int(x) for x in np.random.default_rng(SPEC_PROMPT_SEED).integers(0, SMALL.vocab, SPEC_PROMPT_LEN)]
    rep_prompt = (prompt[:8] * 3)[:20]
    out = {"model": "skinny_mlx_b200.model.SMALL, seed 0, init_device cpu; MTP head seed 13, init_device cpu",
           "prompt": prompt, "tokens": SPEC_TOKENS, "runs": {}}

    def greedy_run(p):
        tr = GapTrace(model)
        toks = spec.greedy(tr, p, SPEC_TOKENS)
        return toks, tr.gaps[:SPEC_TOKENS]

    ref, gaps = greedy_run(prompt)
    out["greedy"], out["gaps"] = ref, gaps
    drafters = {
        "scripted_k2_bad3": (lambda: ScriptDrafter(ref, 3, SMALL.vocab, core.array), 2),
        "scripted_k3_bad2": (lambda: ScriptDrafter(ref, 2, SMALL.vocab, core.array), 3),
        "scripted_k4_bad5": (lambda: ScriptDrafter(ref, 5, SMALL.vocab, core.array), 4),
        "mtp_k2": (lambda: spec.MTPDrafter(model, head, vocab=None), 2),
        "mtp_k3_vocab1024": (lambda: spec.MTPDrafter(model, head, vocab=1024), 3),
    }
    for name, (mk, k) in drafters.items():
        st = {}
        toks = spec.speculative(model, prompt, SPEC_TOKENS, mk(), k, st)
        out["runs"][name] = {"k": k, "tokens": toks, "steps": st["steps"]}
    # model-free prompt lookup on a prompt with repeats (drafts of varying length, none at times)
    ref_rep, gaps_rep = greedy_run(rep_prompt)
    out["repeat_prompt"], out["greedy_repeat"], out["gaps_repeat"] = rep_prompt, ref_rep, gaps_rep
    st = {}
    toks = spec.speculative(model, rep_prompt, SPEC_TOKENS, spec.PromptLookupDrafter(3), 3, st)
    out["runs"]["prompt_lookup_k3"] = {"k": 3, "tokens": toks, "steps": st["steps"], "prompt": "repeat"}
    (HERE / "spec_streams.json").write_text(json.dumps(out, indent=1) + "\n")


def main() -> None:
    if len(sys.argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py <checkout of the reference skinny-mlx>")
    ref_root = Path(sys.argv[1])
    ref_qmm = load_reference_module(ref_root, "skinny_mlx.qmm")
    make_repack(ref_qmm)
    make_config(ref_qmm)
    make_qmm_small()
    make_spec_streams(ref_root)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
