"""Fused verify step of a patched hybrid model (the B200 runtime for config 3 and 4).

The module-by-module forward of `HybridModel` runs every small elementwise step as its own
PyTorch kernel (dozens per layer).  `FusedStep` runs the same model with five kernel kinds and
no intermediate activation round trips:

    prep (residual add + RMSNorm -> qmm input digits)                  skinny_prep mode 0
    qmm on prepared digits                                              skinny_qmm_w4g64_prepared
    GDN mixer (conv .. gated norm -> out_proj digits)                   skinny_gdn_fused
    attention mixer (norm, RoPE, KV append .. gate -> o_proj digits)    skinny_attn_fused
    prep (SwiGLU -> down_proj digits)                                   skinny_prep mode 1

Residual additions are deferred into the next prep.  The result equals the
module-by-module patched forward up to the rounding of the fused reductions (norms, softplus,
silu in f32), and the caches (`Cache`) are the same objects, so `HybridRollback` and the
speculative loop work unchanged.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .model import AttnCache, GDNCache, HybridModel
from .qmm import SkinnyWeight, get_workspace



def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def layer_entry(layer, cfg) -> dict:
    """The weights one decoder layer of a patched hybrid model runs with in the fused step."""
    from .patch import FusedSliceLinear, SkinnyQuantizedLinear

    mlp = layer.mlp
    assert isinstance(mlp.gate_proj, FusedSliceLinear) and isinstance(mlp.down_proj, SkinnyQuantizedLinear)
    ent = {"gate_up": mlp.gate_proj._group.rw, "swiglu": mlp.gate_proj._group.interleaved, "down": mlp.down_proj.rweight,
           "in_norm": layer.input_layernorm.weight, "post_norm": layer.post_attention_layernorm.weight}
    if layer.is_linear:
        g = layer.linear_attn
        ent.update(kind="gdn", mod=g, proj=g.in_proj_qkv._group.rw, out=g.out_proj.rweight,
                   conv_w=g.conv_weight.float().contiguous(), A_log=g.A_log.float().contiguous(),
                   dt_bias=g.dt_bias.float().contiguous(), norm_w=g.norm.weight.float().contiguous())
    else:
        a = layer.self_attn
        (q0, q1), (k0, k1), (v0, v1) = a.q_proj._group.bounds
        D = cfg.head_dim
        assert D == 128 and (q0, k0, v0) == (0, 2 * cfg.n_heads * D, 2 * cfg.n_heads * D
                                             + cfg.n_kv_heads * D), "q|gate, k, v fused in order"
        half = cfg.rotary_dim // 2
        dev = a.q_norm.weight.device
        inv = cfg.rope_theta ** (-torch.arange(0, half, device=dev, dtype=torch.float32) / half)
        ent.update(kind="attn", mod=a, proj=a.q_proj._group.rw, out=a.o_proj.rweight,
                   qn=a.q_norm.weight.float().contiguous(), kn=a.k_norm.weight.float().contiguous(),
                   inv=inv.contiguous())
    return ent


class FusedOps:
    """The launches the fused step is made of (prep, prepared qmm, fused attention), for a
    hybrid-model config `cfg`; subclasses run a model or a draft head with them."""

    cfg = None
    _attn_ws: dict

    @staticmethod
    def _err_word(dev) -> torch.Tensor:
        """Word 0 of the device's qmm workspace: device-side errors of every kernel of the step
        land in one place (skinny_mlx_b200.qmm.device_errors reads it)."""
        return get_workspace(dev, int(_lib.lib().skinny_qmm_workspace_bytes(128, 64)))

    def _attention(self, ent, proj, c: AttnCache, m: int, xq, stream, len_dev=None, tree=None):
        """len_dev: a device int32 holding c.length when the launch runs (graph replay); the
        caller then advances the host length itself.  tree: device int32 parents of the m
        tokens (a draft tree) or None."""
        cfg = self.cfg
        max_len = c.k.shape[0]
        ws = self._attn_ws.get(max_len)
        if ws is None:  # sized for 16 tokens; zero on first use, left zero by every call
            n = int(_lib.lib().skinny_attn_workspace_bytes(16, cfg.n_heads, cfg.n_kv_heads, max_len))
            ws = self._attn_ws[max_len] = torch.zeros(n, dtype=torch.uint8, device=proj.device)
        L0 = c.length
        if tree is None:
            _lib.call("skinny_attn_fused", _p(proj), proj.stride(0), _p(ent["qn"]), _p(ent["kn"]), _p(ent["inv"]),
                      cfg.rotary_dim, 1, cfg.rms_eps, _p(c.k), _p(c.v), L0, _p(len_dev), m, cfg.n_heads,
                      cfg.n_kv_heads, max_len, _p(ws), ws.numel(), _p(xq), None, None, stream)
        else:
            _lib.call("skinny_attn_fused_tree", _p(proj), proj.stride(0), _p(ent["qn"]), _p(ent["kn"]),
                      _p(ent["inv"]), cfg.rotary_dim, 1, cfg.rms_eps, _p(c.k), _p(c.v), L0, _p(len_dev), m,
                      cfg.n_heads, cfg.n_kv_heads, max_len, _p(ws), ws.numel(), _p(xq), None, _p(tree), stream)
        if len_dev is None:
            c.length = L0 + m

    def _qmm(self, xq, w: SkinnyWeight, out, m: int, stream):
        ws = get_workspace(out.device, int(_lib.lib().skinny_qmm_workspace_bytes(w.N, w.K)))
        _lib.call("skinny_qmm_w4g64_prepared", _p(xq), _p(w.w_tc), _p(out), out.stride(0), m, w.N, w.K,
                  _p(ws), ws.numel(), None, 0, None, stream)

    def _gate_up(self, ent, xq_h, gu, xq_i, m: int, stream):
        """gate|up projection and SwiGLU -> down_proj digits: one launch (activation in the qmm
        epilogue) for an interleaved gate|up weight, else the product and skinny_prep mode 1."""
        w = ent["gate_up"]
        if ent.get("swiglu"):
            ws = get_workspace(xq_i.device, int(_lib.lib().skinny_qmm_workspace_bytes(w.N, w.K)))
            _lib.call("skinny_qmm_w4g64_swiglu", _p(xq_h), _p(w.w_tc), _p(xq_i), m, w.N, w.K, _p(ws), ws.numel(),
                      stream)
        else:
            self._qmm(xq_h, w, gu, m, stream)
            self._prep(1, gu, m, w.N // 2, xq_i, stream)

    def _prep(self, mode, x, m, k, xq, stream, d=None, h_out=None, w=None, a_out=None):
        _lib.call("skinny_prep", mode, _p(x), x.stride(0), _p(d), d.stride(0) if d is not None else 0, 0, None,
                  _p(h_out), h_out.stride(0) if h_out is not None else 0, _p(w), self.cfg.rms_eps, m, k,
                  _p(xq), _p(a_out), None, stream)


class FusedStep(FusedOps):
    def __init__(self, model: HybridModel):
        self.model, self.cfg = model, model.cfg
        emb = model.embed_tokens
        if not hasattr(emb, "skinny_head"):
            raise ValueError("FusedStep needs a patched model (skinny_mlx_b200.patch.patch_model)")
        self.head = emb.skinny_head
        self.layers = [layer_entry(layer, self.cfg) for layer in model.layers]
        self.final_norm = model.norm.weight
        self._bufs: dict[int, dict] = {}
        self._attn_ws: dict[int, torch.Tensor] = {}
        self._tree_bufs: dict[int, torch.Tensor] = {}

    @property
    def device(self):
        return self.model.device

    def _tree_dev(self, tree, m: int):
        """The parents of a draft tree as a device int32 [m] tensor (copied there if given on the
        host), or None for a chain."""
        if tree is None or (isinstance(tree, torch.Tensor) and tree.is_cuda):
            return tree
        buf = self._tree_bufs.get(m)
        if buf is None:
            buf = self._tree_bufs[m] = torch.empty(m, dtype=torch.int32, device=self.model.device)
        buf.copy_(torch.as_tensor(tree, dtype=torch.int32))
        return buf

    def make_cache(self, *a, **k):
        return self.model.make_cache(*a, **k)

    @property
    def embed_tokens(self):
        return self.model.embed_tokens

    # ---------------------------------------------------------------- buffers per token count
    def _buffers(self, m: int) -> dict:
        b = self._bufs.get(m)
        if b is None:
            cfg, dev = self.cfg, self.model.device
            L = _lib.lib()
            xq = lambda k: torch.empty(int(L.skinny_xq_bytes(m, k)), dtype=torch.uint8, device=dev)
            widths = {self.layers[i]["proj"].N for i in range(len(self.layers))}
            b = {"h": [torch.empty(m, cfg.hidden, dtype=torch.bfloat16, device=dev) for _ in range(2)],
                 "a": torch.empty(m, cfg.hidden, dtype=torch.bfloat16, device=dev),
                 "xq_h": xq(cfg.hidden), "xq_i": xq(cfg.intermediate),
                 "xq_o": xq(max(cfg.gdn_value_dim, cfg.n_heads * cfg.head_dim)),
                 "proj": {n: torch.empty(m, n, dtype=torch.bfloat16, device=dev) for n in widths},
                 "mix": torch.empty(m, cfg.hidden, dtype=torch.bfloat16, device=dev),
                 "gu": torch.empty(m, 2 * cfg.intermediate, dtype=torch.bfloat16, device=dev),
                 "down": torch.empty(m, cfg.hidden, dtype=torch.bfloat16, device=dev),
                 "logits": torch.empty(m, self.head.N, dtype=torch.bfloat16, device=dev)}
            self._bufs[m] = b
        return b

    # ---------------------------------------------------------------- the step
    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, cache, lens_dev: torch.Tensor | None = None, tree=None
                 ) -> tuple[torch.Tensor, torch.Tensor]:
        """Same contract as HybridModel.forward for 1 <= len(ids) <= 16: (final normed hidden,
        logits) as bf16 [T, H] and [T, V] (views of reused buffers: copy to keep).  lens_dev
        (int32, one entry per attention layer): the attention kernels read the cache lengths there
        and the host lengths are left to the caller (see GraphedStep).  tree: the parents of the
        tokens (host list or device int32 tensor) for a draft-tree verify, which needs recording
        GDN caches (HybridRollback.record) and is followed by HybridRollback.rollback_tree."""
        cfg, m = self.cfg, ids.shape[0]
        if m > 16:  # prefill: the module-by-module forward (qmm in 16-token chunks)
            if tree is not None:
                raise ValueError("a tree verify takes at most 16 tokens")
            return self.model(ids, cache)
        tree = self._tree_dev(tree, m)
        b = self._buffers(m)
        stream = ctypes.c_void_p(torch.cuda.current_stream(self.model.device).cuda_stream)
        emb = self.model.embed_tokens
        # the residual stream alternates between two buffers: a prep reads one and writes the other
        hs = b["h"]
        cur = 0
        ids = ids.to(torch.long).contiguous()
        _lib.call("skinny_embed_w4g64", _p(ids), m, _p(emb.weight), _p(emb.scales), _p(emb.biases),
                  emb.weight.shape[0], cfg.hidden, _p(hs[0]), hs[0].stride(0), stream)
        d = None

        def add_norm(d, w, a_out=None):
            nonlocal cur
            if d is None:
                self._prep(0, hs[cur], m, cfg.hidden, b["xq_h"], stream, w=w, a_out=a_out)
            else:
                self._prep(0, hs[cur], m, cfg.hidden, b["xq_h"], stream, d=d, h_out=hs[1 - cur], w=w, a_out=a_out)
                cur = 1 - cur

        ai = 0
        for ent, c in zip(self.layers, cache.layers):
            # x_l = x_{l-1} + down_{l-1}; digits of input_layernorm(x_l)
            add_norm(d, ent["in_norm"])
            proj = b["proj"][ent["proj"].N]
            self._qmm(b["xq_h"], ent["proj"], proj, m, stream)
            if ent["kind"] == "gdn":
                c: GDNCache
                rec = c.recording
                if rec:
                    c.fed = m
                if tree is not None:
                    if not rec:
                        raise ValueError("a tree verify needs recording GDN caches (HybridRollback.record)")
                    _lib.call("skinny_gdn_fused_tree", _p(proj), proj.stride(0), _p(c.conv), _p(c.conv_full),
                              _p(ent["conv_w"]), _p(ent["A_log"]), _p(ent["dt_bias"]), _p(ent["norm_w"]),
                              cfg.rms_eps, _p(c.state), _p(c.ckpt), _p(b["xq_o"]), None, m, cfg.gdn_v_heads,
                              cfg.gdn_k_heads, cfg.conv_kernel - 1, _p(self._err_word(proj.device)), _p(tree), stream)
                else:
                    _lib.call("skinny_gdn_fused", _p(proj), proj.stride(0), _p(c.conv),
                              _p(c.conv_full if rec else None), _p(ent["conv_w"]), _p(ent["A_log"]),
                              _p(ent["dt_bias"]), _p(ent["norm_w"]), cfg.rms_eps, _p(c.state),
                              _p(c.ckpt if rec and m > 1 else None), _p(b["xq_o"]), None, m, cfg.gdn_v_heads,
                              cfg.gdn_k_heads, cfg.conv_kernel - 1, _p(self._err_word(proj.device)), stream)
            else:
                self._attention(ent, proj, c, m, b["xq_o"], stream,
                                None if lens_dev is None else lens_dev[ai:ai + 1], tree)
                ai += 1
            self._qmm(b["xq_o"], ent["out"], b["mix"], m, stream)
            # h = x_l + mixer; digits of post_attention_layernorm(h)
            add_norm(b["mix"], ent["post_norm"])
            self._gate_up(ent, b["xq_h"], b["gu"], b["xq_i"], m, stream)
            self._qmm(b["xq_i"], ent["down"], b["down"], m, stream)
            d = b["down"]
        add_norm(d, self.final_norm, a_out=b["a"])
        self._qmm(b["xq_h"], self.head, b["logits"], m, stream)
        return b["a"], b["logits"]


class GraphedStep:
    """FusedStep replayed from one CUDA graph per (cache, token count, recording state).

    The step's launches are captured once; per call the host copies the token ids into the
    graph's input buffer and the attention caches' lengths into a device array (one small copy
    each, ordered on the stream before the replay), replays, and advances the host lengths.
    Longer inputs (prefill) run FusedStep eagerly.  Attribute access falls through to the
    FusedStep, so the greedy and speculative loops take either."""

    def __init__(self, fused: FusedStep):
        self.fused = fused
        self._graphs: dict = {}
        self._stream = torch.cuda.Stream(fused.device)

    def __getattr__(self, name):
        return getattr(self.fused, name)

    @staticmethod
    def _lens(cache):
        if not hasattr(cache, "_lens_dev"):
            attn = [c for c in cache.layers if isinstance(c, AttnCache)]
            cache._attn = attn
            cache._lens_dev = torch.zeros(max(len(attn), 1), dtype=torch.int32, device=attn[0].k.device)
            cache._lens_host = torch.zeros(max(len(attn), 1), dtype=torch.int32).pin_memory()
        return cache._attn, cache._lens_dev, cache._lens_host

    def _capture(self, cache, m: int, tree: bool = False):
        f, dev = self.fused, self.fused.device
        attn, lens_dev, _ = self._lens(cache)
        ids_buf = torch.zeros(m, dtype=torch.long, device=dev)
        # a tree graph reads the parents from a device buffer filled before every replay
        par_buf = torch.tensor([-1] + list(range(m - 1)), dtype=torch.int32, device=dev) if tree else None
        gdn = [c for c in cache.layers if isinstance(c, GDNCache)]
        # warm-up on a scratch cache of the same shape, on the capture stream (buffers, the
        # stream's qmm workspace and kernel attributes exist before capture)
        scratch = f.make_cache(max_len=attn[0].k.shape[0], max_verify=gdn[0].max_verify if gdn else 17)
        for c, s2 in zip(cache.layers, scratch.layers):
            if isinstance(c, GDNCache):
                s2.recording = c.recording
        _, slens, _ = self._lens(scratch)
        self._stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self._stream):
            f(ids_buf, scratch, slens, par_buf)
        self._stream.synchronize()
        del scratch
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self._stream):
            f(ids_buf, cache, lens_dev, par_buf)
        # the entry keeps the cache alive: its id (the key) can then not be reused by another
        # cache while the graph, which holds its buffers' addresses, exists
        par_host = torch.zeros(m, dtype=torch.int32).pin_memory() if tree else None
        ent = (ids_buf, g, cache, par_buf, par_host)
        self._graphs[(id(cache), m, tuple(c.recording for c in gdn), tree)] = ent
        return ent

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, cache, tree=None):
        """tree: parents of the tokens (host list) for a draft-tree verify, else None."""
        m = ids.shape[0]
        if m > 16:
            return self.fused(ids, cache, tree=tree)
        gdn = [c for c in cache.layers if isinstance(c, GDNCache)]
        key = (id(cache), m, tuple(c.recording for c in gdn), tree is not None)
        ent = self._graphs.get(key) or self._capture(cache, m, tree is not None)
        ids_buf, g, _, par_buf, par_host = ent
        attn, lens_dev, lens_host = self._lens(cache)
        if hasattr(cache, "_lens_evt"):
            cache._lens_evt.synchronize()  # the previous copy out of the pinned buffers is done
        for i, c in enumerate(attn):
            lens_host[i] = c.length
        ids_buf.copy_(ids, non_blocking=True)
        lens_dev.copy_(lens_host, non_blocking=True)
        if tree is not None:
            par_host.copy_(torch.as_tensor(tree, dtype=torch.int32))
            par_buf.copy_(par_host, non_blocking=True)
        if not hasattr(cache, "_lens_evt"):
            cache._lens_evt = torch.cuda.Event()
        cache._lens_evt.record()
        g.replay()
        for c in attn:
            c.length += m
        for c in gdn:
            if c.recording:
                c.fed = m
        b = self.fused._bufs[m]
        return b["a"], b["logits"]

    def release(self) -> None:
        """Drop the captured graphs (e.g. when their caches are discarded)."""
        self._graphs.clear()


__all__ = ["FusedStep", "GraphedStep"]
