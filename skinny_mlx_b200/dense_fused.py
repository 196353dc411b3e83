"""One rank's verify step of the column-parallel dense model on the fused
kernels of the hybrid step (`skinny_mlx_b200.fused`), with the exchanges the sharding needs.

Per layer, rank g of G:

    prep     residual add (+ the previous layer's down output: every rank's [M, H/G] shard)
             + input RMSNorm -> digits of the full hidden
    qmm      fused q | k | v rows of the rank's heads
    attn     q/k norm, RoPE (all 128 dims), KV append, GQA attention -> digits of the rank's
             heads' output: 2 nq 64-column groups, a contiguous slice of o_proj's input
    qmm      o_proj rows [g H/G, (g+1) H/G) on all ranks' attention digits
    prep     residual add (every rank's o_proj shard) + post-attention RMSNorm -> digits
    qmm      gate | up rows of the rank's slice of the intermediate dimension
    prep     SwiGLU -> digits of the rank's I/G columns (a contiguous slice of down's input)
    qmm      down rows [g H/G, (g+1) H/G) on all ranks' SwiGLU digits

Two exchanges (G > 1):

* "peer" (the default): each rank keeps a buffer the other ranks map through CUDA IPC (NVLink peer
  memory).  The digit producers (attention, SwiGLU prep) write their digit blocks into every
  rank's buffer (skinny_peer_sync mirrors), so each qmm reads its whole input from local memory
  however often its tiles re-read it; the output shards of o_proj and down are read in place
  from their owners by the next prep (one 16-byte load per element group).  Consumers start
  after a bounded wait on per-(layer, kind) flags that each producer launch sets on every rank
  when its last CTA finishes.  No collective runs inside a layer; one NCCL all-gather of the
  logits ends the step.
* "nccl": an all_gather_into_tensor after each of the four producers (the comparison arm).

With G = 1 there is no exchange.  The logits come back as [G, M, V/G] (rank-major shards).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .dense import DenseModel
from .qmm import get_workspace

_KINDS = 4  # attention digits, o_proj shard, SwiGLU digits, down shard


def _p(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class DenseFusedStep:
    """exchange: "peer", "nccl", or "auto" (= "peer": measured on B200, config 5 at M = 8, the
    peer exchange takes 6.54 / 5.82 / 6.26 ms per step at 2 / 4 / 8 ranks against 8.67 / 8.29 /
    9.39 ms with NCCL's all-gathers, since its producers issue one system-scope fence per launch)."""

    def __init__(self, model: DenseModel, exchange: str = "auto"):
        from .patch import SkinnyQuantizedLinear

        self.model, self.cfg, self.G, self.rank = model, model.cfg, model.world, model.rank
        self.group = model.ex.group
        if exchange == "auto":
            exchange = "peer"
        self.exchange = exchange if self.G > 1 else "none"
        assert self.exchange in ("none", "peer", "nccl")
        cfg = self.cfg
        assert cfg.head_dim == 128
        self.layers = []
        for layer in model.layers:
            for lin in (layer.qkv_proj, layer.o_proj, layer.gate_up_proj, layer.down_proj):
                if not isinstance(lin, SkinnyQuantizedLinear):
                    raise ValueError("DenseFusedStep needs a patched model (skinny_mlx_b200.patch.patch_model)")
            self.layers.append({
                "qkv": layer.qkv_proj.rweight, "o": layer.o_proj.rweight, "gu": layer.gate_up_proj.rweight,
                "down": layer.down_proj.rweight, "in_norm": layer.input_layernorm.weight.float().contiguous(),
                "post_norm": layer.post_attention_layernorm.weight.float().contiguous(),
                "qn": layer.q_norm.weight.float().contiguous(), "kn": layer.k_norm.weight.float().contiguous()})
        self.nq, self.nkv = model.layers[0].nq, model.layers[0].nkv
        self.head = model.lm_head.rweight
        self.final_norm = model.norm.weight.float().contiguous()
        dev = model.device
        self.inv = (cfg.rope_theta ** (-torch.arange(0, 64, device=dev, dtype=torch.float32) / 64)).contiguous()
        self._bufs: dict[int, dict] = {}
        self._attn_ws: dict[int, torch.Tensor] = {}
        self._peer = None
        if self.exchange == "peer":
            self._setup_peer()

    @property
    def device(self):
        return self.model.device

    def make_cache(self, *a, **k):
        return self.model.make_cache(*a, **k)

    # ---------------------------------------------------------------- peer memory
    def _setup_peer(self):
        """One IPC buffer per rank: full-size digit buffers (this rank fills its groups), this
        rank's two output shards, and the flag words the other ranks store into."""
        cfg, G, L = self.cfg, self.G, _lib.lib()
        H, I = cfg.hidden, cfg.intermediate
        nl = len(self.layers)
        off, o = {}, 0
        for name, size in (("xq_o", int(L.skinny_xq_bytes(16, cfg.n_heads * 128))),
                           ("xq_i", int(L.skinny_xq_bytes(16, I))),
                           ("o", 16 * (H // G) * 2), ("dn", 16 * (H // G) * 2),
                           ("flags", nl * _KINDS * G * 4)):
            off[name] = o
            o = _align(o + size)
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _lib.call("skinny_ipc_alloc", o, ctypes.byref(ptr), handle)
        handles = [None] * G
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        bases = []
        for r in range(G):
            if r == self.rank:
                bases.append(ptr.value)
            else:
                p = ctypes.c_void_p()
                h = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                _lib.call("skinny_ipc_open", h, ctypes.byref(p))
                bases.append(p.value)
        dev = self.model.device
        counters = torch.zeros(nl * _KINDS, dtype=torch.int32, device=dev)
        epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        err = torch.zeros(4, dtype=torch.int32, device=dev)  # word 0: bits of timed-out peer waits
        me = self.rank

        def flag(r, layer, kind, src):
            return bases[r] + off["flags"] + ((layer * _KINDS + kind) * G + src) * 4

        syncs = []
        for layer in range(nl):
            per = []
            for kind in range(_KINDS):
                sig = _lib.PeerSync()
                sig.epoch = epoch.data_ptr()
                sig.counter = counters.data_ptr() + (layer * _KINDS + kind) * 4
                for r in range(G):
                    sig.signal_flags[r] = flag(r, layer, kind, me)
                sig.err = err.data_ptr()
                sig.n_ranks = G
                wait = _lib.PeerSync()
                wait.epoch = epoch.data_ptr()
                wait.wait_flags = flag(me, layer, kind, 0)
                wait.err = err.data_ptr()
                wait.n_ranks = G
                per.append((sig, wait))
            syncs.append(per)
        self._peer = {"bases": bases, "off": off, "own": ptr, "counters": counters, "epoch": epoch, "syncs": syncs,
                      "err": err}

    def errors(self) -> int:
        """Error bits the step's peer waits recorded (0: none; synchronises)."""
        if self._peer is None:
            return 0
        return int(self._peer["err"][0].item())

    def release(self):
        """Unmap the other ranks' buffers and free this rank's (call on every rank, after the
        last step and before the process group is destroyed)."""
        if self._peer is None:
            return
        torch.cuda.synchronize(self.model.device)
        dist.barrier(group=self.group)
        for r, b in enumerate(self._peer["bases"]):
            if r != self.rank:
                _lib.call("skinny_ipc_close", ctypes.c_void_p(b))
        dist.barrier(group=self.group)
        _lib.call("skinny_ipc_free", self._peer["own"])
        self._peer = None

    def _sync(self, layer, kind, role):
        return ctypes.byref(self._peer["syncs"][layer][kind][0 if role == "signal" else 1])

    def _ranks(self, name, xb=0, per_rank=0):
        """Device addresses of region `name` in every rank's buffer (ctypes array)."""
        arr = (ctypes.c_void_p * 8)()
        for r, b in enumerate(self._peer["bases"]):
            arr[r] = b + self._peer["off"][name] + r * per_rank * xb
        return arr

    # ---------------------------------------------------------------- buffers per token count
    def _buffers(self, m: int) -> dict:
        b = self._bufs.get(m)
        if b is None:
            cfg, G, dev = self.cfg, self.G, self.model.device
            L = _lib.lib()
            xq = lambda k: torch.zeros(int(L.skinny_xq_bytes(m, k)), dtype=torch.uint8, device=dev)
            bf = lambda *shape: torch.zeros(*shape, dtype=torch.bfloat16, device=dev)
            H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim
            b = {"h": [bf(m, H), bf(m, H)], "a": bf(m, H), "xq_h": xq(H),
                 "proj": bf(m, (self.nq + 2 * self.nkv) * D), "gu": bf(m, 2 * I // G),
                 "logits": bf(G, m, self.head.N), "logits_loc": bf(m, self.head.N),
                 "xb": int(L.skinny_xq_bytes(m, 64))}  # bytes of one group's digit block
            if self.exchange == "nccl":
                b.update(xq_o=xq(cfg.n_heads * D), xq_o_loc=xq(self.nq * D), xq_i=xq(I), xq_i_loc=xq(I // G),
                         o_loc=bf(m, H // G), o_all=bf(G, m, H // G), dn_loc=bf(m, H // G), dn_all=bf(G, m, H // G))
            elif self.exchange == "none":
                b.update(xq_o=xq(cfg.n_heads * D), xq_i=xq(I), o_all=bf(1, m, H), dn_all=bf(1, m, H))
            self._bufs[m] = b
        return b

    # ---------------------------------------------------------------- launches
    def _qmm(self, w, out_ptr, ldo, m, stream, xq=None, xq_ranks=None, gpr=0, sync=None):
        ws = get_workspace(self.model.device, int(_lib.lib().skinny_qmm_workspace_bytes(w.N, w.K)))
        xq_arg = xq if isinstance(xq, ctypes.c_void_p) else _p(xq)
        _lib.call("skinny_qmm_w4g64_prepared", xq_arg, _p(w.w_tc), ctypes.c_void_p(out_ptr), ldo, m, w.N, w.K,
                  _p(ws), ws.numel(), xq_ranks, gpr, sync, stream)

    def _own(self, region: str, offset: int = 0) -> ctypes.c_void_p:
        """Address of `region` (+ offset bytes) in this rank's peer buffer."""
        return ctypes.c_void_p(self._peer["bases"][self.rank] + self._peer["off"][region] + offset)

    def _signal_mirrored(self, layer, kind, region, offset):
        """The signal of a digit producer that also writes its digits into every other rank's
        copy of `region` (at the same offset): consumers then read all digits locally."""
        key = ("m", layer, kind, region, offset)
        cache = self._peer.setdefault("mirrored", {})
        s = cache.get(key)
        if s is None:
            base = self._peer["syncs"][layer][kind][0]
            s = _lib.PeerSync()
            ctypes.pointer(s)[0] = base  # copy of the plain signal
            n = 0
            for r, b in enumerate(self._peer["bases"]):
                if r != self.rank:
                    s.mirror[n] = b + self._peer["off"][region] + offset
                    n += 1
            s.n_mirror = n
            cache[key] = s
        return ctypes.byref(s)

    def _prep0(self, x, h_out, w, m, xq, stream, segs=None, a_out=None, sync=None):
        """Residual add of every rank's [m, H/G] shard (segs: their addresses) and RMSNorm."""
        H = self.cfg.hidden
        seg = H // self.G
        _lib.call("skinny_prep", 0, _p(x), H, None, seg, seg if segs is not None else 0, segs,
                  _p(h_out if segs is not None else None), H if segs is not None else 0, _p(w), self.cfg.rms_eps,
                  m, H, _p(xq), _p(a_out), sync, stream)

    def _gather(self, dst, src):
        dist.all_gather_into_tensor(dst, src, group=self.group)

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, caches) -> torch.Tensor:
        """Logits [G, M, V/G] bf16 (rank-major shards of the vocabulary; a reused buffer)."""
        cfg, m, G = self.cfg, ids.shape[0], self.G
        assert 1 <= m <= 16
        b = self._buffers(m)
        dev = self.model.device
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        peer = self.exchange == "peer"
        if peer:
            self._peer["epoch"].add_(1)  # one step: every flag of this step carries the new epoch
        w, s, bb = self.model.embed
        hs, cur = b["h"], 0
        ids = ids.to(torch.long).contiguous()
        _lib.call("skinny_embed_w4g64", _p(ids), m, _p(w), _p(s), _p(bb), w.shape[0], cfg.hidden, _p(hs[0]),
                  hs[0].stride(0), stream)
        D, H, I = cfg.head_dim, cfg.hidden, cfg.intermediate
        xb = b["xb"]
        gpr_o, gpr_i = 2 * self.nq, I // G // 64
        segs_of = lambda buf: None if buf is None else (ctypes.c_void_p * 8)(
            *[buf.data_ptr() + g * m * (H // G) * 2 for g in range(G)])
        prev = None  # how the previous layer's down output is read: (segs, sync) or None
        for li, (ent, c) in enumerate(zip(self.layers, caches)):
            # ---- input norm (+ previous down shards)
            if prev is None:
                self._prep0(hs[cur], None, ent["in_norm"], m, b["xq_h"], stream)
            else:
                self._prep0(hs[cur], hs[1 - cur], ent["in_norm"], m, b["xq_h"], stream, segs=prev[0], sync=prev[1])
                cur = 1 - cur
            self._qmm(ent["qkv"], b["proj"].data_ptr(), b["proj"].stride(0), m, stream, xq=b["xq_h"])
            # ---- attention -> digits of this rank's heads
            max_len = c.k.shape[0]
            ws = self._attn_ws.get(max_len)
            if ws is None:
                n = int(_lib.lib().skinny_attn_workspace_bytes(16, self.nq, self.nkv, max_len))
                ws = self._attn_ws[max_len] = torch.zeros(n, dtype=torch.uint8, device=dev)
            if peer:  # this rank's heads' digits, written here and in every other rank's buffer
                xq_o_mine = self._own("xq_o", self.rank * gpr_o * xb)
                asig = self._signal_mirrored(li, 0, "xq_o", self.rank * gpr_o * xb)
            else:
                xq_o_mine = _p(b["xq_o_loc"] if self.exchange == "nccl" else b["xq_o"])
                asig = None
            _lib.call("skinny_attn_fused", _p(b["proj"]), b["proj"].stride(0), _p(ent["qn"]), _p(ent["kn"]),
                      _p(self.inv), D, 0, cfg.rms_eps, _p(c.k), _p(c.v), c.length, None, m, self.nq, self.nkv,
                      max_len, _p(ws), ws.numel(), xq_o_mine, None, asig, stream)
            c.length += m
            # ---- o_proj -> this rank's shard of the hidden
            if peer:
                o_ptr = self._peer["bases"][self.rank] + self._peer["off"]["o"]
                self._qmm(ent["o"], o_ptr, H // G, m, stream, xq=self._own("xq_o"), sync=self._combined(li, 0, 1))
                o_segs, o_wait = self._ranks("o"), self._sync(li, 1, "wait")
            else:
                if self.exchange == "nccl":
                    self._gather(b["xq_o"], b["xq_o_loc"])
                    out = b["o_loc"]
                else:
                    out = b["o_all"][0]
                self._qmm(ent["o"], out.data_ptr(), out.stride(0), m, stream, xq=b["xq_o"])
                if self.exchange == "nccl":
                    self._gather(b["o_all"], b["o_loc"])
                o_segs, o_wait = segs_of(b["o_all"]), None
            self._prep0(hs[cur], hs[1 - cur], ent["post_norm"], m, b["xq_h"], stream, segs=o_segs, sync=o_wait)
            cur = 1 - cur
            # ---- MLP
            self._qmm(ent["gu"], b["gu"].data_ptr(), b["gu"].stride(0), m, stream, xq=b["xq_h"])
            if peer:
                xq_i_mine = self._own("xq_i", self.rank * gpr_i * xb)
                psig = self._signal_mirrored(li, 2, "xq_i", self.rank * gpr_i * xb)
            else:
                xq_i_mine = _p(b["xq_i_loc"] if self.exchange == "nccl" else b["xq_i"])
                psig = None
            _lib.call("skinny_prep", 1, _p(b["gu"]), b["gu"].stride(0), None, 0, 0, None, None, 0, None, 0.0, m,
                      I // G, xq_i_mine, None, psig, stream)
            if peer:
                dn_ptr = self._peer["bases"][self.rank] + self._peer["off"]["dn"]
                self._qmm(ent["down"], dn_ptr, H // G, m, stream, xq=self._own("xq_i"), sync=self._combined(li, 2, 3))
                prev = (self._ranks("dn"), self._sync(li, 3, "wait"))
            else:
                if self.exchange == "nccl":
                    self._gather(b["xq_i"], b["xq_i_loc"])
                    out = b["dn_loc"]
                else:
                    out = b["dn_all"][0]
                self._qmm(ent["down"], out.data_ptr(), out.stride(0), m, stream, xq=b["xq_i"])
                if self.exchange == "nccl":
                    self._gather(b["dn_all"], b["dn_loc"])
                prev = (segs_of(b["dn_all"]), None)
        self._prep0(hs[cur], hs[1 - cur], self.final_norm, m, b["xq_h"], stream, segs=prev[0], sync=prev[1],
                    a_out=b["a"])
        lg = b["logits_loc"] if G > 1 else b["logits"][0]
        self._qmm(self.head, lg.data_ptr(), lg.stride(0), m, stream, xq=b["xq_h"])
        if G > 1:
            self._gather(b["logits"], b["logits_loc"])
        return b["logits"]

    def _combined(self, layer, wait_kind, signal_kind):
        """One launch that waits for `wait_kind` and signals `signal_kind` (a qmm between them)."""
        key = ("c", layer, wait_kind, signal_kind)
        cache = self._peer.setdefault("combined", {})
        s = cache.get(key)
        if s is None:
            sig = self._peer["syncs"][layer][signal_kind][0]
            wait = self._peer["syncs"][layer][wait_kind][1]
            s = _lib.PeerSync()
            s.epoch = sig.epoch
            s.wait_flags = wait.wait_flags
            s.counter = sig.counter
            for r in range(8):
                s.signal_flags[r] = sig.signal_flags[r]
            s.err = sig.err
            s.n_ranks = sig.n_ranks
            cache[key] = s
        return ctypes.byref(s)


__all__ = ["DenseFusedStep"]
