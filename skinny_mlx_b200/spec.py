"""Greedy speculative acceptance on the device (skinny_mlx/spec.py:136-147).

`accept(logits, draft)` replaces the reference's verify tail -- argmax over the K+1 verified
logits, `.tolist()` of predictions and draft (its one host sync per step) and the Python prefix
loop -- with one kernel launch and a read-back of K+2 int32 values.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_ws: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(dev: torch.device) -> torch.Tensor:
    key = (dev.index if dev.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(dev).cuda_stream)
    ws = _ws.get(key)
    if ws is None:
        ws = torch.zeros(int(_lib.lib().skinny_spec_accept_workspace_bytes()), dtype=torch.uint8, device=dev)
        _ws[key] = ws
    return ws


def accept_device(logits: torch.Tensor, draft: torch.Tensor, result: torch.Tensor | None = None,
                  pred: torch.Tensor | None = None) -> torch.Tensor:
    """Stream-ordered, no host sync.  logits bf16 [K+1, V] (rows contiguous), draft int32 [K] on
    the same device.  Returns result int32 [K+2]: [n, draft[:n] + [pred[n]], -1 ...]."""
    if logits.dtype != torch.bfloat16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a bf16 [K+1, V] tensor with unit column stride")
    rows, v = logits.shape
    if draft.numel() != rows - 1 or draft.dtype != torch.int32:
        raise ValueError("draft must be int32 with K = rows - 1 entries")
    dev = logits.device
    if result is None:
        result = torch.empty(rows + 1, dtype=torch.int32, device=dev)
    ws = _workspace(dev)
    _lib.call("skinny_spec_accept", ctypes.c_void_p(logits.data_ptr()), logits.stride(0), rows, v,
              ctypes.c_void_p(draft.data_ptr() if rows > 1 else 0), ctypes.c_void_p(result.data_ptr()),
              ctypes.c_void_p(pred.data_ptr() if pred is not None else 0), ctypes.c_void_p(ws.data_ptr()),
              ws.numel(), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    return result


def accept(logits: torch.Tensor, draft: torch.Tensor) -> tuple[int, list[int]]:
    """(n accepted draft tokens, emitted tokens draft[:n] + [pred[n]]); one small D2H."""
    r = accept_device(logits, draft).cpu().tolist()
    n = r[0]
    return n, r[1:n + 2]


def accept_tree(logits: torch.Tensor, tokens: torch.Tensor, parent: torch.Tensor) -> tuple[int, list[int], list[int]]:
    """Greedy acceptance of a verified draft tree (one launch, one small D2H): logits bf16
    [M, V] of the M nodes, tokens int32 [M] (node 0 = the last emitted token), parent int32 [M]
    (parent[0] = -1, parent[t] < t), all on the device.  From the root, move to the first child
    whose token equals the current node's prediction while one exists.  Returns (n accepted
    nodes, emitted tokens: theirs + the last node's prediction, the path 0, p1 .. pn)."""
    if logits.dtype != torch.bfloat16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a bf16 [M, V] tensor with unit column stride")
    rows, v = logits.shape
    if tokens.numel() != rows or parent.numel() != rows or tokens.dtype != torch.int32 or parent.dtype != torch.int32:
        raise ValueError("tokens and parent must be int32 with one entry per node")
    dev = logits.device
    result = torch.empty(2 * rows + 1, dtype=torch.int32, device=dev)
    ws = _workspace(dev)
    _lib.call("skinny_spec_accept_tree", ctypes.c_void_p(logits.data_ptr()), logits.stride(0), rows, v,
              ctypes.c_void_p(tokens.data_ptr()), ctypes.c_void_p(parent.data_ptr()), ctypes.c_void_p(result.data_ptr()),
              None, ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    r = result.cpu().tolist()
    n = r[0]
    return n, r[1:n + 2], r[1 + rows:2 + rows + n]


__all__ = ["accept", "accept_device", "accept_tree"]


# ---------------------------------------------------------------------------------------------
# decode loops (skinny_mlx/spec.py:54-156 on B200)
# ---------------------------------------------------------------------------------------------
def _accept_tree_any(logits: torch.Tensor, tokens: torch.Tensor, parent: list[int]) -> tuple[int, list[int], list[int]]:
    if logits.is_cuda:
        return accept_tree(logits, tokens.to(torch.int32), torch.tensor(parent, dtype=torch.int32, device=logits.device))
    pred = torch.argmax(logits.float(), dim=-1).tolist()  # CPU runs of the model (tests)
    tok = tokens.tolist()
    cur, path = 0, [0]
    while True:
        nxt = next((c for c in range(cur + 1, len(parent)) if parent[c] == cur and tok[c] == pred[cur]), None)
        if nxt is None:
            break
        path.append(nxt)
        cur = nxt
    return len(path) - 1, [tok[c] for c in path[1:]] + [pred[cur]], path


def _accept_any(logits: torch.Tensor, draft: torch.Tensor) -> tuple[int, list[int]]:
    if logits.is_cuda:
        return accept(logits, draft)
    pred = torch.argmax(logits.float(), dim=-1).tolist()  # CPU runs of the model (tests)
    d = draft.tolist()
    n = 0
    while n < len(d) and d[n] == pred[n]:
        n += 1
    return n, d[:n] + [pred[n]]


class HybridRollback:
    """Replay-free rollback of the hybrid cache (skinny_mlx/rollback.py:19-73): the verify forward
    writes GDN state checkpoints and records its conv input; rollback selects checkpoint keep-1
    and re-slices the conv window (one launch for all GDN layers) and trims attention caches."""

    def record(self, cache) -> None:
        from .model import GDNCache

        for c in cache.layers:
            if isinstance(c, GDNCache):
                c.recording = True

    def rollback(self, cache, fed: int, keep: int) -> None:
        from .model import AttnCache, GDNCache

        gdn = [c for c in cache.layers if isinstance(c, GDNCache)]
        for c in gdn:
            c.recording = False
        if keep == fed:
            return
        assert 1 <= keep < fed
        if gdn and gdn[0].state.is_cuda:
            from .gdn import rollback

            rollback([c.state for c in gdn], [c.ckpt for c in gdn], keep, fed, [c.conv for c in gdn],
                     [c.conv_full for c in gdn])
        else:
            for c in gdn:
                c.state.copy_(c.ckpt[keep - 1])
                c.conv.copy_(c.conv_full[keep: keep + c.conv.shape[0]])
        for c in cache.layers:
            if isinstance(c, AttnCache):
                c.trim(fed - keep)

    def rollback_tree(self, cache, fed: int, path: list[int]) -> None:
        """After a tree verify of `fed` nodes, keep the accepted path (node indices, root 0
        first): GDN state <- the checkpoint of the path's last node, conv window <- the last W
        conv inputs along the path; attention caches keep the path's keys and values, moved to
        the slots of their positions (L0 + depth), and drop the rest."""
        from .model import AttnCache, GDNCache

        gdn = [c for c in cache.layers if isinstance(c, GDNCache)]
        for c in gdn:
            c.recording = False
        node, n = path[-1], len(path) - 1
        if gdn:
            W = gdn[0].conv.shape[0]
            rows = ([*range(W)] + [W + j for j in path])[-W:]
            if gdn[0].state.is_cuda:
                from .gdn import rollback_tree

                rollback_tree([c.state for c in gdn], [c.ckpt for c in gdn], node, rows, fed, [c.conv for c in gdn],
                              [c.conv_full for c in gdn])
            else:
                for c in gdn:
                    c.state.copy_(c.ckpt[node])
                    c.conv.copy_(c.conv_full[rows])
        attn = [c for c in cache.layers if isinstance(c, AttnCache)]
        if attn and path[1:] != list(range(1, n + 1)):  # the path's keys / values to slots L0 + depth
            L0 = [c.length - fed for c in attn]
            if attn[0].k.is_cuda:
                import ctypes

                arr = ctypes.c_void_p * len(attn)
                _lib.call("skinny_kv_compact", len(attn), arr(*[c.k.data_ptr() for c in attn]),
                          arr(*[c.v.data_ptr() for c in attn]), attn[0].k[0].numel() * attn[0].k.element_size(),
                          (ctypes.c_int32 * len(attn))(*L0), (ctypes.c_int32 * len(path))(*path), len(path),
                          attn[0].k.shape[0], ctypes.c_void_p(torch.cuda.current_stream(attn[0].k.device).cuda_stream))
            else:
                for c, l0 in zip(attn, L0):
                    src = torch.tensor([l0 + j for j in path[1:]])
                    c.k[l0 + 1:l0 + 1 + n] = c.k[src]
                    c.v[l0 + 1:l0 + 1 + n] = c.v[src]
        for c in attn:
            c.length = c.length - fed + 1 + n


def chain_tree(k: int) -> list[int]:
    """Parents of the top-2 chain tree of depth k: node 0 the last emitted token, then per depth
    i = 1 .. k the chain's token c_i (node 2i - 1) and its runner-up s_i (node 2i), both children
    of c_{i-1} (of the root for i = 1).  M = 2k + 1 nodes: the drafter's best guess at every
    position plus the alternative that a chain drafter throws away."""
    par = [-1]
    for i in range(1, k + 1):
        p = 0 if i == 1 else 2 * i - 3
        par += [p, p]
    return par


class MTPDrafter:
    """Chains the MTP head K times (skinny_mlx/spec.py:54-95), scoring drafts over a seeded
    subset of `vocab` token ids (32768 seeded ids; the reference uses the id
    prefix [:vocab]).  Verify always uses the full head, so output is unchanged."""

    def __init__(self, model, head, vocab: int | None = 32768, seed: int = 0):
        from .model import QuantizedLinear

        from .patch import SkinnyQuantizedLinear

        self.model, self.head = model, head
        # a patched head runs on the fused kernels (its module forward is kept for the prompt)
        if isinstance(head.fc, SkinnyQuantizedLinear):
            from .mtp import FusedMTPHead

            self._fwd = FusedMTPHead(head, model.embed_tokens)
        else:
            self._fwd = head
        emb = model.embed_tokens
        V = emb.weight.shape[0]
        if vocab and vocab < V:
            gen = torch.Generator(device="cpu").manual_seed(seed)
            self.ids = torch.randperm(V, generator=gen)[:vocab].sort().values.to(model.device)
        else:
            self.ids = torch.arange(V, device=model.device)
        w, s, b = emb.weight[self.ids], emb.scales[self.ids], emb.biases[self.ids]
        if hasattr(emb, "skinny_head"):  # patched model: the pruned head runs on the same kernel
            from .patch import _qmm
            from .qmm import repack_for_skinny

            rw = repack_for_skinny(w.contiguous(), s.contiguous(), b.contiguous())
            self._logits = lambda h: _qmm(h, rw)
        else:
            ql = QuantizedLinear(w.contiguous(), s.contiguous(), b.contiguous())
            self._logits = ql

    def _step(self, tokens: torch.Tensor, hidden: torch.Tensor) -> torch.Tensor:
        return self._fwd(self.model.embed_tokens(tokens), hidden, self.cache)

    def begin(self, prompt: list[int], h: torch.Tensor, first: int) -> None:
        self.cache = self.head.make_cache()
        ids = torch.tensor(list(prompt[1:]) + [first], device=self.model.device)
        self.h_last = self._step(ids, h)[-1:]
        self.n_spec = 0

    def draft(self, k: int) -> torch.Tensor:
        toks, h = [], self.h_last
        for i in range(k):  # no host sync: the chain feeds verify directly
            t = self.ids[torch.argmax(self._logits(h[-1:]).float(), dim=-1)]
            toks.append(t)
            if i < k - 1:
                h = self._step(t, h[-1:])
        self.n_spec = k - 1
        return torch.cat(toks).to(torch.int32)

    def update(self, h_kept: torch.Tensor, new_tokens: list[int]) -> None:
        self.cache.trim(self.n_spec)
        self.h_last = self._step(torch.tensor(new_tokens, device=self.model.device), h_kept)[-1:]
        self.n_spec = 0

    def draft_tree(self, k: int) -> tuple[torch.Tensor, list[int]]:
        """The top-2 chain tree (chain_tree): the K chained head steps of draft(), keeping each
        step's runner-up as a sibling of its chain token.  Returns (tokens of nodes 1 .. 2k,
        int32 on the device, parents of all 2k + 1 nodes)."""
        toks, h = [], self.h_last
        for i in range(k):
            top = torch.topk(self._logits(h[-1:]).float(), 2, dim=-1).indices[0]
            t2 = self.ids[top]
            toks.append(t2)
            if i < k - 1:
                h = self._step(t2[:1], h[-1:])
        self.n_spec = k - 1
        return torch.cat(toks).to(torch.int32), chain_tree(k)


class GraphedMTPDrafter(MTPDrafter):
    """MTPDrafter whose draft chain (K logits, argmaxes and K - 1 head steps) and whose update
    step (one per accepted count) are replayed from CUDA graphs, so a speculative step costs the
    host two replays instead of some 40 launches.  Needs a patched head (fused kernels).  The
    head's cache length lives on the device while a graph runs (advanced there between draft
    steps); the host copy is kept in step.  The prompt (begin) runs eagerly."""

    def __init__(self, model, head, vocab: int | None = 32768, seed: int = 0):
        from .mtp import FusedMTPHead

        super().__init__(model, head, vocab, seed)
        if not isinstance(self._fwd, FusedMTPHead):
            raise ValueError("GraphedMTPDrafter needs a patched head")
        dev, H = model.device, model.cfg.hidden
        self._h = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)      # h_last
        self._hk = torch.zeros(17, H, dtype=torch.bfloat16, device=dev)    # kept hidden rows
        self._ids_in = torch.zeros(17, dtype=torch.long, device=dev)
        self._ids_host = torch.zeros(17, dtype=torch.long).pin_memory()
        self._toks = torch.zeros(16, dtype=torch.int32, device=dev)
        self._len = torch.zeros(1, dtype=torch.int32, device=dev)
        self._len_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._evt = torch.cuda.Event()
        self._stream = torch.cuda.Stream(dev)
        self._graphs: dict = {}

    def begin(self, prompt: list[int], h: torch.Tensor, first: int) -> None:
        # one head cache for every run of this drafter: the graphs hold its buffers
        if getattr(self, "cache", None) is None:
            self.cache = self.head.make_cache()
        self.cache.length = 0
        ids = torch.tensor(list(prompt[1:]) + [first], device=self.model.device)
        self.h_last = self._step(ids, h)[-1:]
        self.n_spec = 0
        self._h.copy_(self.h_last)

    # -- graph bodies (captured on self._stream; cache = the head's cache)
    def _draft_body(self, k: int, cache) -> None:
        h = self._h
        for i in range(k):
            t = self.ids[torch.argmax(self._logits(h).float(), dim=-1)]
            self._toks[i:i + 1].copy_(t)
            if i < k - 1:
                h = self._fwd.step_ids(t, h, cache, self._len)[-1:]
                self._len.add_(1)

    def _update_body(self, m: int, cache) -> None:
        out = self._fwd.step_ids(self._ids_in[:m], self._hk[:m], cache, self._len)
        self._h.copy_(out[-1:])

    def _capture(self, key, body):
        # warm-up on a scratch cache of the same size (buffers, workspaces), then capture
        scratch = self.head.make_cache(self.cache.k.shape[0])
        self._stream.wait_stream(torch.cuda.current_stream(self.model.device))
        saved = self._h.clone()
        with torch.cuda.stream(self._stream):
            body(scratch)
        self._stream.synchronize()
        self._h.copy_(saved)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self._stream):
            body(self.cache)
        self._graphs[key] = (g, self.cache)
        return g

    def _graph(self, key, body):
        ent = self._graphs.get(key)
        if ent is not None and ent[1] is self.cache:
            return ent[0]
        return self._capture(key, body)

    def _set_len(self) -> None:
        self._evt.synchronize()  # the previous copy out of the pinned word is done
        self._len_host[0] = self.cache.length
        self._len.copy_(self._len_host, non_blocking=True)
        self._evt.record()

    def draft(self, k: int) -> torch.Tensor:
        g = self._graph(("d", k), lambda c: self._draft_body(k, c))
        self._set_len()
        g.replay()
        self.cache.length += k - 1
        self.n_spec = k - 1
        return self._toks[:k]

    def update(self, h_kept: torch.Tensor, new_tokens: list[int]) -> None:
        self.cache.trim(self.n_spec)
        m = len(new_tokens)
        self._evt.synchronize()
        self._ids_host[:m] = torch.tensor(new_tokens, dtype=torch.long)
        self._ids_in[:m].copy_(self._ids_host[:m], non_blocking=True)
        self._hk[:m].copy_(h_kept)
        g = self._graph(("u", m), lambda c: self._update_body(m, c))
        self._set_len()
        g.replay()
        self.cache.length += m
        self.n_spec = 0

    def draft_tree(self, k: int):
        raise NotImplementedError("tree drafts use the eager MTPDrafter (the graphs replay a chain)")


class PromptLookupDrafter:
    """Model-free drafter (skinny_mlx/spec.py:32-51): proposes the up to K tokens that followed the
    latest earlier occurrence of the context's trailing n-gram, for n = ngram down to 1 (none if
    no n-gram recurs).  Every n-gram's two latest start positions are indexed as tokens arrive,
    so a draft costs O(ngram) instead of a scan of the context."""

    def __init__(self, ngram: int = 3, device=None):
        self.ngram, self.device = ngram, device

    def begin(self, prompt, h, first) -> None:
        if self.device is None and h is not None:
            self.device = h.device
        self.ctx: list[int] = []
        self.pos = [dict() for _ in range(self.ngram + 1)]  # n -> {n-gram: (latest start, previous)}
        for t in list(prompt) + [int(first)]:
            self._push(t)

    def _push(self, tok: int) -> None:
        self.ctx.append(int(tok))
        L = len(self.ctx)
        for n in range(1, min(self.ngram, L) + 1):
            key = tuple(self.ctx[L - n:])
            prev = self.pos[n].get(key)
            self.pos[n][key] = (L - n, prev[0] if prev else None)

    def draft(self, k: int) -> torch.Tensor:
        ctx, L = self.ctx, len(self.ctx)
        for n in range(self.ngram, 0, -1):
            if L < n + 1:
                continue
            ent = self.pos[n].get(tuple(ctx[L - n:]))  # ent[0] is the trailing n-gram itself
            if ent is not None and ent[1] is not None:
                s = ent[1]
                return torch.tensor(ctx[s + n: s + n + k], dtype=torch.int32).to(self.device, non_blocking=True)
        return torch.empty(0, dtype=torch.int32, device=self.device)

    def update(self, h_kept, new_tokens) -> None:
        for t in new_tokens:
            self._push(t)


class ScriptedDrafter:
    """Drafts a known greedy continuation `ref`, each proposal replaced by a wrong token with
    probability 1 - p (seeded): speculative decoding at a chosen acceptance rate.  With random
    weights an MTP head accepts almost nothing, so this stands in for a trained head when the
    speculative machinery is timed (K = 2 at p = 0.81 gives the reference's 2.51 tokens/step,
    docs/flatspec-design.md:60-61)."""

    def __init__(self, ref: list[int], p: float, vocab: int, device, seed: int = 0):
        self.ref, self.p, self.vocab, self.device = ref, p, vocab, device
        self.rng = torch.Generator().manual_seed(seed)

    def begin(self, prompt, h, first) -> None:
        self.pos = 1  # ref[0] is emitted by the prefill

    def draft(self, k: int) -> torch.Tensor:
        toks = []
        for i in range(k):
            j = self.pos + i
            t = self.ref[j] if j < len(self.ref) else 0
            if float(torch.rand((), generator=self.rng)) >= self.p:
                t = (t + 1) % self.vocab
            toks.append(t)
        return torch.tensor(toks, dtype=torch.int32).to(self.device, non_blocking=True)

    def update(self, h_kept, new_tokens) -> None:
        self.pos += len(new_tokens)


class ScriptedTreeDrafter:
    """The top-2 chain tree (chain_tree) over a known greedy continuation `ref`: each chain token
    is right with probability p (seeded); where it is wrong, its sibling is right with
    probability p, else both are wrong.  Speculative decoding with a tree at a chosen acceptance
    rate; compare ScriptedDrafter at the same p (the chain alone)."""

    def __init__(self, ref: list[int], p: float, vocab: int, device, seed: int = 0):
        self.ref, self.p, self.vocab, self.device = ref, p, vocab, device
        self.rng = torch.Generator().manual_seed(seed)

    def begin(self, prompt, h, first) -> None:
        self.pos = 1

    def draft_tree(self, k: int) -> tuple[torch.Tensor, list[int]]:
        toks = []
        for i in range(k):
            j = self.pos + i
            t = self.ref[j] if j < len(self.ref) else 0
            chain_ok = float(torch.rand((), generator=self.rng)) < self.p
            sib_ok = not chain_ok and float(torch.rand((), generator=self.rng)) < self.p
            c = t if chain_ok else (t + 1) % self.vocab
            sib = t if sib_ok else (t + 2) % self.vocab
            toks += [c, sib]
        return torch.tensor(toks, dtype=torch.int32).to(self.device, non_blocking=True), chain_tree(k)

    def update(self, h_kept, new_tokens) -> None:
        self.pos += len(new_tokens)


def _fresh_cache(model, cache):
    if cache is None:
        return model.make_cache()
    cache.reset()
    return cache


def greedy(model, prompt: list[int], max_tokens: int, gaps: list | None = None, cache=None) -> list[int]:
    """Plain greedy decoding, one token per forward (skinny_mlx/spec.py:98-107).  `gaps`, when
    given, receives each step's (top1 - top2 logit gap, top1 logit), for the near-tie check.
    `cache` (optional) is reset and reused, e.g. to keep a graph-replayed step's buffers."""
    cache = _fresh_cache(model, cache)
    _, logits = model(torch.tensor(prompt, device=model.device), cache)
    toks = []
    last = logits[-1]
    for i in range(max_tokens):
        if gaps is not None:
            t2 = torch.topk(last.float(), 2).values
            gaps.append((float(t2[0] - t2[1]), float(t2[0])))
        # the token stays on the device and feeds the next step there: no host round trip per
        # token (argmax returns the first maximal index, as the reference's does)
        y = torch.argmax(last).view(1)
        toks.append(y)
        if i + 1 == max_tokens:
            break
        _, logits = model(y, cache)
        last = logits[-1]
    return torch.cat(toks).tolist()


def speculative(model, prompt: list[int], max_tokens: int, drafter, k: int, stats: dict | None = None,
                cache=None) -> list[int]:
    """Greedy-exact speculative decoding (skinny_mlx/spec.py:110-156): each step verifies
    [last token] + K drafts in one forward (M = K+1), accepts the longest matching prefix on the
    device, emits one bonus token and rolls the hybrid cache back to the accepted prefix.
    `cache` (optional) is reset and reused."""
    cache = _fresh_cache(model, cache)
    rb = HybridRollback()
    h, logits = model(torch.tensor(prompt, device=model.device), cache)
    out = [int(torch.argmax(logits[-1].float()))]
    drafter.begin(prompt, h, out[0])
    steps = accepted = 0
    while len(out) < max_tokens:
        draft = drafter.draft(k)  # up to k tokens (a model-free drafter may propose fewer)
        x = torch.cat([torch.tensor([out[-1]], dtype=torch.int32, device=model.device), draft])
        rb.record(cache)
        h, logits = model(x.long(), cache)
        n, new = _accept_any(logits, draft)
        rb.rollback(cache, fed=x.numel(), keep=n + 1)
        drafter.update(h[: n + 1], new)
        out += new
        steps += 1
        accepted += n
    if stats is not None:
        stats.update(steps=steps, tokens_per_step=len(out) / max(steps, 1), accepted=accepted)
    return out[:max_tokens]


def speculative_tree(model, prompt: list[int], max_tokens: int, drafter, k: int, stats: dict | None = None,
                     cache=None) -> list[int]:
    """Greedy-exact speculative decoding with a draft TREE verified in one forward (the wider
    drafts the reference proposes to fill the flat-verify budget, docs/flatspec-design.md:64-69):
    each step the drafter proposes tree nodes (draft_tree(k) -> node tokens, parents), the model
    verifies [last token] + nodes with tree attention and a branch-aware GDN recurrence, the
    device walks the tree along the model's own predictions, and the cache keeps the accepted
    path.  `model` is a HybridModel (module path) or its FusedStep / GraphedStep."""
    cache = _fresh_cache(model, cache)
    rb = HybridRollback()
    h, logits = model(torch.tensor(prompt, device=model.device), cache)
    out = [int(torch.argmax(logits[-1].float()))]
    drafter.begin(prompt, h, out[0])
    steps = accepted = 0
    while len(out) < max_tokens:
        nodes, parent = drafter.draft_tree(k)
        x = torch.cat([torch.tensor([out[-1]], dtype=torch.int32, device=model.device), nodes])
        rb.record(cache)
        h, logits = model(x.long(), cache, tree=parent)
        n, new, path = _accept_tree_any(logits, x, parent)
        rb.rollback_tree(cache, fed=x.numel(), path=path)
        drafter.update(h[path[0]:path[0] + 1] if n == 0 else h[torch.tensor(path, device=h.device)], new)
        out += new
        steps += 1
        accepted += n
    if stats is not None:
        stats.update(steps=steps, tokens_per_step=len(out) / max(steps, 1), accepted=accepted)
    return out[:max_tokens]


__all__ += ["HybridRollback", "MTPDrafter", "GraphedMTPDrafter", "PromptLookupDrafter", "ScriptedDrafter",
            "ScriptedTreeDrafter", "chain_tree", "greedy", "speculative", "speculative_tree"]
