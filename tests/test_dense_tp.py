"""Config 5: the column-parallel dense model.  On CPU, 2 gloo ranks against the unsharded model;
on one GPU, the patched unsharded model against the unpatched one."""

import os

import pytest
import torch
import torch.multiprocessing as mp

from oracle.checks import argmax_violations
from skinny_mlx_b200.dense import DenseModel, small_dense

IDS = [5, 17, 300, 4000, 9, 2222, 123, 77]


def _free_port() -> int:
    """A TCP port on 127.0.0.1 that nothing listens on now (rendezvous of the spawned ranks)."""
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        m = DenseModel(small_dense(), rank, world, seed=3, device="cpu")
        caches = m.make_cache(64)
        m(torch.tensor(IDS[:5]), caches)
        logits = m(torch.tensor(IDS[5:]), caches)
        if rank == 0:
            q.put(logits.float())
    finally:
        dist.destroy_process_group()


def test_column_parallel_equals_unsharded_on_cpu():
    ref_m = DenseModel(small_dense(), 0, 1, seed=3, device="cpu")
    caches = ref_m.make_cache(64)
    ref_m(torch.tensor(IDS[:5]), caches)
    ref = ref_m(torch.tensor(IDS[5:]), caches).float()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # the same rows of the same weights, the same f32 arithmetic per output column
    assert torch.allclose(got, ref, atol=1e-5, rtol=0), (got - ref).abs().max()


@pytest.mark.gpu
def test_dense_patched_matches_unpatched(cuda_lib, dev):
    from skinny_mlx_b200.model import QuantizedLinear
    from skinny_mlx_b200.patch import patch_model

    m = DenseModel(small_dense(), 0, 1, seed=3, device=dev)

    def run():
        caches = m.make_cache(64)
        m(torch.tensor(IDS[:5], device=dev), caches)
        return m(torch.tensor(IDS[5:], device=dev), caches).float()

    rel = lambda a, b: ((a - b).abs().max() / a.abs().max()).item()
    ref = run()
    QuantizedLinear.accumulate = torch.float64
    try:
        floor = rel(ref, run())
    finally:
        QuantizedLinear.accumulate = torch.float32
    stats = patch_model(m)
    assert stats["single"] == 2 * 4 + 1 and stats["fused_groups"] == 0
    got = run()
    assert rel(ref, got) <= max(1.5e-2, 3 * floor), (rel(ref, got), floor)


def _gpu_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from skinny_mlx_b200.patch import patch_model

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        m = DenseModel(small_dense(), rank, world, seed=3, device=f"cuda:{rank}")
        patch_model(m)
        caches = m.make_cache(64)
        m(torch.tensor(IDS[:5], device=f"cuda:{rank}"), caches)
        logits = m(torch.tensor(IDS[5:], device=f"cuda:{rank}"), caches).float().cpu()
        if rank == 0:
            q.put(logits)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_column_parallel_nccl_two_gpus(cuda_lib, dev):
    """2 ranks over NCCL (skipped on a 1-GPU box): sharded logits vs the unsharded patched model."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from skinny_mlx_b200.patch import patch_model

    m = DenseModel(small_dense(), 0, 1, seed=3, device=dev)
    patch_model(m)
    caches = m.make_cache(64)
    m(torch.tensor(IDS[:5], device=dev), caches)
    ref = m(torch.tensor(IDS[5:], device=dev), caches).float().cpu()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # per-row results of the same kernel; stream-K split points differ with the shard sizes
    assert ((ref - got).abs().max() / ref.abs().max()).item() <= 1e-2
    assert not argmax_violations(ref.numpy(), got.numpy())


def _full(logits_shards: torch.Tensor) -> torch.Tensor:
    """[G, M, V/G] rank-major vocabulary shards -> [M, V]."""
    G, M, n = logits_shards.shape
    return logits_shards.permute(1, 0, 2).reshape(M, G * n)


@pytest.mark.gpu
def test_dense_fused_step_matches_module_path(cuda_lib, dev):
    """The fused dense step (prep / prepared qmm / ungated fused attention) against the patched
    module-by-module forward of the same model, prefill then a 3-token verify."""
    from skinny_mlx_b200.dense_fused import DenseFusedStep
    from skinny_mlx_b200.patch import patch_model

    m = DenseModel(small_dense(), 0, 1, seed=3, device=dev)
    patch_model(m)
    f = DenseFusedStep(m)
    ca, cb = m.make_cache(64), m.make_cache(64)
    for ids in (IDS[:5], IDS[5:]):
        t = torch.tensor(ids, device=dev)
        ref = m(t, ca).float()
        got = _full(f(t, cb)).float()
        assert ((ref - got).abs().max() / ref.abs().max()).item() <= 1.5e-2
        assert not argmax_violations(ref.cpu().numpy(), got.cpu().numpy())
    assert [c.length for c in ca] == [c.length for c in cb]


def _gpu_fused_rank(rank, world, port, q, exchange):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    f = None
    try:
        from skinny_mlx_b200.dense_fused import DenseFusedStep
        from skinny_mlx_b200.patch import patch_model

        m = DenseModel(small_dense(), rank, world, seed=3, device=f"cuda:{rank}")
        patch_model(m)
        f = DenseFusedStep(m, exchange=exchange)
        caches = m.make_cache(64)
        out = []
        # prefill, then verify steps of 3, 1 and 16 tokens: every step advances the epoch
        for ids in (IDS[:5], IDS[5:], IDS[:1], (IDS * 2)[:16]):
            out.append(_full(f(torch.tensor(ids, device=f"cuda:{rank}"), caches)).float().cpu())
        errs = f.errors()
        if rank == 0:
            q.put((out, errs))
    finally:
        if f is not None:
            f.release()
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_dense_fused_step_multi_gpu(cuda_lib, dev, exchange, world):
    """2, 4 and 8 ranks (skipped on a box with fewer GPUs): the fused sharded step against the
    unsharded patched module path, with the peer-memory exchange (digit blocks pushed into every
    rank's buffer, output shards read in place over NVLink, per-layer flags) and with NCCL
    all-gathers."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from skinny_mlx_b200.patch import patch_model

    m = DenseModel(small_dense(), 0, 1, seed=3, device=dev)
    patch_model(m)
    caches = m.make_cache(64)
    refs = [m(torch.tensor(ids, device=dev), caches).float().cpu()
            for ids in (IDS[:5], IDS[5:], IDS[:1], (IDS * 2)[:16])]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_fused_rank, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    got, errs = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert errs == 0
    for ref, g in zip(refs, got):
        assert ((ref - g).abs().max() / ref.abs().max()).item() <= 1.5e-2
        assert not argmax_violations(ref.numpy(), g.numpy())


@pytest.mark.gpu
def test_peer_wait_gives_up_and_records(cuda_lib, dev):
    """A consumer whose flag no producer sets: the bounded wait gives up (about a second), sets
    its error bit, and the context stays usable (the digits are still written)."""
    import ctypes

    from skinny_mlx_b200 import _lib

    K, M = 256, 4
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    xq = torch.zeros(int(_lib.lib().skinny_xq_bytes(M, K)), dtype=torch.uint8, device=dev)
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    flags = torch.zeros(2, dtype=torch.int32, device=dev)  # nothing ever stores the epoch here
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    s = _lib.PeerSync()
    s.epoch, s.wait_flags, s.err, s.n_ranks = epoch.data_ptr(), flags.data_ptr(), err.data_ptr(), 2
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.call("skinny_prep", 2, ctypes.c_void_p(x.data_ptr()), K, None, 0, 0, None, None, 0, None, 0.0, M, K,
              ctypes.c_void_p(xq.data_ptr()), None, ctypes.byref(s), stream)
    torch.cuda.synchronize(dev)
    assert int(err.item()) & (1 << 11)
    ref = torch.zeros_like(xq)
    _lib.call("skinny_prep", 2, ctypes.c_void_p(x.data_ptr()), K, None, 0, 0, None, None, 0, None, 0.0, M, K,
              ctypes.c_void_p(ref.data_ptr()), None, None, stream)
    torch.cuda.synchronize(dev)
    assert torch.equal(xq, ref)


@pytest.mark.gpu
def test_prep_mirrors_digits_and_signals(cuda_lib, dev):
    """A digit producer with mirror destinations (the sharded step's push of digit blocks into
    the other ranks' buffers), here two local buffers: every copy equals the plain output, and
    the launch's last CTA stores the epoch into every signal flag."""
    import ctypes

    from skinny_mlx_b200 import _lib

    K, M = 1024, 5
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    x = torch.randn(M, 2 * K, device=dev).to(torch.bfloat16)
    n = int(_lib.lib().skinny_xq_bytes(M, K))
    ref, own, m1, m2 = (torch.zeros(n, dtype=torch.uint8, device=dev) for _ in range(4))
    epoch = torch.full((1,), 7, dtype=torch.int32, device=dev)
    counter = torch.zeros(1, dtype=torch.int32, device=dev)
    flags = torch.zeros(3, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    s = _lib.PeerSync()
    s.epoch, s.counter, s.err, s.n_ranks = epoch.data_ptr(), counter.data_ptr(), err.data_ptr(), 3
    for r in range(3):
        s.signal_flags[r] = flags.data_ptr() + 4 * r
    s.mirror[0], s.mirror[1], s.n_mirror = m1.data_ptr(), m2.data_ptr(), 2
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    _lib.call("skinny_prep", 1, P(x), 2 * K, None, 0, 0, None, None, 0, None, 0.0, M, K, P(ref), None, None, stream)
    _lib.call("skinny_prep", 1, P(x), 2 * K, None, 0, 0, None, None, 0, None, 0.0, M, K, P(own), None,
              ctypes.byref(s), stream)
    torch.cuda.synchronize(dev)
    for buf in (own, m1, m2):
        assert torch.equal(buf, ref)
    assert flags.tolist() == [7, 7, 7] and int(counter.item()) == 0 and int(err.item()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("m", [3, 12])
def test_prepared_qmm_reads_digit_blocks_from_rank_buffers(cuda_lib, dev, m):
    """The prepared qmm's per-rank input (xq_ranks, groups_per_rank): group g's digit block comes
    from buffer g / groups_per_rank, at the offset it has in a full buffer.  Two local buffers
    stand in for two ranks, each holding only its own slice (the rest zero): the result equals
    the call on the full buffer bit for bit."""
    import ctypes

    from skinny_mlx_b200 import _lib
    from skinny_mlx_b200.qmm import get_workspace, quantize, repack_for_skinny

    torch.manual_seed(m)
    K, N = 1024, 640
    G, gpr = K // 64, K // 64 // 2
    w = repack_for_skinny(*quantize(torch.randn(N, K, device=dev) * 0.02))
    ws = get_workspace(dev, int(cuda_lib.skinny_qmm_workspace_bytes(N, K)))
    x = torch.randn(m, K, device=dev).to(torch.bfloat16)
    xq = torch.zeros(int(cuda_lib.skinny_xq_bytes(m, K)), dtype=torch.uint8, device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    assert cuda_lib.skinny_prep(2, P(x), K, None, 0, 0, None, None, 0, None, ctypes.c_float(0), m, K, P(xq), None, None,
                                stream) == 0
    xb = int(cuda_lib.skinny_xq_bytes(m, 64))
    r0, r1 = torch.zeros_like(xq), torch.zeros_like(xq)
    r0[:gpr * xb] = xq[:gpr * xb]
    r1[gpr * xb:] = xq[gpr * xb:]
    y_full = torch.empty(m, N, dtype=torch.bfloat16, device=dev)
    y_ranks = torch.empty_like(y_full)
    assert cuda_lib.skinny_qmm_w4g64_prepared(P(xq), P(w.w_tc), P(y_full), N, m, N, K, P(ws), ws.numel(), None, 0,
                                                 None, stream) == 0
    ranks = (ctypes.c_void_p * 8)(r0.data_ptr(), r1.data_ptr())
    assert cuda_lib.skinny_qmm_w4g64_prepared(None, P(w.w_tc), P(y_ranks), N, m, N, K, P(ws), ws.numel(), ranks, gpr,
                                                 None, stream) == 0
    torch.cuda.synchronize(dev)
    assert torch.equal(y_full, y_ranks)
    assert G == 2 * gpr
