"""GPU tests of skinny_qmm_w4g64_noalloc, the workspace-free entry whose scratch is a static device
array.  Collected last on purpose: it must give the same answers on a device where the other tests
already ran (module loaded, workspaces in use) as it does alone.

Each call goes through the C-ABI and is compared with the workspace entry skinny_qmm_w4g64 (via
skinny_qmm) within the usual tolerance, max|ref - got| / max|ref| <= 1.5e-2, and with the oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant

pytestmark = pytest.mark.gpu

TOL = 1.5e-2
SCRATCH_LIMIT = -9


def _weight(n, k, seed, dev):
    from skinny_mlx_b200.qmm import repack_for_skinny

    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, s, b = quant.quantize(w)
    tw = torch.from_numpy(packed.view(np.int32)).to(dev)
    ts = torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).to(dev)
    tb = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev)
    return (packed, s, b), repack_for_skinny(tw, ts, tb)


def _noalloc(lib, x, sw, out):
    m, k = x.shape
    return lib.skinny_qmm_w4g64_noalloc(
        ctypes.c_void_p(x.data_ptr()), k, ctypes.c_void_p(sw.w_tc.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), out.shape[1], m, sw.N, sw.K,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("n,k,m", [(9728, 2560, 8), (2560, 9728, 16), (200, 192, 3), (151936, 2560, 1)])
def test_noalloc_matches_workspace_entry(cuda_lib, dev, n, k, m):
    from skinny_mlx_b200.qmm import skinny_qmm

    (packed, s, b), sw = _weight(n, k, 7, dev)
    rng = np.random.default_rng(70 + m)
    xb = quant.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    ref_entry = skinny_qmm(x, sw).float()
    outs = [torch.empty(m, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    for o in outs:  # two calls in a row on one stream, sharing the one static scratch
        assert _noalloc(cuda_lib, x, sw, o) == 0
    torch.cuda.synchronize()
    for o in outs:
        assert quant.rel_err(ref_entry.cpu().numpy(), o.float().cpu().numpy()) <= TOL
    assert torch.equal(outs[0], outs[1])
    if n * k <= 9728 * 2560:
        ref = quant.qmm_ref(quant.bf16_bits_to_f32(xb), packed, s, b)
        assert quant.rel_err(ref, outs[1].float().cpu().numpy()) <= TOL


def test_noalloc_rejects_shapes_over_the_scratch(cuda_lib, dev):
    x = torch.zeros(1, 64, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(4608, dtype=torch.uint8, device=dev)
    out = torch.zeros(1, 64, dtype=torch.bfloat16, device=dev)
    st = cuda_lib.skinny_qmm_w4g64_noalloc(
        ctypes.c_void_p(x.data_ptr()), 64, ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), 2048 * 128 + 1, 1, 2048 * 128 + 1, 64,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == SCRATCH_LIMIT
    assert b"262144" in cuda_lib.skinny_strerror(st)
    # K over the x-prep capacity of the scratch (512 groups of 64 columns); checked on the host,
    # nothing is read through these pointers
    kbig = 513 * 64
    st = cuda_lib.skinny_qmm_w4g64_noalloc(
        ctypes.c_void_p(x.data_ptr()), kbig, ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), 64, 1, 64, kbig,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == SCRATCH_LIMIT


def test_noalloc_shape_switch_and_error_word(cuda_lib, dev):
    """Different shapes back to back on one stream, sharing the scratch: a cluster split-K shape
    (fewer tiles than SMs), a stream-K shape whose tiles straddle CTAs (it uses the scratch's
    per-tile arrival counters, which every call clears first), a tail shape, then the first shape
    again.  Each result equals the oracle; after each call the error word, copied out by
    skinny_qmm_w4g64_noalloc_errors into device memory and into pinned host memory, is 0."""
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    err_dev = torch.full((1,), -1, dtype=torch.int32, device=dev)
    err_host = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    for i, (n, k, m) in enumerate([(2560, 9728, 8), (20000, 256, 16), (200, 192, 3), (2560, 9728, 8)]):
        (packed, s, b), sw = _weight(n, k, 90 + i % 3, dev)
        rng = np.random.default_rng(900 + i)
        xb = quant.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
        x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
        out = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        assert _noalloc(cuda_lib, x, sw, out) == 0
        assert cuda_lib.skinny_qmm_w4g64_noalloc_errors(ctypes.c_void_p(err_dev.data_ptr()), stream) == 0
        assert cuda_lib.skinny_qmm_w4g64_noalloc_errors(ctypes.c_void_p(err_host.data_ptr()), stream) == 0
        torch.cuda.synchronize()
        assert int(err_dev.item()) == 0 and int(err_host.item()) == 0
        ref = quant.qmm_ref(quant.bf16_bits_to_f32(xb), packed, s, b)
        assert quant.rel_err(ref, out.float().cpu().numpy()) <= TOL, (n, k, m)
        err_dev.fill_(-1)
        err_host.fill_(-1)
    assert cuda_lib.skinny_qmm_w4g64_noalloc_errors(None, stream) == -1
