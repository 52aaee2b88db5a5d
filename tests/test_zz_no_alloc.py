"""The allocation-free window-attention entry point (fsattn_window_prefill_static) against the regular one.

Some callers may not create device memory when they need a prefill (a frozen memory plan, a plugin that must leave its host
framework's allocator alone, a latency path that cannot take cudaMalloc's device synchronisation). For them the library
carries the kernel's scratch as a fixed array. This file is collected last on purpose: a run that stops at the first failure
has then already run every other test."""
import ctypes

import pytest
import torch

from oracle import fsl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _inputs(B, H, N, seed, dev):
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn(B, H, N, 64, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    return Q, K, V


def test_static_scratch_matches_regular_entry_point_twice(dev):
    from freesolo_b200 import ops
    cos, sin = (t.to(dev) for t in fsl.rope_tables(64, 4096, torch.bfloat16))
    # calls in a row with different shapes and data (a larger one, then smaller ones): a call must not see anything an
    # earlier one left in the shared array. The regular entry point runs the same kernel on a caller-owned workspace, so
    # the two must agree bit for bit; the oracle comparison catches a fault they would share.
    for B, H, N, pos0, seed in ((1, 2, 700, 0, 1), (2, 3, 1333, 64, 2), (1, 2, 300, 0, 3), (1, 1, 129, 7, 4)):
        Q, K, V = _inputs(B, H, N, seed, dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        want = ops.window_prefill(Q, K, V, cos, sin, 512, 0.125, pos0=pos0)
        got = ops.window_prefill_static(Q, K, V, cos, sin, 512, 0.125, pos0=pos0, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.equal(got, want), f"B={B} H={H} N={N}: the static-scratch call differs from the regular entry point"
        ref = fsl.window_attention(Q.cpu().float(), K.cpu().float(), V.cpu().float(), cos.cpu(), sin.cpu(), 512, 0.125,
                                   q_pos0=pos0, k_pos0=pos0, act_dtype=torch.bfloat16).to(torch.bfloat16)
        d = (got.view(B, N, H, 64).transpose(1, 2).float().cpu() - ref.float()).abs()
        assert d.max().item() <= 2e-2 and (d.mean() / ref.float().abs().mean()).item() <= 1e-3, \
            f"B={B} H={H} N={N} vs oracle: max-abs {d.max().item():.3e}, mean-rel {(d.mean() / ref.float().abs().mean()).item():.3e}"


def test_static_scratch_rejects_what_it_cannot_hold(dev):
    from freesolo_b200 import lib as L, ops
    cos, sin = (t.to(dev) for t in fsl.rope_tables(64, 2048, torch.bfloat16))
    Q, K, V = _inputs(1, 1, 256, 3, dev)
    with pytest.raises(RuntimeError, match="multiples of 64"):
        ops.window_prefill_static(Q, K, V, cos, sin, 96, 0.125)
    # a shape beyond the built-in array is refused on the host before anything is launched (pointers are never touched)
    a = L.WindowPrefill()
    a.q = a.k = a.v = L.BHND(Q.data_ptr(), 0, 0, 64)
    a.cos, a.sin, a.out = cos.data_ptr(), sin.data_ptr(), Q.data_ptr()
    a.B, a.H, a.D, a.N, a.W, a.pos0 = 1, 16, 64, 131072, 512, 0
    rc = L.load().fsattn_window_prefill_static(ctypes.byref(a), None)
    assert rc == L.EINVAL and "built-in array" in L.last_error()
