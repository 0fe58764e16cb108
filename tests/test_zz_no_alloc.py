"""The allocation-free decode attention (vox_cuda_attention_decode_noalloc).

Callers that cannot allocate device memory (hosts that forbid cudaMalloc once
running) use this entry point; its scratch is a fixed device array inside the
library.  This file is collected last so that a run that stops at the first
failure has run every other test already; it also passes on its own in a
fresh process (the entry point needs no vox_cuda_init).
"""
import numpy as np
import pytest

import bind as B
import gen_golden as G
import voxcuda as V

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-5   # the tolerance the decode-attention parity tests use


def _run(fn, q, k, v, cap, pos, torch):
    out = torch.empty(B.Q_DIM, dtype=torch.float32, device="cuda")
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), cap, pos, out.data_ptr(), None)
    assert rc == 0, V.last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("L,slot,seed", [(777, -1, 46), (8192, 5000, 44)])
def test_noalloc_matches_allocating_entry_twice(L, slot, seed):
    import torch
    torch.cuda.set_device(0)
    lib = V.lib()
    q, k, v = G.attn_decode_inputs(L, seed)
    cap, pos = (L, L + slot) if slot >= 0 else (L, L - 1)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    # two calls in a row: the static scratch keeps the first call's contents
    a1 = _run(lib.vox_cuda_attention_decode_noalloc, dq, dk, dv, cap, pos, torch)
    a2 = _run(lib.vox_cuda_attention_decode_noalloc, dq, dk, dv, cap, pos, torch)
    V.init(0)
    ref = _run(lib.vox_cuda_attention_decode_dev, dq, dk, dv, cap, pos, torch)
    assert B.rel_l2(a1, ref) < ATTN_TOL
    assert B.rel_l2(a2, ref) < ATTN_TOL
    # a different, shorter window after a full one: stale partials are not read
    q2, k2, v2 = G.attn_decode_inputs(100, 7)
    d2 = [torch.from_numpy(a).cuda() for a in (q2, k2, v2)]
    b1 = _run(lib.vox_cuda_attention_decode_noalloc, *d2, 100, 99, torch)
    bref = _run(lib.vox_cuda_attention_decode_dev, *d2, 100, 99, torch)
    assert B.rel_l2(b1, bref) < ATTN_TOL


def test_noalloc_on_a_caller_stream_and_each_visible_device():
    """A stream handle from the caller, and - where more than one GPU is
    visible - the same call on every device (each looks up its own copy of
    the array), against the allocating entry point."""
    import torch
    lib = V.lib()
    q, k, v = G.attn_decode_inputs(512, 41)
    for dev in range(torch.cuda.device_count()):
        torch.cuda.set_device(dev)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        s = torch.cuda.Stream()
        out = torch.empty(B.Q_DIM, dtype=torch.float32, device="cuda")
        rc = lib.vox_cuda_attention_decode_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), 512, 511,
                                                   out.data_ptr(), s.cuda_stream)
        assert rc == 0, V.last_error()
        got = out.cpu().numpy()
        V.check(lib.vox_cuda_set_device(dev), "set_device")
        V.init(dev)
        ref = _run(lib.vox_cuda_attention_decode_dev, dq, dk, dv, 512, 511, torch)
        assert B.rel_l2(got, ref) < ATTN_TOL, dev
    torch.cuda.set_device(0)
    V.check(lib.vox_cuda_set_device(0), "set_device")


def test_noalloc_rejects_a_ring_smaller_than_the_window():
    import torch
    z = torch.zeros(16 * B.KV_DIM, dtype=torch.float32, device="cuda")
    q = torch.zeros(B.Q_DIM, dtype=torch.float32, device="cuda")
    rc = V.lib().vox_cuda_attention_decode_noalloc(q.data_ptr(), z.data_ptr(), z.data_ptr(), 16, 16,
                                                   q.data_ptr(), None)
    assert rc == V.ERR_CAPACITY
    assert "cannot hold" in V.last_error()
