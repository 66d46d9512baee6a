"""The allocation-free decode-attention entry point against the regular one.

ylm_k_decode_attention_noalloc serves callers that cannot allocate device
memory: it keeps its scratch in a fixed array inside the library instead of
allocating per call. This file is named to be collected last, so a run that
stops at the first failure has already run every other test; it also passes on
its own in a fresh process (the first call on the device does the one-time
look-up of that array)."""
import ctypes

import numpy as np
import pytest

from yalama_b200 import engine as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

# same tolerance as the decode-attention parity test; the two entry points run
# the same kernel, so in practice they agree bit for bit
TOL = 2e-3


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _tables(max_pos, theta=1e6):
    inv = (1.0 / np.power(np.float64(np.float32(theta)),
                          (np.arange(64, dtype=np.float32) / np.float32(64)).astype(np.float64))).astype(np.float32)
    ang = (np.arange(max_pos, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return (torch.from_numpy(np.cos(ang.astype(np.float64)).astype(np.float16)).cuda(),
            torch.from_numpy(np.sin(ang.astype(np.float64)).astype(np.float16)).cuda())


def _run_pair(hq, hkv, slot, norm):
    L = E.lib()
    D, cap, max_pos = 128, slot + 32, slot + 8
    g = torch.Generator().manual_seed(hq * 131 + slot)
    qkv = (torch.randn((hq + 2 * hkv) * D, generator=g) * 0.5).half().cuda()
    kc0 = (torch.randn(hkv, cap, D, generator=g) * 0.5).half().cuda()
    vc0 = torch.randn(hkv, cap, D, generator=g).half().cuda()
    qn = (1 + 0.1 * torch.randn(D, generator=g)).half().cuda() if norm else None
    kn = (1 + 0.1 * torch.randn(D, generator=g)).half().cuda() if norm else None
    cos, sin = _tables(max_pos)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    pos = slot - 1
    for call in range(2):  # two calls in a row: the fixed scratch keeps the previous contents
        kc_a, vc_a, kc_b, vc_b = kc0.clone(), vc0.clone(), kc0.clone(), vc0.clone()
        out_a = torch.empty(hq * D, dtype=torch.float16, device="cuda")
        out_b = torch.full((hq * D,), float("nan"), dtype=torch.float16, device="cuda")
        E.check(L.ylm_k_decode_attention(_ptr(qkv), _ptr(qn), _ptr(kn), 1e-6, _ptr(cos), _ptr(sin), max_pos,
                                         _ptr(kc_a), _ptr(vc_a), cap, hq, hkv, slot, pos, _ptr(out_a), stream),
                "ylm_k_decode_attention")
        E.check(L.ylm_k_decode_attention_noalloc(_ptr(qkv), _ptr(qn), _ptr(kn), 1e-6, _ptr(cos), _ptr(sin), max_pos,
                                                 _ptr(kc_b), _ptr(vc_b), cap, hq, hkv, slot, pos, _ptr(out_b),
                                                 stream), "ylm_k_decode_attention_noalloc")
        torch.cuda.synchronize()
        a, b = out_a.float().cpu().numpy(), out_b.float().cpu().numpy()
        assert np.all(np.isfinite(b)), call
        assert np.max(np.abs(a - b)) <= TOL, call
        assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b), call


CASES = [(24, 8, 767, False), (16, 8, 40, True), (28, 4, 5000, False)]


@pytest.mark.parametrize("hq,hkv,slot,norm", CASES)
def test_noalloc_matches_allocating_entry_point(hq, hkv, slot, norm):
    # the cluster kernel: the fixed array holds only the step state
    _run_pair(hq, hkv, slot, norm)


@pytest.mark.parametrize("hq,hkv,slot,norm", CASES)
def test_noalloc_matches_allocating_entry_point_split_kernel(hq, hkv, slot, norm):
    # the split-K kernel: the fixed array also holds the partials and the
    # KV-head tickets, which the previous call left behind
    with E.split_attention():
        _run_pair(hq, hkv, slot, norm)


def test_noalloc_rejects_null_buffers():
    L = E.lib()
    assert L.ylm_k_decode_attention_noalloc(None, None, None, 1e-6, None, None, 16, None, None, 8, 4, 2, 0, 0, None,
                                            None) == E.Status.INVALID_ARG


def test_noalloc_rejects_partials_beyond_its_scratch():
    # split-K partials of 4096 query heads over 512 KV heads (one split each):
    # 4096 x 130 floats > 2 MiB. The size check returns before any device
    # access, so the non-null placeholder pointers are never dereferenced.
    L = E.lib()
    p = ctypes.c_void_p(256)
    with E.split_attention():
        st = L.ylm_k_decode_attention_noalloc(p, None, None, 1e-6, p, p, 16, p, p, 8, 4096, 512, 0, 0, p, None)
    assert st == E.Status.UNSUPPORTED
