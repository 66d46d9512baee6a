"""Kernel-level parity through the C ABI on the GPU: the decode GEMV, the
prefill GEMM, one decode-attention step and the sampler, against FP32/FP64
numpy references and, for sampling, the oracle's bit-exact restatement."""
import ctypes

import numpy as np
import pytest

from yalama_b200 import engine as E
from oracle import sampler as S
from oracle.numerics import round_f16

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def fp16_tol(ref, mag, k):
    """One FP16 rounding of the result (half an ulp, taken as a full ulp) plus
    the FP32 accumulation error of a k-term dot product, 4 sqrt(k) 2^-24 sum|a_i b_i|
    (the probabilistic bound for round-to-nearest summation)."""
    ulp = np.maximum(np.abs(ref), 6.1e-5) * 2.0 ** -10
    return 1.01 * ulp + 4.0 * np.sqrt(k) * 2.0 ** -24 * mag


@pytest.mark.parametrize("n,k", [(5120, 3072), (3072, 8192), (16384, 3072), (1000, 1000), (17, 384), (3, 8),
                                 (151936, 1024), (4096, 14336)])
def test_gemv_matches_fp32(n, k):
    rng = np.random.default_rng(n * 7 + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = rng.standard_normal(k).astype(np.float16)
    wd, xd = dev(w), dev(x)
    y = torch.empty(n, dtype=torch.float16, device="cuda")
    E.check(E.lib().ylm_k_gemv(ptr(wd), n, k, ptr(xd), ptr(y), stream()), "gemv")
    torch.cuda.synchronize()
    ref = w.astype(np.float64) @ x.astype(np.float64)
    mag = np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64))
    got = y.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref) <= fp16_tol(ref, mag, k))


@pytest.mark.parametrize("tc", [1, 0])
# the last two have more tiles than SMs: each persistent CTA takes several
# tiles and reuses both TMEM accumulators (ragged in T, N and K)
@pytest.mark.parametrize("t,n,k", [(1, 64, 64), (37, 300, 256), (512, 1024, 3072), (128, 5120, 3072),
                                   (200, 16384, 1024), (129, 257, 136), (777, 9000, 320), (1024, 16384, 512)])
def test_gemm_matches_fp32(t, n, k, tc):
    rng = np.random.default_rng(t + n + k)
    a = rng.standard_normal((t, k)).astype(np.float16)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16)
    ad, wd = dev(a), dev(w)
    c = torch.empty((t, n), dtype=torch.float16, device="cuda")
    E.check(E.lib().ylm_k_gemm(ptr(ad), ptr(wd), t, n, k, ptr(c), tc, stream()), "gemm")
    torch.cuda.synchronize()
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    mag = np.abs(a.astype(np.float64)) @ np.abs(w.astype(np.float64)).T
    got = c.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(got - ref) <= fp16_tol(ref, mag, k))


@pytest.mark.parametrize("tc", [1, 0])
@pytest.mark.parametrize("hq,hkv,t,cap", [(16, 8, 37, 64), (24, 8, 512, 600), (28, 4, 1000, 1000), (8, 8, 1, 16),
                                           (64, 8, 130, 200), (4, 2, 65, 65), (32, 8, 2048, 2100),
                                           (8, 2, 257, 300)])
def test_prefill_attention_matches_fp32(hq, hkv, t, cap, tc):
    # causal attention over cache slots [0, t); slots past t hold NaN, which
    # must never reach the output (the reference never reads them either)
    rng = np.random.default_rng(hq * 7 + t)
    D = 128
    q = rng.standard_normal((t, hq * D)).astype(np.float16)
    kc = np.full((hkv, cap, D), np.nan, dtype=np.float16)
    vc = np.full((hkv, cap, D), np.nan, dtype=np.float16)
    kc[:, :t] = rng.standard_normal((hkv, t, D)).astype(np.float16)
    vc[:, :t] = rng.standard_normal((hkv, t, D)).astype(np.float16)
    qd, kd, vd = dev(q), dev(kc), dev(vc)
    out = torch.empty((t, hq * D), dtype=torch.float16, device="cuda")
    E.check(E.lib().ylm_k_prefill_attention(ptr(qd), ptr(kd), ptr(vd), cap, hq, hkv, t, ptr(out), tc, stream()),
            "prefill attention")
    torch.cuda.synchronize()
    qf = qd.float().reshape(t, hq, D).transpose(0, 1)                   # [hq, t, D]
    kf = kd[:, :t].float().repeat_interleave(hq // hkv, dim=0)          # [hq, t, D]
    vf = vd[:, :t].float().repeat_interleave(hq // hkv, dim=0)
    sc = (qf @ kf.transpose(1, 2)) / np.sqrt(D)
    mask = torch.triu(torch.ones(t, t, dtype=torch.bool, device="cuda"), 1)
    sc = sc.masked_fill(mask, float("-inf"))
    ref = (torch.softmax(sc, dim=-1) @ vf).transpose(0, 1).reshape(t, hq * D)
    got = out.float()
    assert torch.isfinite(got).all()
    # P is rounded to FP16 before P V (one rounding per probability), and the
    # output to FP16
    err = (got - ref).abs().max().item()
    assert err < 4e-3, err


def rope_tables(max_pos, theta=1e6):
    half = 64
    inv = (1.0 / np.power(np.float64(np.float32(theta)), (np.arange(half, dtype=np.float32) / np.float32(half))
                          .astype(np.float64))).astype(np.float32)
    ang = (np.arange(max_pos, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return (np.cos(ang.astype(np.float64)).astype(np.float32).astype(np.float16),
            np.sin(ang.astype(np.float64)).astype(np.float32).astype(np.float16))


def ref_prep(x, w_norm, eps, cos, sin):
    x = x.astype(np.float32)
    if w_norm is not None:
        sq = round_f16(x * x)
        mean = round_f16(np.float32(sq.astype(np.float64).sum() / 128))
        d = round_f16(np.float32(1.0 / np.sqrt(np.float64(mean) + np.float64(np.float32(eps)))))
        x = round_f16(round_f16(x * d) * w_norm.astype(np.float32))
    c = np.concatenate([cos, cos]).astype(np.float32)
    s = np.concatenate([sin, sin]).astype(np.float32)
    rot = np.concatenate([-x[64:], x[:64]])
    return round_f16(round_f16(x * c) + round_f16(rot * s))


@pytest.mark.parametrize("split", [0, 1], ids=["cluster", "split_k"])
@pytest.mark.parametrize("hq,hkv,slot,norm", [(16, 8, 40, True), (24, 8, 767, False), (28, 4, 8300, False),
                                              (8, 8, 0, False), (64, 8, 100, False), (4, 2, 5, True),
                                              (32, 8, 2560, False)])
def test_decode_attention_step(hq, hkv, slot, norm, split):
    # split = 1: the split-K kernel, which runs where cluster launches are unavailable
    E.check(E.lib().ylm_set_attention_path(split), "path")
    try:
        _decode_attention_step(hq, hkv, slot, norm)
    finally:
        E.lib().ylm_set_attention_path(0)


def _decode_attention_step(hq, hkv, slot, norm):
    rng = np.random.default_rng(hq * 1000 + slot)
    D, cap, max_pos = 128, slot + 64, slot + 16
    pos = max(0, slot - 1)
    qkv = (rng.standard_normal((hq + 2 * hkv) * D) * 0.5).astype(np.float16)
    kc = (rng.standard_normal((hkv, cap, D)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((hkv, cap, D)).astype(np.float16)
    qn = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float16) if norm else None
    kn = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float16) if norm else None
    cos, sin = rope_tables(max_pos)
    d_qkv, d_kc, d_vc, d_cos, d_sin = dev(qkv), dev(kc), dev(vc), dev(cos), dev(sin)
    d_qn = dev(qn) if norm else None
    d_kn = dev(kn) if norm else None
    out = torch.empty(hq * D, dtype=torch.float16, device="cuda")
    E.check(E.lib().ylm_k_decode_attention(ptr(d_qkv), ptr(d_qn) if norm else None, ptr(d_kn) if norm else None,
                                           1e-6, ptr(d_cos), ptr(d_sin), max_pos, ptr(d_kc), ptr(d_vc), cap, hq,
                                           hkv, slot, pos, ptr(out), stream()), "attn")
    torch.cuda.synchronize()
    # reference: new k/v appended at `slot`, attention over [0, slot]
    k_new = np.stack([ref_prep(qkv[(hq + g) * D:(hq + g + 1) * D], kn, 1e-6, cos[pos], sin[pos]) for g in range(hkv)])
    v_new = qkv[(hq + hkv) * D:].reshape(hkv, D).astype(np.float32)
    K = kc.astype(np.float64).copy()
    Vv = vc.astype(np.float64).copy()
    K[:, slot] = k_new
    Vv[:, slot] = v_new
    got_k = d_kc.cpu().numpy()[:, slot].astype(np.float32)
    got_v = d_vc.cpu().numpy()[:, slot].astype(np.float32)
    np.testing.assert_array_equal(got_k, k_new.astype(np.float16).astype(np.float32))
    np.testing.assert_array_equal(got_v, v_new)
    G = hq // hkv
    ref = np.empty(hq * D)
    for h in range(hq):
        g = h // G
        q = ref_prep(qkv[h * D:(h + 1) * D], qn, 1e-6, cos[pos], sin[pos]).astype(np.float64)
        s = K[g, :slot + 1] @ q / np.sqrt(D)
        p = np.exp(s - s.max())
        p /= p.sum()
        ref[h * D:(h + 1) * D] = p @ Vv[g, :slot + 1]
    got = out.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got - ref)) < 2e-3


@pytest.mark.parametrize("vocab", [1000, 32768, 128256, 151936])
def test_sampler_greedy_lowest_index_on_ties(vocab):
    rng = np.random.default_rng(vocab)
    logits = (rng.standard_normal(vocab) * 2).astype(np.float16)
    m = logits.max()
    ties = rng.choice(vocab, 5, replace=False)
    logits[ties] = m + np.float16(1.0)
    d = dev(logits)
    out = ctypes.c_int64()
    E.check(E.lib().ylm_k_sample(ptr(d), vocab, 1, 1, 1.0, None, -1.0, ctypes.byref(out), None, None, stream()), "s")
    assert out.value == int(ties.min()) == S.greedy(logits.astype(np.float32))


@pytest.mark.parametrize("vocab,k,temp", [(1000, 40, 0.6), (128256, 40, 0.6), (151936, 2, 0.05), (32768, 64, 0.7),
                                          (128256, 1, 0.3)])
def test_sampler_topk_bit_exact(vocab, k, temp):
    rng = np.random.default_rng(vocab + k)
    # heavily tied FP16 logits, as random-init models produce
    logits = np.round(rng.standard_normal(vocab) * 8).astype(np.float16) / np.float16(4)
    masked = rng.choice(vocab, 50, replace=False)
    bits = np.zeros((vocab + 31) // 32, np.uint32)
    for i in masked:
        bits[i >> 5] |= np.uint32(1) << np.uint32(i & 31)
    d, dm = dev(logits), dev(bits.view(np.int32))
    for trial in range(20):
        u = float(rng.random())
        u = np.float32(max(u, 1e-6))
        out = ctypes.c_int64()
        ids = np.zeros(64, np.int64)
        probs = np.zeros(64, np.float32)
        E.check(E.lib().ylm_k_sample(ptr(d), vocab, 0, k, temp, ptr(dm), float(u), ctypes.byref(out),
                                     ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                     probs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), stream()), "s")
        vals, want_ids = S.topk_candidates(logits.astype(np.float32), k, temp, masked)
        want_p = S.topk_probs(vals)
        np.testing.assert_array_equal(ids[:k], want_ids)
        np.testing.assert_array_equal(probs[:k], want_p)
        assert out.value == S.draw(want_p, want_ids, u)
