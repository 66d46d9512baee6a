"""The sampler against LibTorch's own CUDA ops, as ChatSession::Sample calls
them (src/ChatSession.cpp:560-593): argmax, ``logits / Temp``, masked ids to
-1e9, ``torch::topk``, ``torch::softmax``. The fixture
(tests/golden/sampler_torch_cuda.npz) was produced by the reference harness's
``--sample-fixture`` mode with the LibTorch CUDA FP16 build
(tests/golden/make_sampler_golden.py); its logit rows are regenerated here.

What is pinned, per row and (K, Temp):
- the greedy id (argmax: the first maximal index);
- the top-k values, FP16, in order (bit for bit);
- the softmax probabilities, FP16, in order (bit for bit);
- the ids: for every value, the same set of ids, except for the value tied at
  the k-th place, where LibTorch keeps an unspecified subset of the tied ids.
  The order of ids among equal values is LibTorch's own (not specified by its
  API); the engine and the oracle order them by index. The draw itself
  (torch::multinomial) is not reproducible: the engine's contract is the
  inverse-CDF draw over this candidate order with a given uniform, which
  tests/test_gpu_kernels.py and tests/test_gpu_model.py check bit for bit.
"""
import ctypes
import importlib.util
import os

import numpy as np
import pytest

from oracle import sampler as S

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "golden", "sampler_torch_cuda.npz")


def _gen():
    spec = importlib.util.spec_from_file_location("make_sampler_golden",
                                                  os.path.join(HERE, "golden", "make_sampler_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


@pytest.fixture(scope="module")
def fixture():
    if not os.path.exists(FIXTURE):
        pytest.fail(f"{FIXTURE} is missing: generate it on a GPU with tests/golden/make_sampler_golden.py")
    z = np.load(FIXTURE)
    g = _gen()
    return z, g.logit_rows(), [int(i) for i in z["masked"]], [(int(k), float(t)) for k, t in z["params"]]


def check_candidates(ids, vals, probs, z, i, r, k):
    """ids/vals/probs: one sampler's top-k for row r of parameter set i."""
    rid = z[f"p{i}_ids"][r]
    rv = z[f"p{i}_vals"][r].view(np.float16).astype(np.float32)
    rp = z[f"p{i}_probs"][r].view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(np.asarray(vals, np.float32), rv)
    np.testing.assert_array_equal(np.asarray(probs, np.float32), rp)
    kth = rv[k - 1]
    for v in np.unique(rv):
        a = set(int(x) for x in np.asarray(ids)[rv == v])
        b = set(int(x) for x in rid[rv == v])
        if v == kth:
            assert len(a) == len(b)
        else:
            assert a == b, (i, r, float(v), sorted(a - b), sorted(b - a))


def test_oracle_sampler_matches_libtorch_cuda(fixture):
    z, rows, masked, params = fixture
    for i, (k, t) in enumerate(params):
        for r in range(rows.shape[0]):
            lg = rows[r].astype(np.float32)
            assert S.greedy(lg) == int(z[f"p{i}_greedy"][r])
            vals, ids = S.topk_candidates(lg, k, t, masked)
            check_candidates(ids, vals, S.topk_probs(vals), z, i, r, k)


@pytest.mark.gpu
def test_engine_sampler_matches_libtorch_cuda(fixture):
    import torch
    from yalama_b200 import engine as E
    z, rows, masked, params = fixture
    V = rows.shape[1]
    bits = np.zeros((V + 31) // 32, np.uint32)
    for m in masked:
        bits[m >> 5] |= np.uint32(1) << np.uint32(m & 31)
    dm = torch.from_numpy(bits.view(np.int32)).cuda()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for r in range(rows.shape[0]):
        d = torch.from_numpy(rows[r].view(np.int16)).cuda()
        out = ctypes.c_int64()
        E.check(E.lib().ylm_k_sample(ctypes.c_void_p(d.data_ptr()), V, 1, 1, 1.0, None, -1.0, ctypes.byref(out),
                                     None, None, s), "greedy")
        greedy_id = out.value
        for i, (k, t) in enumerate(params):
            assert greedy_id == int(z[f"p{i}_greedy"][r])
            ids = np.zeros(64, np.int64)
            probs = np.zeros(64, np.float32)
            E.check(E.lib().ylm_k_sample(ctypes.c_void_p(d.data_ptr()), V, 0, k, t,
                                         ctypes.c_void_p(dm.data_ptr()), 0.5, ctypes.byref(out),
                                         ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                         probs.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), s), "topk")
            # the candidate values in order are the reference's, so the scaled
            # values of the engine's ids are those of the fixture
            vals, _ = S.topk_candidates(rows[r].astype(np.float32), k, t, masked)
            check_candidates(ids[:k], vals, probs[:k], z, i, r, k)
