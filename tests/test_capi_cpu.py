"""C-ABI checks that need no GPU: the library loads, exports every entry point
the header declares, its struct layouts match the ctypes mirror, and the host
logic (config parsing, snapshot resolution, argument validation) behaves."""
import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from yalama_b200 import engine as E
from yalama_b200 import synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "yalama_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ylm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = E.lib()
    syms = declared_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the ctypes table covers the same set
    assert sorted(E.SIGNATURES) == syms


def test_struct_layouts_match_c():
    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "yalama_b200.h"
#define P(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("ylm_model_config %zu\n", sizeof(ylm_model_config));
  printf("ylm_engine_options %zu\n", sizeof(ylm_engine_options));
  printf("ylm_sampling %zu\n", sizeof(ylm_sampling));
  P(ylm_model_config, vocab_size) P(ylm_model_config, eos_ids) P(ylm_model_config, n_eos)
  P(ylm_engine_options, nccl_id) P(ylm_engine_options, init_seed) P(ylm_engine_options, zero_kv_on_begin)
  P(ylm_engine_options, prefill_tensor_cores) P(ylm_engine_options, init_std) P(ylm_engine_options, decode_persistent)
  P(ylm_sampling, seed) P(ylm_sampling, masked_ids) P(ylm_sampling, n_masked)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "l.c")
        open(src, "w").write(prog)
        exe = os.path.join(d, "l")
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), src, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    c = dict(line.split() for line in out if line)
    assert int(c["ylm_model_config"]) == ctypes.sizeof(E.ModelConfig)
    assert int(c["ylm_engine_options"]) == ctypes.sizeof(E.EngineOptions)
    assert int(c["ylm_sampling"]) == ctypes.sizeof(E.Sampling)
    for k, v in c.items():
        if "." in k:
            t, f = k.split(".")
            cls = {"ylm_model_config": E.ModelConfig, "ylm_engine_options": E.EngineOptions,
                   "ylm_sampling": E.Sampling}[t]
            assert getattr(cls, f).offset == int(v), k


def test_status_strings_and_defaults():
    L = E.lib()
    assert L.ylm_status_string(0) == b"ok"
    assert b"KV cache" in L.ylm_status_string(2)
    o = E.default_options()
    assert (o.kv_cache_gb, o.kv_cache_enabled, o.rope_compat, o.use_cuda_graph, o.tp_size) == (2, 1, 1, 1, 1)


@pytest.mark.parametrize("name", ["qwen3-0.6b", "llama3.2-3b", "qwen2.5-7b", "llama3.1-8b"])
def test_config_from_json_matches_spec(name, tmp_path):
    spec = synth.PRESETS[name]
    p = tmp_path / "config.json"
    import json
    p.write_text(json.dumps(spec.config_json()))
    c = E.config_from_json(str(p))
    want = E.config_from_spec(spec)
    for f, _ in E.ModelConfig._fields_:
        if f == "eos_ids":
            assert c.eos_ids[0] == want.eos_ids[0]
            continue
        a, b = getattr(c, f), getattr(want, f)
        assert a == pytest.approx(b), f


def test_config_rejects_unknown_model_type(tmp_path):
    p = tmp_path / "config.json"
    p.write_text('{"model_type": "gpt2"}')
    with pytest.raises(E.YlmError) as ei:
        E.config_from_json(str(p))
    assert ei.value.status == E.Status.LOAD_ERROR
    assert "Unsupported model type" in str(ei.value)


def test_resolve_snapshot(tmp_path):
    spec = synth.tiny_spec("llama", layers=1, vocab=64)
    snap = synth.write_snapshot(str(tmp_path), spec, dtype="F16")
    assert E.resolve_snapshot(str(tmp_path)) == snap
    with pytest.raises(E.YlmError):
        E.resolve_snapshot(str(tmp_path / "nope"))


def test_kernel_entry_points_validate_arguments():
    L = E.lib()
    # rejected before touching any device
    assert L.ylm_k_gemv(None, 4, 8, None, None, None) == E.Status.INVALID_ARG
    assert L.ylm_k_gemm(None, None, 1, 1, 1, None, 1, None) == E.Status.INVALID_ARG
    assert L.ylm_k_sample(None, 10, 1, 1, 1.0, None, 0.5, None, None, None, None) == E.Status.INVALID_ARG
    assert L.ylm_k_decode_attention(None, None, None, 1e-6, None, None, 16, None, None, 8, 4, 2, 0, 0, None,
                                    None) == E.Status.INVALID_ARG


def test_create_rejects_bad_shapes():
    spec = synth.tiny_spec("llama", layers=1)
    c = E.config_from_spec(spec)
    c.head_dim = 64
    with pytest.raises(E.YlmError) as ei:
        E.Engine(None, c)
    assert ei.value.status == E.Status.UNSUPPORTED


def test_engine_calls_reject_a_null_engine():
    # every engine-level call checks its handle before any device work, so a
    # NULL engine is INVALID_ARG (ylm_destroy(NULL) is a no-op, like free)
    L = E.lib()
    inv = E.Status.INVALID_ARG
    assert L.ylm_destroy(None) == E.Status.OK
    assert L.ylm_begin_infer(None) == inv
    assert L.ylm_infer(None, None, None, None, None) == inv
    assert L.ylm_logits(None, None, 0) == inv
    assert L.ylm_logits_device(None, None, None) == inv
    assert L.ylm_set_sampling(None, None) == inv
    assert L.ylm_sample(None, 1, None) == inv
    assert L.ylm_decode(None, 0, 1, None) == inv
    assert L.ylm_generate(None, None, 0, 0, None, 0, None, None, None, None) == inv
    assert L.ylm_set_draw(None, 0.5) == inv
    assert L.ylm_last_topk(None, None, None, None, None) == inv
    assert L.ylm_info(None, None, None, None) == inv
    assert L.ylm_last_prefill_ms(None, None) == inv
    assert L.ylm_decode_path(None, None) == inv
    assert L.ylm_time_decode(None, 1, None) == inv
    assert L.ylm_time_segment(None, 0, 1, None, None) == inv
    assert L.ylm_exchange_stats(None, 0, None, None, None) == inv
    assert L.ylm_time_allreduce(None, 1, None) == inv
    assert L.ylm_debug_drop_output(None, 0) == inv
    assert L.ylm_options_default(None) == inv
    assert L.ylm_config_from_json(None, None) == inv
    assert L.ylm_resolve_snapshot(None, None, 0) == inv


def test_more_kernel_entry_points_validate_arguments():
    L = E.lib()
    inv = E.Status.INVALID_ARG
    assert L.ylm_k_prefill_attention(None, None, None, 16, 4, 2, 8, None, 1, None) == inv
    # grouped-query shapes the kernels do not cover: hq not a multiple of hkv,
    # more than 8 query heads per KV head
    p = ctypes.c_void_p(256)
    assert L.ylm_k_decode_attention(p, None, None, 1e-6, p, p, 16, p, p, 8, 6, 4, 0, 0, p, None) == inv
    assert L.ylm_k_decode_attention(p, None, None, 1e-6, p, p, 16, p, p, 8, 18, 2, 0, 0, p, None) == inv
    # slot past the cache, RoPE position past the table
    assert L.ylm_k_decode_attention(p, None, None, 1e-6, p, p, 16, p, p, 8, 4, 2, 8, 0, p, None) == inv
    assert L.ylm_k_decode_attention(p, None, None, 1e-6, p, p, 16, p, p, 8, 4, 2, 0, 16, p, None) == inv
    assert L.ylm_k_decode_attention_noalloc(p, None, None, 1e-6, p, p, 16, p, p, 8, 4, 2, 8, 0, p, None) == inv
