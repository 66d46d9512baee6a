"""The drop-in facade end to end on the GPU: the reference's own
ChatSession::Generate (src/ChatSession.cpp:64-277, compiled unmodified with its
tokenizer, chat templates and ConfigManager) over yalama_b200/host/Model.cpp and
the engine, on a synthetic snapshot with a byte-level BPE tokenizer.json. The
ids ChatSession feeds back to Model::Infer must be the engine's own greedy token
loop (ylm_generate) on the prompt ids ChatSession built."""
import json
import os
import subprocess

import pytest

from yalama_b200 import engine as E
from yalama_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "yalama_b200", "host", "_build", "facade_chat")


@pytest.mark.parametrize("fam,family", [("llama", "llama"), ("qwen3", "qwen")])
def test_chat_session_generate_through_facade(fam, family, tmp_path):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} is missing: build it with `make -C yalama_b200/host` where the reference sources are")
    kw = dict(model_type=fam, heads=8, kv_heads=2, vocab=1024, max_pos=512)
    if fam == "llama":
        kw.update(tied=False, rope_theta=5e5)
    spec = synth.tiny_spec(**kw)
    root = str(tmp_path / "model")
    snap = synth.write_snapshot(root, spec, seed=3, dtype="F16")
    specials = synth.write_tokenizer(snap, spec, family)
    eos = specials[synth.SPECIAL_TOKENS[family][-1]]
    r = subprocess.run([BIN, "--model", root, "--message", "Tell me about the engine and the tokens."],
                       capture_output=True, text=True, errors="replace", timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["ok"], out
    prompt, fed = out["prompt"], out["fed"]
    assert len(prompt) > 10 and all(0 <= t < spec.vocab for t in prompt)
    # the prompt carries the chat template's special tokens
    assert set(specials.values()) & set(prompt)
    assert len(fed) >= 1
    eng = E.Engine(snap, E.config_from_spec(spec))
    try:
        g = eng.generate(prompt, len(fed) + 1, eos_ids=[eos])
        assert [int(t) for t in g["ids"][:len(fed)]] == fed
    finally:
        eng.close()
