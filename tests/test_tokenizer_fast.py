"""The O(n log n) BPE encoder (yalama_b200/host/FastTokenizer.h) against the
reference's own tokenizer classes, compiled from the reference tree
(src/tokenizer/*.cpp, yalama_b200/host/Makefile): for each family (Llama: text
split at spaces and punctuation; Qwen and Mistral: the whole text between
special tokens is one BPE piece), the ids of EncodeWithoutChatTemplate must be
identical. Tokenizers are synthetic (yalama_b200.synth.write_bpe_tokenizer:
20k nested merges); texts cover special tokens inside, at the ends and
adjacent, whitespace runs, multi-byte characters, characters outside the
vocabulary, and the empty string. One long Qwen prompt also checks that the
encoder is not quadratic."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
REF = os.environ.get("YLM_REFERENCE_SRC", "/root/reference")
BIN = os.path.join(ROOT, "yalama_b200", "host", "_build", "tokenizer_bench")
FAMILIES = ["llama", "qwen", "mistral"]


@pytest.fixture(scope="module")
def bench_bin():
    if not os.path.isdir(os.path.join(REF, "src")):
        pytest.skip("the reference sources are not present on this machine")
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "yalama_b200", "host"), "-j8", f"REF={REF}",
                        f"PYTHON={sys.executable}", os.path.join(ROOT, "yalama_b200", "host", "_build",
                                                                 "tokenizer_bench")],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return BIN


@pytest.fixture(scope="module")
def tokenizers(tmp_path_factory):
    from yalama_b200 import synth
    out = {}
    for fam in FAMILIES:
        d = str(tmp_path_factory.mktemp(f"tok_{fam}"))
        synth.write_bpe_tokenizer(d, fam, 20000, seed=3)
        out[fam] = d
    return out


def encode_both(binary, model, fam, text, tmp_path, reps=1):
    p = tmp_path / "text.txt"
    p.write_bytes(text.encode())
    r = subprocess.run([binary, "--model", model, "--family", fam, "--text", str(p), "--reps", str(reps),
                        "--ref-reps", "1"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def edge_texts(fam):
    from yalama_b200 import synth
    sp = synth.SPECIAL_TOKENS["qwen" if fam == "qwen" else "llama"]
    body = synth.bpe_text(fam, 600, seed=3)
    return [
        "",
        "a",
        " ",
        sp[1],
        sp[0] + sp[1] + sp[-1],
        sp[1] + body + sp[-1],
        body + sp[0],
        "   " + body + "\n\n\t  " + body + "  ",
        body.replace(" ", "  ") + " 😀 ∑ ñ \x01\x7f",
        "user" + sp[1] + "\n" + body + sp[-1] + sp[1] + "assistant\n",
    ]


@pytest.mark.parametrize("fam", FAMILIES)
def test_fast_bpe_ids_equal_reference_on_edge_cases(bench_bin, tokenizers, fam, tmp_path):
    for i, text in enumerate(edge_texts(fam)):
        res = encode_both(bench_bin, tokenizers[fam], fam, text, tmp_path)
        assert res["equal"], (fam, i, res)


@pytest.mark.parametrize("fam", FAMILIES)
@pytest.mark.parametrize("specials_every", [0, 40])
def test_fast_bpe_ids_equal_reference_on_prompts(bench_bin, tokenizers, fam, specials_every, tmp_path):
    from yalama_b200 import synth
    text = synth.bpe_text(fam, 8000, seed=5, specials_every=specials_every)
    res = encode_both(bench_bin, tokenizers[fam], fam, text, tmp_path)
    assert res["equal"], res
    assert res["tokens"] > 1000


def test_fast_bpe_is_not_quadratic(bench_bin, tokenizers, tmp_path):
    """A 32 KB Qwen prompt is one BPE piece: the reference's merge loop is
    quadratic in it, the heap merge is not (measured: about 2 s against 20 ms)."""
    from yalama_b200 import synth
    text = synth.bpe_text("qwen", 32000, seed=7)
    res = encode_both(bench_bin, tokenizers["qwen"], "qwen", text, tmp_path, reps=3)
    assert res["equal"], res
    assert res["fast_ms"] * 10 < res["ref_ms"], res
