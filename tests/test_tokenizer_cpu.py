"""Tokenizers on CPU: a small Hugging Face tokenizer built offline (a
character-level WordLevel model saved with ``save_pretrained``) through
``HFTokenizer``, a checkpoint directory with that tokenizer through
``LLMEngine.from_pretrained`` (the oracle kernels), ``--tokenizer-path``, and
the byte tokenizer's chat fallback."""
import importlib
import json

import pytest
import torch

PKG = "3080_mod_p2p_sglang_patch_b200"
models = importlib.import_module(f"{PKG}.models")
eng_mod = importlib.import_module(f"{PKG}.engine")
tk = importlib.import_module(f"{PKG}.engine.tokenizer")

TEMPLATE = ("{% for m in messages %}<{{ m['role'] }}>{{ m['content'] }}{% endfor %}"
            "{% if add_generation_prompt %}<assistant>{% endif %}")


def make_tokenizer(path, template=TEMPLATE):
    """Characters a-z, space and punctuation as single tokens (ids 3..), with
    <s>=0, </s>=1, <unk>=2; saved as tokenizer.json plus its config."""
    from tokenizers import Tokenizer, decoders, models as tmodels, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {"<s>": 0, "</s>": 1, "<unk>": 2}
    for i, c in enumerate("abcdefghijklmnopqrstuvwxyz .,!?<>"):
        vocab[c] = 3 + i
    t = Tokenizer(tmodels.WordLevel(vocab, unk_token="<unk>"))
    t.pre_tokenizer = pre_tokenizers.Split("", "isolated")
    t.decoder = decoders.Fuse()
    f = PreTrainedTokenizerFast(tokenizer_object=t, bos_token="<s>", eos_token="</s>", unk_token="<unk>")
    if template:
        f.chat_template = template
    f.save_pretrained(str(path))
    return vocab


def test_hf_tokenizer_encode_decode_and_chat(tmp_path):
    vocab = make_tokenizer(tmp_path)
    tok = tk.HFTokenizer(str(tmp_path))
    ids = tok.encode("hi there")
    assert ids == [vocab[c] for c in "hi there"] and tok.decode(ids) == "hi there"
    assert tok.decode(ids + [1]) == "hi there"                             # special tokens dropped
    chat = tok.chat([{"role": "user", "content": "hi"}])
    assert all(isinstance(t, int) for t in chat)                          # ids, not an encoding's keys
    assert tok.decode(chat) == "<user>hi<assistant>"
    over = tk.HFTokenizer(str(tmp_path), chat_template="{{ messages[0]['content'] }}!")
    assert over.decode(over.chat([{"role": "user", "content": "yo"}])) == "yo!"


def test_hf_tokenizer_without_a_template_and_the_byte_fallback(tmp_path):
    make_tokenizer(tmp_path, template=None)
    tok = tk.HFTokenizer(str(tmp_path))
    assert tok.decode(tok.chat([{"role": "user", "content": "ab"}])) == "user ab"  # ':' and '\n' are <unk>
    b = tk.ByteTokenizer()
    assert b.decode(b.chat([{"role": "user", "content": "x"}])) == "<|user|>x<|assistant|>"
    assert tk.ByteTokenizer(TEMPLATE).decode(tk.ByteTokenizer(TEMPLATE).chat([{"role": "a", "content": "b"}])) \
        == "<a>b<assistant>"


def _checkpoint(tmp_path, with_tokenizer=True):
    cfg = models.LlamaConfig.tiny()
    w = models.LlamaWeights(cfg, 0, 1, "cpu", seed=5, full_init=True)
    d = tmp_path / "ckpt"
    models.save_llama(str(d), cfg, w)
    if with_tokenizer:
        make_tokenizer(d)
    with open(d / "generation_config.json", "w") as f:
        json.dump({"eos_token_id": 1}, f)
    return d


def test_from_pretrained_loads_the_checkpoint_tokenizer(tmp_path):
    d = _checkpoint(tmp_path)
    eng = eng_mod.LLMEngine.from_pretrained(str(d), device="cpu", impl="oracle", max_batch=2, max_seq=128,
                                            chunk=64, use_graphs=False)
    assert isinstance(eng.tokenizer, tk.HFTokenizer) and eng.default_stop_ids == (1,)
    out = eng.generate_text("abc", {"max_new_tokens": 3})
    assert 1 <= len(out["token_ids"]) <= 3 and out["text"] == eng.tokenizer.decode(out["token_ids"])


def test_tokenizer_path_overrides_and_must_exist(tmp_path):
    d = _checkpoint(tmp_path, with_tokenizer=False)
    kw = dict(device="cpu", impl="oracle", max_batch=2, max_seq=128, chunk=64, use_graphs=False)
    assert eng_mod.LLMEngine.from_pretrained(str(d), **kw).tokenizer is None      # none in the checkpoint
    with pytest.raises(FileNotFoundError):
        tk.HFTokenizer(str(d))                         # config.json alone is not a tokenizer
    tdir = tmp_path / "tok"
    make_tokenizer(tdir)
    eng = eng_mod.LLMEngine.from_pretrained(str(d), tokenizer_path=str(tdir), **kw)
    assert eng.tokenizer.encode("ab") == [3, 4]
    with pytest.raises(Exception):
        eng_mod.LLMEngine.from_pretrained(str(d), tokenizer_path=str(tmp_path / "missing"), **kw)


def test_cli_tokenizer_path_flag():
    cli = importlib.import_module(f"{PKG}.server.cli")
    args = cli.build_parser().parse_args(["--model-path", "x", "--tokenizer-path", "/t"])
    assert args.tokenizer_path == "/t"


def test_chat_endpoint_with_the_checkpoint_tokenizer(tmp_path):
    """/v1/chat/completions renders the checkpoint's template into token ids."""
    import threading

    import requests

    from conftest import free_port

    srv = importlib.import_module(f"{PKG}.server")
    d = _checkpoint(tmp_path)
    eng = eng_mod.LLMEngine.from_pretrained(str(d), device="cpu", impl="oracle", max_batch=2, max_seq=128,
                                            chunk=64, use_graphs=False)
    server = srv.EngineServer(eng, max_prompt=eng.max_seq, stop_ids=eng.default_stop_ids)
    loop = threading.Thread(target=server.serve_forever, daemon=True)
    loop.start()
    port = free_port()
    http, _ = srv.start_http(srv.build_app(server, "ckpt", eng.tokenizer), "127.0.0.1", port)
    try:
        r = requests.post(f"http://127.0.0.1:{port}/v1/chat/completions",
                          json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 2}, timeout=120)
        assert r.status_code == 200, r.text
        body = r.json()
        assert body["usage"]["prompt_tokens"] == len("<user>hi<assistant>")
        assert 1 <= body["usage"]["completion_tokens"] <= 2
    finally:
        server.stop()
        loop.join(timeout=30)
        http.should_exit = True
