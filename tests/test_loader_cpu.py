"""Hugging Face Llama checkpoint loading (safetensors reader/writer, config
mapping, TP sharding into the engine's layout), on CPU tensors."""
import importlib
import json

import torch

models = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models")
ops = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops")

HF_CFG = {"architectures": ["LlamaForCausalLM"], "hidden_size": 256, "num_hidden_layers": 2,
          "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 128, "intermediate_size": 384,
          "vocab_size": 512, "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "max_position_embeddings": 1024,
          "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                           "original_max_position_embeddings": 256}}


def _checkpoint(tmp_path, tied=False):
    g = torch.Generator().manual_seed(0)
    H, D, F = 256, 128, 384
    t = {"model.embed_tokens.weight": torch.randn(512, H, generator=g).to(torch.bfloat16),
         "model.norm.weight": torch.randn(H, generator=g).to(torch.bfloat16)}
    if not tied:
        t["lm_head.weight"] = torch.randn(512, H, generator=g).to(torch.bfloat16)
    for i in range(2):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = torch.randn(H, generator=g).to(torch.bfloat16)
        t[p + "post_attention_layernorm.weight"] = torch.randn(H, generator=g).to(torch.bfloat16)
        t[p + "self_attn.q_proj.weight"] = torch.randn(4 * D, H, generator=g).to(torch.bfloat16)
        t[p + "self_attn.k_proj.weight"] = torch.randn(2 * D, H, generator=g).to(torch.bfloat16)
        t[p + "self_attn.v_proj.weight"] = torch.randn(2 * D, H, generator=g).to(torch.bfloat16)
        t[p + "self_attn.o_proj.weight"] = torch.randn(H, 4 * D, generator=g).to(torch.float16)  # mixed dtypes
        t[p + "mlp.gate_proj.weight"] = torch.randn(F, H, generator=g).to(torch.float32)
        t[p + "mlp.up_proj.weight"] = torch.randn(F, H, generator=g).to(torch.bfloat16)
        t[p + "mlp.down_proj.weight"] = torch.randn(H, F, generator=g).to(torch.bfloat16)
    names = sorted(t)
    half = len(names) // 2  # two shards, like a real multi-file checkpoint
    models.write_safetensors(str(tmp_path / "model-00001.safetensors"), {k: t[k] for k in names[:half]},
                             {"format": "pt"})
    models.write_safetensors(str(tmp_path / "model-00002.safetensors"), {k: t[k] for k in names[half:]})
    (tmp_path / "config.json").write_text(json.dumps(HF_CFG))
    return t


def test_safetensors_roundtrip_and_slices(tmp_path):
    src = {"a": torch.randn(6, 5).to(torch.bfloat16), "b": torch.arange(12, dtype=torch.float32).view(3, 4),
           "c": torch.randn(7).to(torch.float16)}
    models.write_safetensors(str(tmp_path / "x.safetensors"), src, {"k": "v"})
    f = models.SafeTensors(str(tmp_path / "x.safetensors"))
    assert sorted(f.keys()) == ["a", "b", "c"] and f.meta == {"k": "v"}
    for k, v in src.items():
        got = f.get(k)
        assert got.dtype == v.dtype and torch.equal(got, v)
    assert torch.equal(f.get("a", rows=(2, 4)), src["a"][2:4])
    assert torch.equal(f.get("b", cols=(1, 3)), src["b"][:, 1:3])


def test_config_mapping():
    cfg = models.config_from_hf(HF_CFG, name="t")
    assert (cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab) == \
        (256, 2, 4, 2, 128, 384, 512)
    assert dict(cfg.rope_scaling)["rope_type"] == "llama3"


def test_tp_shards_match_the_checkpoint(tmp_path):
    t = _checkpoint(tmp_path)
    D = 128
    for tp in (1, 2):
        for r in range(tp):
            cfg, w = models.load_llama(str(tmp_path), r, tp, "cpu")
            nq, nkv, F = 4 // tp, 2 // tp, 384 // tp
            V = 512 // tp
            bf = lambda x: x.to(torch.bfloat16)  # noqa: E731
            assert torch.equal(w.embed, t["model.embed_tokens.weight"][r * V:(r + 1) * V])
            assert torch.equal(w.lm_head, t["lm_head.weight"][r * V:(r + 1) * V])
            assert w.vocab_start == r * V and (w.nq, w.nkv) == (nq, nkv)
            L, p = w.layers[1], "model.layers.1."
            want_qkv = torch.cat([t[p + "self_attn.q_proj.weight"][r * nq * D:(r + 1) * nq * D],
                                  t[p + "self_attn.k_proj.weight"][r * nkv * D:(r + 1) * nkv * D],
                                  t[p + "self_attn.v_proj.weight"][r * nkv * D:(r + 1) * nkv * D]])
            assert torch.equal(L["qkv"], want_qkv)
            assert torch.equal(L["o"], bf(t[p + "self_attn.o_proj.weight"][:, r * nq * D:(r + 1) * nq * D]))
            want_gu = torch.cat([bf(t[p + "mlp.gate_proj.weight"][r * F:(r + 1) * F]),
                                 t[p + "mlp.up_proj.weight"][r * F:(r + 1) * F]])
            assert torch.equal(L["gate_up"], want_gu)
            assert torch.equal(L["down"], t[p + "mlp.down_proj.weight"][:, r * F:(r + 1) * F])
            assert torch.equal(L["ln1"], t[p + "input_layernorm.weight"])
            assert all(v.dtype == torch.bfloat16 and v.is_contiguous() for v in L.values())


def test_tied_embeddings(tmp_path):
    t = _checkpoint(tmp_path, tied=True)
    _, w = models.load_llama(str(tmp_path), 1, 2, "cpu")
    assert torch.equal(w.lm_head, t["model.embed_tokens.weight"][256:])


def test_llama3_rope_scaling_bands():
    """Long wavelengths are divided by the factor, short ones kept, the band
    between interpolated (Llama 3.1 rescaling); plain RoPE without scaling."""
    base = ops.rope_cos_sin(4, 128, 500000.0, "cpu")
    sc = ops.rope_cos_sin(4, 128, 500000.0, "cpu", dict(HF_CFG["rope_scaling"]))
    ang_b = torch.atan2(base[1, 64:], base[1, :64])  # position 1: angle = inv_freq
    ang_s = torch.atan2(sc[1, 64:], sc[1, :64])
    assert torch.allclose(ang_s[:4], ang_b[:4])            # high frequencies unchanged
    assert torch.allclose(ang_s[-4:], ang_b[-4:] / 8.0, rtol=1e-4)  # low frequencies / factor
    mid = (ang_s / ang_b)[4:-4]
    assert bool(((mid <= 1.0 + 1e-6) & (mid >= 1 / 8.0 - 1e-6)).all())


def test_stop_token_ids_from_checkpoint(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"eos_token_id": 2}))
    assert models.stop_token_ids(str(tmp_path)) == (2,)
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [128001, 128009]}))
    assert models.stop_token_ids(str(tmp_path)) == (128001, 128009)  # generation config wins
    assert models.stop_token_ids(str(tmp_path / "missing")) == ()


def test_qwen3_checkpoint_qk_norm(tmp_path):
    """Qwen3ForCausalLM: the Llama decoder plus per-head q/k RMSNorm; the norm
    weights are loaded on every rank and applied to the fused qkv in place."""
    cfg_json = dict(HF_CFG, architectures=["Qwen3ForCausalLM"], rope_scaling=None, tie_word_embeddings=True)
    t = _checkpoint(tmp_path, tied=True)
    g = torch.Generator().manual_seed(5)
    extra = {}
    for i in range(2):
        extra[f"model.layers.{i}.self_attn.q_norm.weight"] = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
        extra[f"model.layers.{i}.self_attn.k_norm.weight"] = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    models.write_safetensors(str(tmp_path / "model-00003.safetensors"), extra)
    (tmp_path / "config.json").write_text(json.dumps(cfg_json))
    cfg, w = models.load_llama(str(tmp_path), 1, 2, "cpu")
    assert cfg.qk_norm and torch.equal(w.layers[1]["q_norm"], extra["model.layers.1.self_attn.q_norm.weight"])
    model = models.LlamaTP(cfg, w, tp=None, impl="native")
    nq, nkv, D = w.nq, w.nkv, 128
    qkv = torch.randn(5, (nq + 2 * nkv) * D, generator=g).to(torch.bfloat16)
    before = qkv.clone()
    model._qk_norm(qkv, w.layers[1], nq, nkv, D)

    def rms(x, wt):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.eps) * wt.float()).to(torch.bfloat16)

    q = before[:, :nq * D].view(5, nq, D)
    k = before[:, nq * D:(nq + nkv) * D].view(5, nkv, D)
    assert torch.equal(qkv[:, :nq * D].view(5, nq, D), rms(q, w.layers[1]["q_norm"]))
    assert torch.equal(qkv[:, nq * D:(nq + nkv) * D].view(5, nkv, D), rms(k, w.layers[1]["k_norm"]))
    assert torch.equal(qkv[:, (nq + nkv) * D:], before[:, (nq + nkv) * D:])  # v untouched


def test_unsupported_architecture_is_rejected():
    import pytest

    with pytest.raises(ValueError):
        models.config_from_hf(dict(HF_CFG, architectures=["MixtralForCausalLM"]))
    with pytest.raises(ValueError):
        models.config_from_hf(dict(HF_CFG, attention_bias=True))
