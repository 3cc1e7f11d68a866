"""Hugging Face Llama checkpoint loading (safetensors reader/writer, config
mapping, TP sharding into the engine's layout), on CPU tensors."""
import importlib
import json

import pytest
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
    model = models.LlamaTP(cfg, w, tp=None, impl="oracle")
    nq, nkv, D = w.nq, w.nkv, 128
    args = model._qk_norm_args(w.layers[1])
    assert args["q_norm"] is w.layers[1]["q_norm"] and args["k_norm"] is w.layers[1]["k_norm"]
    # the RoPE step applies the norm: q and cached k are rope(rmsnorm(head)), v is copied as is
    qkv = torch.randn(5, (nq + 2 * nkv) * D, generator=g).to(torch.bfloat16)
    pos = torch.arange(5, dtype=torch.int32)
    cs = ops.rope_cos_sin(64, D, cfg.rope_theta, "cpu")
    kc = torch.zeros(2, nkv, 16, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.arange(16, 21, dtype=torch.int64)
    q = model.k.rope_and_cache(qkv, pos, cs, nq, nkv, slots, kc, vc, **args)

    def rms(x, wt):
        xf = x.float()
        return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.eps) * wt.float()

    ref = importlib.import_module("3080_mod_p2p_sglang_patch_b200.ops.reference")
    want_q = ref.rope(rms(qkv[:, :nq * D].view(5, nq, D), w.layers[1]["q_norm"]), pos, cs).to(torch.bfloat16)
    want_k = ref.rope(rms(qkv[:, nq * D:(nq + nkv) * D].view(5, nkv, D), w.layers[1]["k_norm"]), pos, cs)
    assert torch.equal(q, want_q)
    assert torch.equal(kc[1, :, :5, :].permute(1, 0, 2), want_k.to(torch.bfloat16))
    assert torch.equal(vc[1, :, :5, :].permute(1, 0, 2), qkv[:, (nq + nkv) * D:].view(5, nkv, D))
    assert "q_norm" not in models.LlamaTP(models.config_from_hf(HF_CFG), w, impl="oracle")._qk_norm_args(w.layers[1])


def test_qwen2_biases_and_sliding_windows(tmp_path):
    """Qwen2ForCausalLM: q/k/v biases sharded like the projections' rows;
    MistralForCausalLM: the sliding window caps the positions; a Llama
    checkpoint with attention biases (o_proj too) is refused."""
    cfg_json = dict(HF_CFG, architectures=["Qwen2ForCausalLM"], rope_scaling=None)
    t = _checkpoint(tmp_path)
    g = torch.Generator().manual_seed(9)
    extra = {}
    for i in range(2):
        for proj, rows in (("q_proj", 4 * 128), ("k_proj", 2 * 128), ("v_proj", 2 * 128)):
            extra[f"model.layers.{i}.self_attn.{proj}.bias"] = torch.randn(rows, generator=g).to(torch.bfloat16)
    models.write_safetensors(str(tmp_path / "model-00003.safetensors"), extra)
    (tmp_path / "config.json").write_text(json.dumps(cfg_json))
    for r in range(2):
        cfg, w = models.load_llama(str(tmp_path), r, 2, "cpu")
        assert cfg.qkv_bias and not cfg.qk_norm
        p = "model.layers.1.self_attn."
        want = torch.cat([extra[p + "q_proj.bias"][r * 256:(r + 1) * 256], extra[p + "k_proj.bias"][r * 128:(r + 1) * 128],
                          extra[p + "v_proj.bias"][r * 128:(r + 1) * 128]])
        assert torch.equal(w.layers[1]["qkv_bias"], want)
        assert torch.equal(w.layers[1]["qkv"][:256], t[p + "q_proj.weight"][r * 256:(r + 1) * 256])
    mis = models.config_from_hf(dict(HF_CFG, architectures=["MistralForCausalLM"], sliding_window=512))
    assert mis.max_pos == 512 and not mis.qkv_bias
    assert models.config_from_hf(dict(HF_CFG, architectures=["MistralForCausalLM"], sliding_window=None)).max_pos == 1024
    q2 = models.config_from_hf(dict(HF_CFG, architectures=["Qwen2ForCausalLM"], use_sliding_window=True,
                                    sliding_window=256))
    assert q2.max_pos == 256
    assert models.config_from_hf(dict(HF_CFG, architectures=["Qwen2ForCausalLM"], sliding_window=256)).max_pos == 1024
    with pytest.raises(ValueError, match="biases"):
        models.config_from_hf(dict(HF_CFG, attention_bias=True))


def test_unsupported_architecture_is_rejected():

    with pytest.raises(ValueError):
        models.config_from_hf(dict(HF_CFG, architectures=["MixtralForCausalLM"]))
    with pytest.raises(ValueError):
        models.config_from_hf(dict(HF_CFG, attention_bias=True))


# ---------------------------------------------------------------- AWQ int4

def _nibbles_by_hand(word: int):
    """Output column -> value of one AWQ-packed int32, decoded bit by bit:
    nibble i sits at bits 4i..4i+3 and holds column (0, 2, 4, 6, 1, 3, 5, 7)[i]."""
    word &= 0xFFFFFFFF
    order = (0, 2, 4, 6, 1, 3, 5, 7)
    cols = [0] * 8
    for i in range(8):
        cols[order[i]] = (word >> (4 * i)) & 0xF
    return cols


def test_awq_packing_golden_and_roundtrip():
    p = models.awq_pack(torch.arange(8, dtype=torch.int32).view(1, 8))
    assert p.dtype == torch.int32 and p.item() == 0x75316420
    g = torch.Generator().manual_seed(1)
    q = torch.randint(0, 16, (5, 64), generator=g, dtype=torch.int32)
    packed = models.awq_pack(q)
    assert bool((packed < 0).any())                       # high nibbles >= 8 wrap to negative words
    assert torch.equal(models.awq_unpack(packed), q)
    for r in range(5):
        for c in range(8):
            assert _nibbles_by_hand(int(packed[r, c])) == q[r, 8 * c:8 * c + 8].tolist()


def test_awq_dequant_matches_the_formula_and_bounds_the_error():
    g = torch.Generator().manual_seed(2)
    N, K, G = 48, 256, 64
    w = torch.randn(N, K, generator=g)
    qw, qz, s = models.awq_quantize(w, G)
    assert qw.shape == (K, N // 8) and qz.shape == (K // G, N // 8) and s.shape == (K // G, N)
    assert s.dtype == torch.float16
    deq = models.awq_dequant(qw, qz, s, G)
    assert deq.shape == (N, K)
    # independent decode of one element per group
    for n, k in ((0, 0), (17, 100), (47, 255), (9, 64)):
        q = _nibbles_by_hand(int(qw[k, n // 8]))[n % 8]
        z = _nibbles_by_hand(int(qz[k // G, n // 8]))[n % 8]
        assert deq[n, k].item() == (q - z) * s[k // G, n].float().item()
    step = s.float().repeat_interleave(G, 0).t()          # [N, K] quantization step
    assert bool(((deq - w).abs() <= step * 0.5 + 1e-3).all())


def _awq_checkpoint(tmp_path, group):
    """The bf16 test checkpoint with every decoder linear but layer 0's v_proj
    stored AWQ-quantized (that one stays bf16, as ``modules_to_not_convert``
    would leave it). Returns the fp32 weights the loader must produce."""
    t = _checkpoint(tmp_path)
    want, out = {}, {}
    for name, v in t.items():
        quant = ".layers." in name and name.endswith("_proj.weight") and name != \
            "model.layers.0.self_attn.v_proj.weight"
        if not quant:
            out[name] = v
            want[name] = v.float()
            continue
        base = name[:-len(".weight")]
        qw, qz, s = models.awq_quantize(v, group)
        out[base + ".qweight"], out[base + ".qzeros"], out[base + ".scales"] = qw, qz, s
        want[name] = models.awq_dequant(qw, qz, s, group)
    for f in tmp_path.glob("*.safetensors"):
        f.unlink()
    models.write_safetensors(str(tmp_path / "model.safetensors"), out)
    cfg = dict(HF_CFG, quantization_config={"quant_method": "awq", "bits": 4, "group_size": group,
                                            "zero_point": True, "version": "gemm",
                                            "modules_to_not_convert": ["model.layers.0.self_attn.v_proj"]})
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    return want


def test_awq_checkpoint_loads_dequantized_tp_shards(tmp_path):
    want = _awq_checkpoint(tmp_path, group=64)
    D = 128
    bf = lambda x: x.to(torch.bfloat16)  # noqa: E731
    for tp in (1, 2):
        for r in range(tp):
            _, w = models.load_llama(str(tmp_path), r, tp, "cpu")
            nq, nkv, F = 4 // tp, 2 // tp, 384 // tp
            for i in (0, 1):
                L, p = w.layers[i], f"model.layers.{i}."
                want_qkv = torch.cat([want[p + "self_attn.q_proj.weight"][r * nq * D:(r + 1) * nq * D],
                                      want[p + "self_attn.k_proj.weight"][r * nkv * D:(r + 1) * nkv * D],
                                      want[p + "self_attn.v_proj.weight"][r * nkv * D:(r + 1) * nkv * D]])
                assert torch.equal(L["qkv"], bf(want_qkv))
                assert torch.equal(L["o"], bf(want[p + "self_attn.o_proj.weight"][:, r * nq * D:(r + 1) * nq * D]))
                want_gu = torch.cat([want[p + "mlp.gate_proj.weight"][r * F:(r + 1) * F],
                                     want[p + "mlp.up_proj.weight"][r * F:(r + 1) * F]])
                assert torch.equal(L["gate_up"], bf(want_gu))
                assert torch.equal(L["down"], bf(want[p + "mlp.down_proj.weight"][:, r * F:(r + 1) * F]))
                assert all(v.dtype == torch.bfloat16 and v.is_contiguous() for v in L.values())
            V = 512 // tp
            assert torch.equal(w.embed, bf(want["model.embed_tokens.weight"][r * V:(r + 1) * V]))


def test_awq_rejects_unsupported_configs_and_misaligned_shards(tmp_path):
    loader = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models.loader")
    assert loader.awq_group_size({"quant_method": "awq", "bits": 4, "group_size": 128}) == 128
    for qc in ({"quant_method": "gptq", "bits": 4}, {"quant_method": "awq", "bits": 8},
               {"quant_method": "awq", "bits": 4, "version": "gemv"},
               {"quant_method": "awq", "bits": 4, "zero_point": False}):
        with pytest.raises(ValueError):
            loader.awq_group_size(qc)
    _awq_checkpoint(tmp_path, group=128)
    models.load_llama(str(tmp_path), 0, 1, "cpu")          # whole tensors: any group size works
    with pytest.raises(ValueError, match="group"):
        models.load_llama(str(tmp_path), 1, 2, "cpu")      # down_proj shard of 192 inputs vs group 128


def test_rope_scaling_types():
    """linear scaling divides every frequency by the factor; scalings the
    table does not implement are refused when the config is read."""
    base = ops.rope_cos_sin(8, 128, 10000.0, "cpu")
    lin = ops.rope_cos_sin(8, 128, 10000.0, "cpu", {"rope_type": "linear", "factor": 4.0})
    ang_b = torch.atan2(base[1, 64:], base[1, :64])
    ang_l = torch.atan2(lin[1, 64:], lin[1, :64])
    assert torch.allclose(ang_l, ang_b / 4.0, rtol=1e-5, atol=1e-7)
    assert torch.equal(ops.rope_cos_sin(8, 128, 10000.0, "cpu", {"rope_type": "default"}), base)
    for kind in ("yarn", "dynamic", "longrope"):
        with pytest.raises(ValueError, match="rope scaling"):
            models.config_from_hf(dict(HF_CFG, rope_scaling={"rope_type": kind, "factor": 4.0}))
        with pytest.raises(ValueError, match="rope scaling"):
            ops.rope_cos_sin(8, 128, 10000.0, "cpu", {"type": kind, "factor": 4.0})
    assert dict(models.config_from_hf(dict(HF_CFG, rope_scaling={"type": "linear", "factor": 2.0})).rope_scaling)


def test_non_silu_activation_is_refused():
    with pytest.raises(ValueError, match="activation"):
        models.config_from_hf(dict(HF_CFG, hidden_act="gelu_pytorch_tanh"))
    assert models.config_from_hf(dict(HF_CFG, hidden_act="silu")).ffn == 384


def test_awq_int4_shards_stay_packed_and_match_the_bf16_load(tmp_path):
    """``load_llama(..., int4=True)``: the decoder linears stay AWQ-packed
    (``ops.Int4Weight``), sharded like the bf16 weights; expanding a shard
    gives exactly the bf16 shard the dequantizing load produces."""
    loader = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models.loader")
    _awq_checkpoint(tmp_path, group=64)
    for tp in (1, 2):
        for r in range(tp):
            _, wq = models.load_llama(str(tmp_path), r, tp, "cpu", int4=True)
            _, wb = models.load_llama(str(tmp_path), r, tp, "cpu")
            for i in (0, 1):
                for k in ("qkv", "o", "gate_up", "down"):
                    a, b = wq.layers[i][k], wb.layers[i][k]
                    if i == 0 and k == "qkv":   # layer 0's v_proj is stored unquantized: stays bf16
                        assert isinstance(a, torch.Tensor) and torch.equal(a, b)
                        continue
                    assert isinstance(a, ops.Int4Weight) and a.shape == tuple(b.shape), (i, k)
                    dense = loader.awq_dequant(a.qweight, a.qzeros, a.scales, a.group).to(torch.bfloat16)
                    assert torch.equal(dense, b), (tp, r, i, k)


def test_quantize_random_weights_to_int4():
    cfg = models.LlamaConfig.tiny()
    w = models.LlamaWeights(cfg, 0, 1, "cpu", seed=0, full_init=True)
    ref = {k: w.layers[0][k].float().clone() for k in ("qkv", "o", "gate_up", "down")}
    models.quantize_weights_int4(w, group=128)
    loader = importlib.import_module("3080_mod_p2p_sglang_patch_b200.models.loader")
    for k, dense in ref.items():
        q = w.layers[0][k]
        assert isinstance(q, ops.Int4Weight) and q.shape == tuple(dense.shape)
        err = (loader.awq_dequant(q.qweight, q.qzeros, q.scales, q.group) - dense).abs().max().item()
        assert err <= dense.abs().max().item() / 15 + 1e-3            # within one quantization step


def test_save_and_reload_round_trip(tmp_path):
    """save_llama writes a Hugging Face checkpoint (split projections, sharded
    files) that load_llama reads back exactly, at TP 1 and 2, for the Llama,
    Qwen2 and Qwen3 variants."""
    base = models.LlamaConfig.tiny()
    for extra in ({}, {"qkv_bias": True}, {"qk_norm": True}):
        cfg = models.LlamaConfig(**{**base.__dict__, **extra, "name": "rt"})
        w = models.LlamaWeights(cfg, 0, 1, "cpu", seed=3, full_init=True)
        d = tmp_path / ("m" + "".join(extra))
        models.save_llama(str(d), cfg, w, shard_bytes=2 << 20)
        assert len(list(d.glob("*.safetensors"))) > 1                        # sharded
        cfg2, w1 = models.load_llama(str(d), 0, 1, "cpu")
        assert (cfg2.qk_norm, cfg2.qkv_bias, cfg2.hidden, cfg2.vocab) == (cfg.qk_norm, cfg.qkv_bias, 512, 4096)
        for L, L1 in zip(w.layers, w1.layers):
            assert L.keys() == L1.keys() and all(torch.equal(L[k], L1[k]) for k in L)
        assert torch.equal(w.embed, w1.embed) and torch.equal(w.lm_head, w1.lm_head)
        w2 = models.LlamaWeights(cfg, 1, 2, "cpu", seed=3, full_init=True)   # rank 1 of TP=2, drawn directly
        _, r1 = models.load_llama(str(d), 1, 2, "cpu")
        assert all(torch.equal(a[k], b[k]) for a, b in zip(w2.layers, r1.layers) for k in a)
